// tcgen05 / TMEM projection GEMM for sm_100a ("swap-AB" orientation).
//
// Every projection of the reference graph (qkv_proj, o_proj, gate_up_proj, down_proj, the tied
// lm_head; fast_dllm_relax/model/cuda.py:331-430, 704-711) is Y[tok, out] = X[tok, in] * W[out, in]^T
// with a skinny token count (8..32 rows per request at decode).  The weight matrix is therefore the
// MMA's M operand (128 weight rows per CTA = one "slab") and the tokens are the MMA's N (16..256),
// so a decode step streams each weight byte from HBM exactly once while the tensor core runs a
// legal 128 x N x 16 shape.
//
// Per CTA (4 warps): thread 0 issues TMA loads of 128x64 weight tiles and Nx64 activation tiles
// into a multi-stage shared-memory ring (128-byte swizzle, K-major); thread 32 issues
// tcgen05.mma (kind::f16, fp32 accumulate in TMEM) and frees each ring slot with tcgen05.commit;
// then all 4 warps drain the TMEM accumulator (each warp reads its 32-lane quarter with
// tcgen05.ld) into a shared fp32 tile and run the fused epilogue.  Small grids use split-K: each
// split writes an fp32 partial tile, and the last CTA to arrive (an atomic counter that resets
// itself) sums the partials in split order, so results are deterministic.
//
// Every mbarrier wait is bounded (kWaitLimitNs); on expiry the kernel records an error code,
// drains its own in-flight TMA copies (bounded), frees its TMEM and returns.
#include <algorithm>

#include "common.cuh"
#include "epilogue.cuh"
#include "kernels.h"

namespace fdllm {

template <int NT>
struct TcCfg {
  static constexpr int kA = 128 * 64 * 2;  // weight tile: 128 rows x 64 bf16
  static constexpr int kB = NT * 64 * 2;   // activation tile: NT tokens x 64 bf16
  static constexpr int kStage = kA + kB;
  static constexpr int kStages = NT <= 16 ? 10 : (NT <= 64 ? 8 : (NT <= 128 ? 6 : 4));
  static constexpr int kTmemCols = NT < 32 ? 32 : NT;
  static constexpr int kAcc = NT * 128 * 4;  // fp32 epilogue tile (reuses the ring)
  static constexpr int kPipe = kStages * kStage;
  static constexpr int kRegion = kPipe > kAcc ? kPipe : kAcc;
  static constexpr int kBarBytes = 256;
  static constexpr int kSmem = 1024 + kRegion + kBarBytes;
  static_assert(NT % 16 == 0 && NT >= 16 && NT <= 256, "MMA N must be a multiple of 16 in [16, 256]");
  static_assert(kA % 1024 == 0 && kB % 1024 == 0, "tiles must keep 1024-byte alignment");
  static_assert(kSmem <= 227 * 1024, "shared memory budget");
};

template <int NT>
__global__ void __launch_bounds__(128, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const GemmArgs g) {
  using C = TcCfg<NT>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = base;
  uint8_t* sB = base + C::kStages * C::kA;
  float* acc = reinterpret_cast<float*>(base);
  uint64_t* full = reinterpret_cast<uint64_t*>(base + C::kRegion);
  uint64_t* empty = full + C::kStages;
  uint64_t* accf = empty + C::kStages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accf + 1);
  int* last_flag = reinterpret_cast<int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int slab = blockIdx.x, tile = blockIdx.y, split = blockIdx.z;
  const int tok0 = tile * NT;
  const int kb_total = g.K / 64;
  const int kb0 = split * g.kb_per_split;
  const int kb1 = min(kb0 + g.kb_per_split, kb_total);
  const int nk = max(kb1 - kb0, 0);

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(accf, 1);
    *last_flag = 0;
    mbar_fence_init();
    tma_prefetch_map(&tmA);
    tma_prefetch_map(&tmB);
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, C::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before_sync();
  __syncthreads();
  tc_fence_after_sync();
  const uint32_t tmem = *tmem_slot;

  if (threadIdx.x == 0) {
    // ---------------- TMA producer ----------------
    const uint64_t pol_w = l2_policy_evict_first();  // weights stream through once
    const uint64_t pol_x = l2_policy_evict_last();   // activations are re-read by every slab
    int issued = 0;
    for (int i = 0; i < nk; ++i) {
      const int s = i % C::kStages;
      const uint32_t ph = (i / C::kStages) & 1u;
      if (!mbar_wait(&empty[s], ph ^ 1u)) {
        report_error(g.err, kErrTimeoutProducer);
        break;
      }
      mbar_arrive_expect_tx(&full[s], C::kStage);
      const int k0 = (kb0 + i) * 64;
      uint8_t* a = sA + s * C::kA;
      if (g.paired) {
        const int inter = g.N / 2;
        tma_load_2d(a, &tmA, &full[s], k0, slab * 64, pol_w);
        tma_load_2d(a + C::kA / 2, &tmA, &full[s], k0, inter + slab * 64, pol_w);
      } else {
        tma_load_2d(a, &tmA, &full[s], k0, slab * 128, pol_w);
      }
      tma_load_2d(sB + s * C::kB, &tmB, &full[s], k0, tok0, pol_x);
      ++issued;
    }
    // Drain: every copy this thread issued must have landed before shared memory is reused.
    for (int i = max(0, issued - C::kStages); i < issued; ++i) {
      if (!mbar_wait(&full[i % C::kStages], (i / C::kStages) & 1u)) {
        report_error(g.err, kErrTimeoutProducer);
        break;
      }
    }
  } else if (threadIdx.x == 32) {
    // ---------------- MMA issuer ----------------
    constexpr uint32_t idesc = umma_idesc_bf16(128, NT);
    for (int i = 0; i < nk; ++i) {
      const int s = i % C::kStages;
      const uint32_t ph = (i / C::kStages) & 1u;
      if (!mbar_wait(&full[s], ph)) {
        report_error(g.err, kErrTimeoutMma);
        break;
      }
      tc_fence_after_sync();
      const uint64_t ad = umma_desc_sw128(sA + s * C::kA);
      const uint64_t bd = umma_desc_sw128(sB + s * C::kB);
#pragma unroll
      for (int kk = 0; kk < 4; ++kk)
        tc_mma_bf16(tmem, ad + 2 * kk, bd + 2 * kk, idesc, (i > 0 || kk > 0) ? 1u : 0u);
      tc_commit(&empty[s]);
    }
    tc_commit(accf);
  }
  __syncwarp();

  // ---------------- epilogue: TMEM -> shared fp32 tile ----------------
  if (!mbar_wait(accf, 0)) report_error(g.err, kErrTimeoutEpilogue);
  tc_fence_after_sync();
  __syncthreads();  // the producer's drain is complete before the ring is overwritten
  const uint32_t lane_base = static_cast<uint32_t>(warp * 32) << 16;
#pragma unroll
  for (int c0 = 0; c0 < NT; c0 += 32) {
    uint32_t r[32];
    tmem_ld_32x32b_x32(tmem + lane_base + static_cast<uint32_t>(c0), r);
    tmem_ld_wait();
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (c0 + j < NT) acc[(c0 + j) * 128 + warp * 32 + lane] = __uint_as_float(r[j]);
  }
  if (nk == 0) {  // empty K range: the accumulator was never written
    for (int idx = threadIdx.x; idx < NT * 128; idx += blockDim.x) acc[idx] = 0.f;
  }
  tc_fence_before_sync();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after_sync();
    tmem_dealloc(tmem, C::kTmemCols);
  }

  // ---------------- split-K: last CTA reduces in split order ----------------
  if (g.splits > 1) {
    float* part = g.partials + (static_cast<size_t>(slab) * g.n_tok_tiles + tile) * g.splits * (NT * 128);
    for (int idx = threadIdx.x; idx < NT * 128; idx += blockDim.x)
      __stcg(&part[static_cast<size_t>(split) * NT * 128 + idx], acc[idx]);
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
      int* ctr = g.counters + slab * g.n_tok_tiles + tile;
      const int prev = atomicAdd(ctr, 1);
      const int last = (prev == g.splits - 1);
      if (last) atomicExch(ctr, 0);
      *last_flag = last;
    }
    __syncthreads();
    if (!*last_flag) return;
    __threadfence();
    for (int idx = threadIdx.x; idx < NT * 128; idx += blockDim.x) {
      float sum = 0.f;
      for (int s = 0; s < g.splits; ++s)
        sum += (s == split) ? acc[idx] : __ldcg(&part[static_cast<size_t>(s) * NT * 128 + idx]);
      acc[idx] = sum;
    }
    __syncthreads();
  }
  gemm_epilogue<bf16>(g, acc, NT, tok0, slab);
}

template <int NT>
static int launch_nt(const GemmArgs& a, const CUtensorMap& tmA, const CUtensorMap& tmB, cudaStream_t s) {
  using C = TcCfg<NT>;
  dim3 grid(a.n_slabs, a.n_tok_tiles, a.splits);
  gemm_tc_kernel<NT><<<grid, 128, C::kSmem, s>>>(tmA, tmB, a);
  count_launch();
  return cudaGetLastError();
}

template <int NT>
static cudaError_t set_attr() {
  return cudaFuncSetAttribute(gemm_tc_kernel<NT>, cudaFuncAttributeMaxDynamicSharedMemorySize, TcCfg<NT>::kSmem);
}

int init_gemm_tc_attributes() {
  cudaError_t e = set_attr<16>();
  if (e == cudaSuccess) e = set_attr<32>();
  if (e == cudaSuccess) e = set_attr<64>();
  if (e == cudaSuccess) e = set_attr<128>();
  if (e == cudaSuccess) e = set_attr<256>();
  return e;
}

int gemm_tc_smem_bytes(int nt) {
  switch (nt) {
    case 16: return TcCfg<16>::kSmem;
    case 32: return TcCfg<32>::kSmem;
    case 64: return TcCfg<64>::kSmem;
    case 128: return TcCfg<128>::kSmem;
    case 256: return TcCfg<256>::kSmem;
    default: return -1;
  }
}

int gemm_tc_stages(int nt) {
  switch (nt) {
    case 16: return TcCfg<16>::kStages;
    case 32: return TcCfg<32>::kStages;
    case 64: return TcCfg<64>::kStages;
    case 128: return TcCfg<128>::kStages;
    case 256: return TcCfg<256>::kStages;
    default: return -1;
  }
}

int launch_gemm_tc(const GemmArgs& a, const CUtensorMap& tmA, const CUtensorMap& tmB, int nt, cudaStream_t s) {
  switch (nt) {
    case 16: return launch_nt<16>(a, tmA, tmB, s);
    case 32: return launch_nt<32>(a, tmA, tmB, s);
    case 64: return launch_nt<64>(a, tmA, tmB, s);
    case 128: return launch_nt<128>(a, tmA, tmB, s);
    case 256: return launch_nt<256>(a, tmA, tmB, s);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace fdllm
