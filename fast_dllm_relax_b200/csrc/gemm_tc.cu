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
// tcgen05.ld) into a shared fp32 tile and run the fused epilogue.  Small grids use split-K over a
// thread-block cluster: the partial tiles stay in shared memory and the cluster members reduce
// disjoint token rows through distributed shared memory, in split order (deterministic).
//
// Every mbarrier wait is bounded (kWaitLimitNs); on expiry the kernel records an error code,
// drains its own in-flight TMA copies (bounded), frees its TMEM and returns.
#include <algorithm>

#include "common.cuh"
#include "epilogue.cuh"
#include "kernels.h"

namespace fdllm {

// Sum of a row's n per-slab statistics in slab order with every load in flight at once (a
// load-add loop waits for each load; L2 round trips are the cost of these short phases).
// kL2: L2-only loads, for statistics that other CTAs of the same launch wrote; otherwise plain
// loads (written by an earlier launch), which one L1 line fill serves for several rows.
constexpr int kMaxRowSs = 20;  // hidden <= 2560 (the fused norms' limit)
template <bool kL2>
__device__ __forceinline__ float sum_row_ss(const float* p, int n) {
  if (n > kMaxRowSs) {
    float ss = 0.f;
    for (int j = 0; j < n; ++j) ss += kL2 ? __ldcg(p + j) : p[j];
    return ss;
  }
  float v[kMaxRowSs];
#pragma unroll
  for (int j = 0; j < kMaxRowSs; ++j) v[j] = j < n ? (kL2 ? __ldcg(p + j) : p[j]) : 0.f;
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < kMaxRowSs; ++j)
    if (j < n) ss += v[j];
  return ss;
}

template <int NT>
struct TcCfg {
  static constexpr int kA = 128 * 64 * 2;  // weight tile: 128 rows x 64 bf16
  static constexpr int kB = NT * 64 * 2;   // activation tile: NT tokens x 64 bf16
  static constexpr int kStage = kA + kB;
  // Ring depth: for NT <= 128 the CTA stays under ~110 KB of shared memory, so a CTA of the next
  // projection (launched early, prefetching its weights) can sit beside a draining one on each SM.
  // NT = 256 keeps 2 stages so that two CTAs share an SM: one's epilogue overlaps the other's
  // mainloop (their TMEM accumulators, 256 columns each, fill the SM's 512).
  static constexpr int kStages = NT <= 32 ? 5 : (NT <= 64 ? 4 : (NT <= 128 ? 3 : 2));
  static constexpr int kTmemCols = NT < 32 ? 32 : NT;
  static constexpr int kChunk = NT < 64 ? NT : 64;  // token columns drained and finished at a time
  static constexpr int kAcc = kChunk * 128 * 4;     // fp32 epilogue chunk (reuses the ring)
  static constexpr int kPipe = kStages * kStage;
  static constexpr int kRegion = kPipe > kAcc ? kPipe : kAcc;
  static constexpr int kBarBytes = 512;  // barriers, TMEM slot, fused-norm row scales (NT <= 64)
  static constexpr int kSmem = 1024 + kRegion + kBarBytes;
  static_assert(NT % 16 == 0 && NT >= 16 && NT <= 256, "MMA N must be a multiple of 16 in [16, 256]");
  static_assert(kA % 1024 == 0 && kB % 1024 == 0, "tiles must keep 1024-byte alignment");
  static_assert(kSmem <= 227 * 1024, "shared memory budget");
};

// At most 128 registers a thread (min 4 blocks): a CTA must fit beside a 192-thread attention CTA
// of up to 256 registers a thread in one SM's 64K registers for programmatic launch to overlap them.
template <int NT, bool KT>
__global__ void __launch_bounds__(128, 4)
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
  uint64_t* ready = accf + 1;  // fused-norm mode: B tile normalized in place, MMA may read it
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(ready + C::kStages);
  __shared__ __align__(16) unsigned char s_epi[5120];  // epilogue scratch; norm weights in the mainloop

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // tile-major grids (several token tiles, no split): the token tiles of one weight slab are
  // neighbouring CTAs, so the slab streams from HBM once and the other tiles read it from L2
  const int slab = g.tile_major ? blockIdx.y : blockIdx.x, tile = g.tile_major ? blockIdx.x : blockIdx.y;
  const int split = blockIdx.z;
  const int tok0 = tile * NT;
  const int kb_total = g.K / 64;
  const int kb0 = split * g.kb_per_split;
  const int kb1 = min(kb0 + g.kb_per_split, kb_total);
  const int nk = max(kb1 - kb0, 0);

  if (threadIdx.x == 0) {
    ktrace_stamp<KT>(g.ktrace, 0);
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&ready[s], 2);  // one arrival per normalizing warp
      mbar_init(&empty[s], 1);
    }
    mbar_init(accf, 1);
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
  pdl_trigger();  // the next kernel may launch now and start streaming its own weights

  if (threadIdx.x == 0) {
    // ---------------- TMA producer ----------------
    const uint64_t pol_w = l2_policy_evict_first();  // weights stream through once
    const uint64_t pol_x = l2_policy_evict_last();   // activations are re-read by every slab
    auto load_a = [&](int i) {
      const int s = i % C::kStages;
      const int k0 = (kb0 + i) * 64;
      uint8_t* a = sA + s * C::kA;
      if (g.paired) {
        const int inter = g.N / 2;
        tma_load_2d(a, &tmA, &full[s], k0, slab * 64, pol_w);
        tma_load_2d(a + C::kA / 2, &tmA, &full[s], k0, inter + slab * 64, pol_w);
      } else {
        tma_load_2d(a, &tmA, &full[s], k0, slab * 128, pol_w);
      }
    };
    auto load_b = [&](int i) {
      const int s = i % C::kStages;
      tma_load_2d(sB + s * C::kB, &tmB, &full[s], (kb0 + i) * 64, tok0, pol_x);
    };
    const int l2_ahead = (g.tune >> kGemmTuneL2Shift) & 0xff;
    auto prefetch_a = [&](int i) {  // k block i of the weights into L2
      if (i >= nk) return;
      const int k0 = (kb0 + i) * 64;
      if (g.paired) {
        tma_prefetch_l2_2d(&tmA, k0, slab * 64);
        tma_prefetch_l2_2d(&tmA, k0, g.N / 2 + slab * 64);
      } else {
        tma_prefetch_l2_2d(&tmA, k0, slab * 128);
      }
    };
    // Weights do not depend on the previous kernel: fill the ring with them before waiting for it.
    const int pre = min(nk, C::kStages);
    for (int i = 0; i < pre; ++i) {
      mbar_arrive_expect_tx(&full[i], C::kStage);  // A + B bytes; the B half lands after the wait
      load_a(i);
    }
    for (int i = pre; i < pre + l2_ahead; ++i) prefetch_a(i);  // and a few more into L2
    pdl_wait();
    ktrace_stamp<KT>(g.ktrace, 1);
    for (int i = 0; i < pre; ++i) load_b(i);
    int issued = pre;
    for (int i = pre; i < nk; ++i) {
      const int s = i % C::kStages;
      const uint32_t ph = (i / C::kStages) & 1u;
      if (!mbar_wait(&empty[s], ph ^ 1u)) {
        report_wait(g.err, kErrTimeoutProducer, 1, g.M, g.splits);
        break;
      }
      mbar_arrive_expect_tx(&full[s], C::kStage);
      load_a(i);
      load_b(i);
      prefetch_a(i + l2_ahead);
      ++issued;
    }
    // Drain: every copy this thread issued must have landed before shared memory is reused.
    for (int i = max(0, issued - C::kStages); i < issued; ++i) {
      if (!mbar_wait(&full[i % C::kStages], (i / C::kStages) & 1u)) {
        report_wait(g.err, kErrTimeoutProducer, 2, g.M, g.splits);
        break;
      }
    }
  } else if (warp >= 2 && g.norm_x != nullptr) {
    // ---------------- B normalizers (fused RMSNorm), warps 2 and 3 ----------------
    // The B tile arrives by TMA un-normalized; these warps rewrite it in place as
    // xn = T(w * T(x * rs)) (model/cuda.py:269-275) and then release it to the MMA issuer.
    // rs[t] = rsqrt(mean(x[t]^2) + eps) comes from the per-slab sums of squares that the residual
    // epilogue producing x left behind; the norm weights are staged in shared memory once.
    const int wt = threadIdx.x - 64;  // 0..63
    float* rs = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(full) + 256);  // NT (<= 64) floats
    bf16* s_w = reinterpret_cast<bf16*>(s_epi);                                      // K (<= 2560) weights
    pdl_wait();
    const int nrow = min(NT, g.M - tok0);
    for (int t = wt; t < nrow; t += 64) {
      const float ss = sum_row_ss<false>(g.norm_ss + static_cast<size_t>(tok0 + t) * g.norm_ss_ld, g.norm_ss_ld);
      rs[t] = rsqrtf(ss / static_cast<float>(g.K) + g.norm_eps);
    }
    {  // norm weights to shared memory, every load in flight at once (K <= 2560: 5 chunks a thread)
      constexpr int kWPer = 5;
      const uint4* wsrc = static_cast<const uint4*>(g.norm_w);
      uint4 wr[kWPer];
#pragma unroll
      for (int i = 0; i < kWPer; ++i)
        if (wt + 64 * i < g.K / 8) wr[i] = wsrc[wt + 64 * i];
#pragma unroll
      for (int i = 0; i < kWPer; ++i)
        if (wt + 64 * i < g.K / 8) reinterpret_cast<uint4*>(s_w)[wt + 64 * i] = wr[i];
    }
    asm volatile("bar.sync 1, 64;" ::: "memory");  // the two normalizing warps only
    const int cc = wt & 7;  // 16-byte chunk (8 columns) of the 64-column k-block this thread handles
    for (int i = 0; i < nk; ++i) {
      const int s = i % C::kStages;
      const uint32_t ph = (i / C::kStages) & 1u;
      if (!mbar_wait(&full[s], ph)) {
        report_wait(g.err, kErrTimeoutMma, 3, g.M, g.splits);
        break;
      }
      const uint4 wu = reinterpret_cast<const uint4*>(s_w)[(kb0 + i) * 8 + cc];
      const bf16* w8 = reinterpret_cast<const bf16*>(&wu);
      uint8_t* bt = sB + s * C::kB;
      for (int t = wt >> 3; t < nrow; t += 8) {
        uint4* p = reinterpret_cast<uint4*>(bt + (t >> 3) * 1024 + (t & 7) * 128 + ((cc ^ (t & 7)) << 4));
        uint4 u = *p;
        __nv_bfloat162* x2 = reinterpret_cast<__nv_bfloat162*>(&u);
        const float r = rs[t];
#pragma unroll
        for (int v = 0; v < 4; ++v) {
          const float2 xf = __bfloat1622float2(x2[v]);
          const float2 xn = round2_bf16(xf.x * r, xf.y * r);
          x2[v] = __floats2bfloat162_rn(__bfloat162float(w8[2 * v]) * xn.x, __bfloat162float(w8[2 * v + 1]) * xn.y);
        }
        *p = u;
      }
      fence_proxy_async_smem();
      __syncwarp();
      if ((wt & 31) == 0) mbar_arrive(&ready[s]);
    }
  } else if (threadIdx.x == 32) {
    // ---------------- MMA issuer ----------------
    constexpr uint32_t idesc = umma_idesc_bf16(128, NT);
    for (int i = 0; i < nk; ++i) {
      const int s = i % C::kStages;
      const uint32_t ph = (i / C::kStages) & 1u;
      if (!mbar_wait(g.norm_x ? &ready[s] : &full[s], ph)) {
        report_wait(g.err, kErrTimeoutMma, 4, g.M, g.splits);
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
  pdl_wait();  // every thread below reads or writes memory the previous kernel may still touch
  // The accumulator is finished kChunk token columns at a time (the shared fp32 chunk reuses the
  // ring).  Split-K: the g.splits CTAs of one (slab, token tile) form one cluster; each keeps its
  // fp32 partial chunk in shared memory, member r sums rows [r*kChunk/S, (r+1)*kChunk/S) of the
  // chunk over all members through distributed shared memory in rank (= split) order --
  // deterministic, no global round trip -- and runs the epilogue for those rows only.
  const uint32_t S = static_cast<uint32_t>(g.splits > 1 ? g.splits : 1);
  const uint32_t rank = g.splits > 1 ? cluster_ctarank() : 0u;
  const int lr0 = static_cast<int>(rank * C::kChunk / S), lr1 = static_cast<int>((rank + 1) * C::kChunk / S);
  // One chunk (NT <= 64): this thread's epilogue inputs are loaded before the accumulator is ready.
  EpiPre<bf16> pre;
  if (NT <= 64 && (g.tune & kGemmTunePrefetch))
    epi_prefetch<bf16>(g, tok0, slab, S > 1 ? lr0 : 0, S > 1 ? lr1 : NT, threadIdx.x, blockDim.x, pre);
  // qkv without a prefetched chunk (large calls): warps 2-3, idle while the main loop runs, build the
  // tile's per-token destinations and prefetch its K / V cache rows into L2 (the barrier after the
  // accumulator wait publishes them).  Not with the fused norm, whose weights s_epi holds.
  const bool early_dest = g.epi.kind == kEpiQkvRope && g.norm_x == nullptr && pre.n == 0;
  if (early_dest && warp >= 2)
    qkv_dest_setup<bf16>(g, tok0, 0, NT, s_epi, static_cast<int>(threadIdx.x) - 64, static_cast<int>(blockDim.x) - 64,
                         true);
  if (!mbar_wait(accf, 0)) report_wait(g.err, kErrTimeoutEpilogue, 5, g.M, g.splits);
  if (threadIdx.x == 0) ktrace_stamp<KT>(g.ktrace, 2);
  tc_fence_after_sync();
  __syncthreads();  // the producer's drain is complete before the ring is overwritten
  const uint32_t lane_base = static_cast<uint32_t>(warp * 32) << 16;
  for (int ch = 0; ch < NT / C::kChunk; ++ch) {
    const int cb = ch * C::kChunk;
    if (ch > 0) {  // the previous chunk is consumed (its epilogue, and the peers' reads of it)
      if (S > 1) {
        cluster_sync();
      } else {
        __syncthreads();
      }
    }
#pragma unroll
    for (int c0 = 0; c0 < C::kChunk; c0 += 32) {
      uint32_t r[32];
      tmem_ld_32x32b_x32(tmem + lane_base + static_cast<uint32_t>(cb + c0), r);
      tmem_ld_wait();
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (c0 + j < C::kChunk) acc[(c0 + j) * 128 + warp * 32 + lane] = __uint_as_float(r[j]);
    }
    if (nk == 0) {  // empty K range: the accumulator was never written
      for (int idx = threadIdx.x; idx < C::kChunk * 128; idx += blockDim.x) acc[idx] = 0.f;
    }
    if (ch == NT / C::kChunk - 1) {  // every column drained: free TMEM
      tc_fence_before_sync();
      __syncthreads();
      if (threadIdx.x == 0) ktrace_stamp<KT>(g.ktrace, 3);
      if (warp == 0) {
        tc_fence_after_sync();
        tmem_dealloc(tmem, C::kTmemCols);
        if (lane == 0) ktrace_stamp<KT>(g.ktrace, 8);
      }
    } else {
      __syncthreads();
    }
    if (S > 1) {
      constexpr int kMaxS = 16;
      cluster_sync();  // every member's partial chunk is complete
      const uint32_t acc_addr = smem_addr(acc);
      float4* acc4 = reinterpret_cast<float4*>(acc);
      for (int c = lr0 * 32 + threadIdx.x; c < lr1 * 32; c += blockDim.x) {
        float4 v[kMaxS];
#pragma unroll
        for (int m = 0; m < kMaxS; ++m)
          v[m] = (static_cast<uint32_t>(m) < S) ? ld_dsmem_f4(map_shared_rank(acc_addr + c * 16, m))
                                                : make_float4(0.f, 0.f, 0.f, 0.f);
        float4 sum = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int m = 0; m < kMaxS; ++m) {
          if (static_cast<uint32_t>(m) < S) {
            sum.x += v[m].x;
            sum.y += v[m].y;
            sum.z += v[m].z;
            sum.w += v[m].w;
          }
        }
        acc4[c] = sum;  // only this member reads or writes its own rows from here on
      }
      __syncthreads();
      if (threadIdx.x == 0 && ch == NT / C::kChunk - 1) ktrace_stamp<KT>(g.ktrace, 4);
      // Last chunk: this member's reads of its peers' partials are done.  Arrive now and wait
      // only before leaving, so the closing barrier overlaps the epilogue.
      if (ch == NT / C::kChunk - 1) cluster_arrive();
    }
    // acc holds token columns [cb, cb + kChunk); the epilogue indexes it as the whole tile
    gemm_epilogue<bf16>(g, acc - static_cast<size_t>(cb) * 128, NT, tok0, slab, S > 1 ? cb + lr0 : cb,
                        S > 1 ? cb + lr1 : cb + C::kChunk, s_epi, static_cast<int>(threadIdx.x),
                        static_cast<int>(blockDim.x), 0, NT <= 64 ? &pre : nullptr, early_dest ? 0 : -1,
                        early_dest ? 0 : -1);
  }
  if (threadIdx.x == 0) ktrace_stamp<KT>(g.ktrace, 5);

  if (S > 1) cluster_wait();  // no member leaves while another may still read its shared memory
  if (threadIdx.x == 0) ktrace_stamp<KT>(g.ktrace, 7);
}

// ---- persistent variant for large token counts (prefill, batched serving) --------------------------
// One CTA per SM walks its tiles (slab-major: neighbouring CTAs share a weight slab in L2) with
// three roles: warp 0 issues TMA for every tile's k blocks through a 4-stage ring, warp 1 issues
// tcgen05.mma into one of two TMEM accumulators (2 x 256 columns: the whole TMEM), warps 2-9 drain
// the other accumulator 32 token columns at a time through shared memory into the fused epilogue
// (two warps per TMEM lane quarter, 16 columns each).
// The epilogue of tile i therefore overlaps the mainloop of tile i + 1.
// The lm_head's confidence epilogues (g.conf_t) swap the operands: 128 tokens are the MMA's M and a
// pair of weight slabs its N = 256, so TMEM lane = token and each epilogue thread reduces one
// token's 128 logits of one slab without crossing lanes.
template <int NT>
struct PCfg {
  static_assert(NT == 96 || NT == 128 || NT == 256, "persistent token tiles: 96, 128 or 256");
  static constexpr int kStages = NT == 256 ? 4 : 6;
  static constexpr uint32_t kTmemCols = 2 * NT <= 256 ? 256 : 512;  // a power of two >= 2 NT
  static constexpr uint32_t kAccStride = kTmemCols / 2;                // accumulator 1's first column
  static constexpr int kStage = 128 * 64 * 2 + NT * 64 * 2;  // A + B of one k block
  static constexpr int kChunk = 32;
  static constexpr int kSmem = 1024 + kStages * kStage + kChunk * 128 * 4 + 256;
  static_assert(kSmem <= 227 * 1024 - 5120, "shared memory budget");
};
constexpr int kPEpi = 256;  // epilogue threads (warps 2-9)

// Confidence / log-softmax-gather partial of one token and one 128-row vocabulary slab
// (model/metal.py:316-374), from the token's 128 fp32 logits in TMEM columns [taddr, taddr + 128)
// of this thread's lane (the tokens-on-M tile).  Same result, bit for bit, as the shared-memory
// path of gemm_epilogue (kEpiConf / kEpiLseGather), whose warp gives lane l the values f = l,
// l + 32, l + 64, l + 96: the logits are rounded to bf16; the maximum and its first index; then
// exp(v - max) summed into 32 four-term column sums in that order, which are added in lane 0's
// xor-butterfly tree (offsets 16, 8, 4, 2, 1).  kFull: all 128 rows are below N.
template <bool kFull>
__device__ __forceinline__ void conf_slab_from_tmem(const GemmArgs& g, uint32_t taddr, int tok, int slab, int tg) {
  const int f0 = slab * 128;
  const int nv = kFull ? 128 : min(128, g.N - f0);
  float best = -INFINITY, tv = 0.f;
  int best_i = 0x7fffffff;
  // 16 columns per TMEM load keeps the live set small (the column sums plus one load)
  uint32_t r[16];
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    tmem_ld_32x32b_x16(taddr + c * 16, r);
    tmem_ld_wait();
    float v[16];
#pragma unroll
    for (int j = 0; j < 16; j += 2) {
      const float2 p = round2_bf16(__uint_as_float(r[j]), __uint_as_float(r[j + 1]));
      v[j] = (kFull || c * 16 + j < nv) ? p.x : __int_as_float(0x7fc00000);  // rows >= N: NaN, never chosen
      v[j + 1] = (kFull || c * 16 + j + 1 < nv) ? p.y : __int_as_float(0x7fc00000);
      if (c * 16 + j == tg) tv = p.x;
      if (c * 16 + j + 1 == tg) tv = p.y;
    }
    float m = v[0];
#pragma unroll
    for (int j = 1; j < 16; ++j) m = fmaxf(m, v[j]);  // NaN-ignoring; -inf only if no value is larger
    int mi = 0x7fffffff;
#pragma unroll
    for (int j = 15; j >= 0; --j)
      if (v[j] == m) mi = f0 + c * 16 + j;  // first index of the group's maximum
    // groups ascend, so an equal later maximum keeps the earlier index; an all-NaN group has none
    if (m > best || (best_i == 0x7fffffff && m == best)) {
      best = m;
      best_i = mi;
    }
  }
  float s[32];
#pragma unroll
  for (int j = 0; j < 32; ++j) s[j] = 0.f;
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    tmem_ld_32x32b_x16(taddr + c * 16, r);
    tmem_ld_wait();
#pragma unroll
    for (int j = 0; j < 16; j += 2) {
      const float2 p = round2_bf16(__uint_as_float(r[j]), __uint_as_float(r[j + 1]));
      const int f = c * 16 + j;  // column sum f % 32
      if (kFull || f < nv) s[f & 31] += expf(p.x - best);
      if (kFull || f + 1 < nv) s[(f + 1) & 31] += expf(p.y - best);
    }
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1)
#pragma unroll
    for (int j = 0; j < off; ++j) s[j] += s[j + off];
  if (tok < g.M)
    *reinterpret_cast<float4*>(g.epi.part + (static_cast<size_t>(tok) * g.n_slabs + slab) * 4) =
        make_float4(best, __int_as_float(best_i), s[0], tv);
}

template <int NT, bool KT, bool TR = false>
__global__ void __launch_bounds__(64 + kPEpi, 1)
    gemm_tc_persist_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                           const GemmArgs g) {
  constexpr int kPNT = NT;
  constexpr int kPStages = PCfg<NT>::kStages;
  constexpr int kPStage = PCfg<NT>::kStage;
  constexpr int kPChunk = PCfg<NT>::kChunk;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* ring = base;  // stage s: A at s * kPStage, B at s * kPStage + 16 KB
  float* acc = reinterpret_cast<float*>(base + kPStages * kPStage);
  uint64_t* full = reinterpret_cast<uint64_t*>(base + kPStages * kPStage + kPChunk * 128 * 4);
  uint64_t* empty = full + kPStages;
  uint64_t* tfull = empty + kPStages;  // [2] accumulator complete
  uint64_t* tempty = tfull + 2;        // [2] accumulator drained
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  __shared__ __align__(16) unsigned char s_epi[5120];

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // tokens-on-M tiles (g.conf_t): A = 128 token rows, B = two weight slabs (256 rows), so a tile is
  // (slab pair, 128-token tile); the ring stage has the same 16 + 32 KB split as NT = 256
  static_assert(!TR || NT == 256, "tokens-on-M tiles use the 256-column stage");
  constexpr bool tr = TR;
  const int n_wt = tr ? (g.n_slabs + 1) / 2 : g.n_slabs;  // weight tiles
  const int tok_h = tr ? 128 : kPNT;                      // token rows per tile
  const int n_tiles = n_wt * g.n_tok_tiles;
  const int nk = g.K / 64;
  const int S = g.splits > 1 ? g.splits : 1;  // split-K: unit = (tile, split), neighbours split one tile
  const int n_units = n_tiles * S;
  auto kb_range = [&](int u, int* kb0, int* kb1) {
    const int sp = u % S;
    *kb0 = sp * g.kb_per_split;
    *kb1 = min(nk, *kb0 + g.kb_per_split);
  };
  if (threadIdx.x == 0) {
    for (int i = 0; i < kPStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], 1);
    }
    mbar_fence_init();
    tma_prefetch_map(&tmA);
    tma_prefetch_map(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, PCfg<NT>::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before_sync();
  __syncthreads();
  tc_fence_after_sync();
  const uint32_t tmem = *tmem_slot;
  pdl_trigger();

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer ----------------
      const uint64_t pol_w = l2_policy_evict_first();
      const uint64_t pol_x = l2_policy_evict_last();
      // Weight k blocks this far beyond the one being loaded are prefetched into L2: the CTAs that
      // share a slab walk it in step, so without it each k block arrives at HBM latency and only
      // the shared-memory ring covers that latency.
      const int l2a = (g.tune >> kGemmTunePersistL2Shift) & 0xff;
      auto prefetch_a = [&](int kb, int slab) {
        if (tr) {
          tma_prefetch_l2_2d(&tmA, kb * 64, slab * 256);
          tma_prefetch_l2_2d(&tmA, kb * 64, slab * 256 + 128);
        } else if (g.paired) {
          tma_prefetch_l2_2d(&tmA, kb * 64, slab * 64);
          tma_prefetch_l2_2d(&tmA, kb * 64, g.N / 2 + slab * 64);
        } else {
          tma_prefetch_l2_2d(&tmA, kb * 64, slab * 128);
        }
      };
      pdl_wait();
      ktrace_stamp<KT>(g.ktrace, 1);
      uint32_t it = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < n_units && ok; u += gridDim.x) {
        const int t = u / S;
        const int slab = t / g.n_tok_tiles, tok0 = (t % g.n_tok_tiles) * tok_h;
        int kb0, kb1;
        kb_range(u, &kb0, &kb1);
        for (int kb = kb0; kb < min(kb1, kb0 + l2a); ++kb) prefetch_a(kb, slab);
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
          if (kb + l2a < kb1) prefetch_a(kb + l2a, slab);
          const int s = it % kPStages;
          if (!mbar_wait(&empty[s], ((it / kPStages) & 1u) ^ 1u)) {
            report_wait(g.err, kErrTimeoutProducer, 11, g.M, g.splits);
            ok = false;
            break;
          }
          uint8_t* a = ring + s * kPStage;
          if (tr) {
            // an odd slab count leaves the last pair one slab: its second half is not loaded, and
            // the accumulator columns it feeds are never read
            const bool second = 2 * slab + 1 < g.n_slabs;
            mbar_arrive_expect_tx(&full[s], second ? kPStage : kPStage - 16384);
            tma_load_2d(a, &tmB, &full[s], kb * 64, tok0, pol_x);
            tma_load_2d(a + 16384, &tmA, &full[s], kb * 64, slab * 256, pol_w);
            if (second) tma_load_2d(a + 32768, &tmA, &full[s], kb * 64, slab * 256 + 128, pol_w);
            continue;
          }
          mbar_arrive_expect_tx(&full[s], kPStage);
          if (g.paired) {
            tma_load_2d(a, &tmA, &full[s], kb * 64, slab * 64, pol_w);
            tma_load_2d(a + 8192, &tmA, &full[s], kb * 64, g.N / 2 + slab * 64, pol_w);
          } else {
            tma_load_2d(a, &tmA, &full[s], kb * 64, slab * 128, pol_w);
          }
          tma_load_2d(a + 16384, &tmB, &full[s], kb * 64, tok0, pol_x);  // NT token rows
        }
      }
      for (uint32_t i = it > static_cast<uint32_t>(kPStages) ? it - kPStages : 0u; i < it; ++i)
        if (!mbar_wait(&full[i % kPStages], (i / kPStages) & 1u)) break;
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer ----------------
      constexpr uint32_t idesc = umma_idesc_bf16(128, kPNT);
      uint32_t it = 0, ti = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < n_units && ok; u += gridDim.x, ++ti) {
        const uint32_t buf = ti & 1u;
        int kb0, kb1;
        kb_range(u, &kb0, &kb1);
        if (!mbar_wait(&tempty[buf], ((ti >> 1) & 1u) ^ 1u)) {  // the epilogue released this accumulator
          report_wait(g.err, kErrTimeoutMma, 13, g.M, g.splits);
          break;
        }
        tc_fence_after_sync();
        const uint32_t d = tmem + buf * PCfg<NT>::kAccStride;
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
          const int s = it % kPStages;
          if (!mbar_wait(&full[s], (it / kPStages) & 1u)) {
            report_wait(g.err, kErrTimeoutMma, 14, g.M, g.splits);
            ok = false;
            break;
          }
          tc_fence_after_sync();
          const uint64_t ad = umma_desc_sw128(ring + s * kPStage);
          const uint64_t bd = umma_desc_sw128(ring + s * kPStage + 16384);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) tc_mma_bf16(d, ad + 2 * kk, bd + 2 * kk, idesc, (kb > kb0 || kk > 0) ? 1u : 0u);
          tc_commit(&empty[s]);
        }
        if (ok) tc_commit(&tfull[buf]);
      }
    }
  } else {
    // ---------------- epilogue warps 2-9 ----------------
    const int tid = threadIdx.x - 64;
    const int q = warp & 3;             // TMEM lane quarter this warp may access
    const int half = (warp - 2) >> 2;   // which 16 of the chunk's 32 columns it drains
    pdl_wait();
    __shared__ int s_last;
    uint32_t ti = 0;
    for (int u = blockIdx.x; u < n_units; u += gridDim.x, ++ti) {
      const int t = u / S, sp = u % S;
      const int slab = t / g.n_tok_tiles, tok0 = (t % g.n_tok_tiles) * tok_h;
      const uint32_t buf = ti & 1u;
      if (!mbar_wait(&tfull[buf], (ti >> 1) & 1u)) {
        report_wait(g.err, kErrTimeoutEpilogue, 15, g.M, g.splits);
        break;
      }
      tc_fence_after_sync();
      if (tr) {
        // tokens-on-M tile: lane quarter q holds tokens tok0 + 32 q + lane, and `half` picks the
        // pair's slab (accumulator columns [128 half, 128 half + 128))
        const int sl = 2 * slab + half;
        if (sl < g.n_slabs) {  // warp-uniform
          const int tok = tok0 + q * 32 + lane;
          const int tg = (g.epi.kind == kEpiLseGather && tok < g.M) ? g.epi.target[tok] - sl * 128 : -1;
          const uint32_t taddr = tmem + buf * PCfg<NT>::kAccStride + (static_cast<uint32_t>(q * 32) << 16) +
                                 static_cast<uint32_t>(half * 128);
          if ((sl + 1) * 128 <= g.N)
            conf_slab_from_tmem<true>(g, taddr, tok, sl, tg);
          else
            conf_slab_from_tmem<false>(g, taddr, tok, sl, tg);
        }
        tc_fence_before_sync();
        named_sync(1, kPEpi);
        if (tid == 0) mbar_arrive(&tempty[buf]);  // the accumulator is free for the tile after next
        continue;
      }
      // split-K: this unit's fp32 partial tile [NT][128] (tile t, split sp)
      float4* mine = S > 1 ? reinterpret_cast<float4*>(g.ppart + (static_cast<size_t>(t) * S + sp) * kPNT * 128) : nullptr;
      for (int cb = 0; cb < kPNT && tok0 + cb < g.M; cb += kPChunk) {
        uint32_t r[16];
        tmem_ld_32x32b_x16(tmem + buf * PCfg<NT>::kAccStride + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(cb + half * 16),
                           r);
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 16; ++j) acc[(half * 16 + j) * 128 + q * 32 + lane] = __uint_as_float(r[j]);
        named_sync(1, kPEpi);
        if (S > 1) {  // publish this split's chunk; the tile's last split finishes the tile
          const float4* a4 = reinterpret_cast<const float4*>(acc);
          for (int i = tid; i < kPChunk * 32; i += kPEpi) __stcg(mine + cb * 32 + i, a4[i]);
        } else {  // the tile's per-token destinations are built with its first chunk
          gemm_epilogue<bf16>(g, acc - static_cast<size_t>(cb) * 128, kPNT, tok0, slab, cb, cb + kPChunk, s_epi, tid,
                              kPEpi, 1, nullptr, 0, cb == 0 ? kPNT : 0);
        }
        named_sync(1, kPEpi);
      }
      tc_fence_before_sync();
      named_sync(1, kPEpi);
      if (tid == 0) mbar_arrive(&tempty[buf]);  // the accumulator is free for the tile after next
      if (S > 1) {
        // pmerge_all (each CTA holds at most one unit, so a tile's S splits run at the same time):
        // every split waits for all S partials and merges every S-th 32-column chunk of the tile.
        // Otherwise the tile's last split merges the whole tile.
        if (tid == 0) {
          __threadfence();
          const unsigned old = atomicAdd(g.pctr + t, 1u);
          if (g.pmerge_all) {
            s_last = wait_count_geq(g.pctr + t, static_cast<unsigned>(S)) ? 1 : 0;
            if (!s_last) report_wait(g.err, kErrTimeoutEpilogue, 16, g.M, g.splits);
          } else {
            s_last = (old == static_cast<unsigned>(S) - 1u) ? 1 : 0;
            if (s_last) {
              __threadfence();
              g.pctr[t] = 0u;  // the last arrival: nobody else touches this counter in this launch
            }
          }
        }
        named_sync(1, kPEpi);
        if (s_last) {  // sum the S partials in split order (deterministic), then the epilogue
          const float4* p0 = reinterpret_cast<const float4*>(g.ppart + static_cast<size_t>(t) * S * kPNT * 128);
          for (int cb = g.pmerge_all ? sp * kPChunk : 0; cb < kPNT && tok0 + cb < g.M;
               cb += g.pmerge_all ? S * kPChunk : kPChunk) {
            float4* a4 = reinterpret_cast<float4*>(acc);
            for (int i = tid; i < kPChunk * 32; i += kPEpi) {
              float4 v[4];
#pragma unroll
              for (int j = 0; j < 4; ++j)
                v[j] = j < S ? __ldcg(p0 + static_cast<size_t>(j) * kPNT * 32 + cb * 32 + i) : make_float4(0.f, 0.f, 0.f, 0.f);
              float4 sum = v[0];
#pragma unroll
              for (int j = 1; j < 4; ++j) {
                if (j < S) {
                  sum.x += v[j].x;
                  sum.y += v[j].y;
                  sum.z += v[j].z;
                  sum.w += v[j].w;
                }
              }
              a4[i] = sum;
            }
            named_sync(1, kPEpi);
            gemm_epilogue<bf16>(g, acc - static_cast<size_t>(cb) * 128, kPNT, tok0, slab, cb, cb + kPChunk, s_epi, tid,
                                kPEpi, 1);
            named_sync(1, kPEpi);
          }
        }
        if (g.pmerge_all && tid == 0) {  // the tile's last split to finish resets both counters
          unsigned* done = g.pctr + n_tiles;
          if (atomicAdd(done + t, 1u) == static_cast<unsigned>(S) - 1u) {
            g.pctr[t] = 0u;
            done[t] = 0u;
          }
        }
      }
    }
  }
  __syncwarp();
  tc_fence_before_sync();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after_sync();
    tmem_dealloc(tmem, PCfg<NT>::kTmemCols);
  }
  if (threadIdx.x == 0) ktrace_stamp<KT>(g.ktrace, 7);
}

int launch_gemm_tc_persist(const GemmArgs& a, const CUtensorMap& tmA, const CUtensorMap& tmB, int nt, int grid,
                           cudaStream_t s) {
  const bool kt = a.ktrace != nullptr;
  if (nt == 256 && a.conf_t)
    return kt ? launch_k(gemm_tc_persist_kernel<256, true, true>, dim3(grid), dim3(64 + kPEpi), PCfg<256>::kSmem, s, tmA, tmB, a)
              : launch_k(gemm_tc_persist_kernel<256, false, true>, dim3(grid), dim3(64 + kPEpi), PCfg<256>::kSmem, s, tmA, tmB, a);
  if (nt == 256)
    return kt ? launch_k(gemm_tc_persist_kernel<256, true>, dim3(grid), dim3(64 + kPEpi), PCfg<256>::kSmem, s, tmA, tmB, a)
              : launch_k(gemm_tc_persist_kernel<256, false>, dim3(grid), dim3(64 + kPEpi), PCfg<256>::kSmem, s, tmA, tmB, a);
  if (nt == 128)
    return kt ? launch_k(gemm_tc_persist_kernel<128, true>, dim3(grid), dim3(64 + kPEpi), PCfg<128>::kSmem, s, tmA, tmB, a)
              : launch_k(gemm_tc_persist_kernel<128, false>, dim3(grid), dim3(64 + kPEpi), PCfg<128>::kSmem, s, tmA, tmB, a);
  if (nt == 96)
    return kt ? launch_k(gemm_tc_persist_kernel<96, true>, dim3(grid), dim3(64 + kPEpi), PCfg<96>::kSmem, s, tmA, tmB, a)
              : launch_k(gemm_tc_persist_kernel<96, false>, dim3(grid), dim3(64 + kPEpi), PCfg<96>::kSmem, s, tmA, tmB, a);
  return cudaErrorInvalidValue;
}

template <int NT>
static int launch_nt(const GemmArgs& a, const CUtensorMap& tmA, const CUtensorMap& tmB, cudaStream_t s) {
  using C = TcCfg<NT>;
  dim3 grid = a.tile_major ? dim3(a.n_tok_tiles, a.n_slabs, a.splits) : dim3(a.n_slabs, a.n_tok_tiles, a.splits);
  if (a.ktrace != nullptr) return launch_kc(gemm_tc_kernel<NT, true>, grid, dim3(128), C::kSmem, s, a.splits, tmA, tmB, a);
  return launch_kc(gemm_tc_kernel<NT, false>, grid, dim3(128), C::kSmem, s, a.splits, tmA, tmB, a);
}

template <int NT, bool KT>
static cudaError_t set_attr1() {
  cudaError_t e = cudaFuncSetAttribute(gemm_tc_kernel<NT, KT>, cudaFuncAttributeMaxDynamicSharedMemorySize, TcCfg<NT>::kSmem);
  // split-K clusters of up to 16 CTAs (above the portable 8)
  if (e == cudaSuccess) e = cudaFuncSetAttribute(gemm_tc_kernel<NT, KT>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
  return e;
}

template <int NT>
static cudaError_t set_attr() {
  cudaError_t e = set_attr1<NT, false>();
  if (e == cudaSuccess) e = set_attr1<NT, true>();
  return e;
}

int init_gemm_tc_attributes() {
  cudaError_t e = cudaFuncSetAttribute(gemm_tc_persist_kernel<256, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       PCfg<256>::kSmem);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(gemm_tc_persist_kernel<256, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, PCfg<256>::kSmem);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(gemm_tc_persist_kernel<256, false, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, PCfg<256>::kSmem);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(gemm_tc_persist_kernel<256, true, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, PCfg<256>::kSmem);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(gemm_tc_persist_kernel<128, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, PCfg<128>::kSmem);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(gemm_tc_persist_kernel<128, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, PCfg<128>::kSmem);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(gemm_tc_persist_kernel<96, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, PCfg<96>::kSmem);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(gemm_tc_persist_kernel<96, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, PCfg<96>::kSmem);
  if (e == cudaSuccess) e = set_attr<16>();
  if (e == cudaSuccess) e = set_attr<32>();
  if (e == cudaSuccess) e = set_attr<64>();
  if (e == cudaSuccess) e = set_attr<128>();
  if (e == cudaSuccess) e = set_attr<256>();
  return e;
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
