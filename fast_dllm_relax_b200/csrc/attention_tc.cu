// GQA attention on the 5th-generation tensor cores (tcgen05 / TMEM) for calls with many query
// rows: prefill (build_prefix_cache / forward_hidden under the implicit block-causal mask) and
// batched cached steps.
//
// Reference semantics: fast_dllm_relax/model/cuda.py:401-466 (dense: scores * head_dim**-0.5, the
// block-causal mask q//bs >= k//bs, softmax, P.V) and runtime.py:63-73 (cached: every query row
// attends cache rows [0, prefix_len + attend_rel)); the arithmetic is the flash-attention one of
// the reference runtime's callback (runtime.py:30-48): fp32 scores and row maxima, the
// unnormalised probabilities rounded to bf16 for the P.V product, fp32 accumulation, one division
// by the fp32 row sum at the end.
//
// One CTA per (request, query tile, KV head).  The query tile packs TQ = 128 / G tokens of the G
// query heads that share the KV head into the 128 rows of the MMA (row = token * G + head), so each
// K/V tile staged in shared memory serves the whole group.  Roles (192 threads):
//   warp 0, lane 0  TMA producer: K and V tiles of 64 keys (two 64-column boxes each, 128-byte
//                   swizzle) through a 3-stage ring, from per-request 3D tensor maps whose key
//                   extent is the attended length (keys past it read as zeros);
//   warp 1, lane 0  MMA issuer: S_j = Q K_j^T (M 128, N 64, K 128) into one of two TMEM buffers,
//                   then O_{j-1} = P_{j-1} V_{j-1} (M 128, N 128, K 64; V is the MN-major operand)
//                   into one of two more; warp 1 also owns the TMEM allocation;
//   warps 2-5       one query row per thread (the TMEM lane quarter of warp % 4): stage Q, read
//                   S_j from TMEM, mask, online softmax, write P_j (bf16, swizzled) to shared
//                   memory, and fold O_{j-1} from TMEM into fp32 registers with the rescale.
// Every wait is bounded (kWaitLimitNs): on expiry the thread records an error with its wait site
// and the CTA drains and leaves.  No thread-block cluster: every TMA load reads this GPU's
// own memory into this CTA only.
#include "common.cuh"
#include "kernels.h"

namespace fdllm {

namespace {

constexpr int kRows = 128;                    // MMA M: packed (token, head) query rows
constexpr int kKeys = 64;                     // keys per tile (S columns, P.V reduction)
constexpr int kStages = 3;                    // K/V ring depth
constexpr int kQBytes = kRows * 128 * 2;      // Q tile: two 64-column sub-tiles of 128 rows (32 KB)
constexpr int kKvHalf = kKeys * 64 * 2;       // one 64-column box of 64 keys (8 KB)
constexpr int kKvStage = 4 * kKvHalf;         // K (2 boxes) + V (2 boxes) = 32 KB
constexpr int kPBytes = kRows * kKeys * 2;    // P tile: 128 rows x 64 keys bf16 (16 KB)
constexpr int kOffQ = 0;
constexpr int kOffKv = kOffQ + kQBytes;
constexpr int kOffP = kOffKv + kStages * kKvStage;
constexpr int kOffBar = kOffP + 2 * kPBytes;
constexpr int kSmem = 1024 + kOffBar + 256;  // + alignment slack, barriers, TMEM slot
constexpr uint32_t kTmemS = 0;                // S buffers: columns [0, 64), [64, 128)
constexpr uint32_t kTmemO = 128;              // O buffers: columns [128, 256), [256, 384)
constexpr float kLog2e = 1.4426950408889634f;
static_assert(kSmem <= 227 * 1024, "shared memory budget");

struct TcBars {
  uint64_t kv_full[kStages], kv_empty[kStages];
  uint64_t q_ready;
  uint64_t s_full[2], s_free[2];
  uint64_t p_full[2], p_empty[2];
  uint64_t o_full[2], o_free[2];
  uint32_t tmem;
};
static_assert(sizeof(TcBars) <= 256, "barrier block");

// Keys the row of request-local token `tok` attends (0 for a padding row).
__device__ __forceinline__ int row_key_limit(const ReqDesc& r, int tok, int causal_block) {
  if (tok >= r.n_q) return 0;
  if (causal_block > 0) return min(r.attend_len, (tok / causal_block + 1) * causal_block);
  return r.attend_len;
}

__device__ __forceinline__ bool wait_or_report(uint64_t* bar, uint32_t parity, int* err, int site, int rows) {
  if (mbar_wait(bar, parity)) return true;
  report_wait(err, kErrTimeoutMma, site, rows, 0);
  return false;
}

// O_reg = O_reg * alpha + O_i, the P_i V_i product in TMEM buffer i & 1 (this warp's lane quarter
// at `tmem_row`); then the buffer is released to the MMA issuer.
__device__ __forceinline__ bool fold_o(float (&o)[128], int i, float alpha, TcBars* bar, uint32_t tmem_row, int lane,
                                       int* err, int rows) {
  const int ob = i & 1;
  if (!wait_or_report(&bar->o_full[ob], (i >> 1) & 1u, err, 27, rows)) return false;
  tc_fence_after_sync();
#pragma unroll
  for (int c0 = 0; c0 < 128; c0 += 32) {
    uint32_t v[32];
    tmem_ld_32x32b_x32(tmem_row + kTmemO + ob * 128 + c0, v);
    tmem_ld_wait();
#pragma unroll
    for (int c = 0; c < 32; ++c) o[c0 + c] = fmaf(o[c0 + c], alpha, __uint_as_float(v[c]));
  }
  tc_fence_before_sync();
  __syncwarp();
  if (lane == 0) mbar_arrive(&bar->o_free[ob]);
  return true;
}

}  // namespace

template <bool KT>
__global__ void __launch_bounds__(192, 1) attn_tc_kernel(const AttnArgs a, const CUtensorMap* maps, int tq) {
  // The request table, Q and this layer's K/V rows come from kernels earlier in the stream (the
  // per-call prepare kernel among them): wait for them before reading anything.
  pdl_wait();
  pdl_trigger();
  if (threadIdx.x == 0) ktrace_stamp<KT>(a.ktrace, 1);
  const int G = a.hq / a.hkv;
  const int qtile = blockIdx.x, kvh = blockIdx.y, req = blockIdx.z;
  const ReqDesc r = a.reqs[req];
  const int tok0 = qtile * tq;  // first request-local token of this tile
  if (tok0 >= r.n_q) return;    // uniform over the CTA: nothing allocated yet
  const int tok_last = min(tok0 + tq, r.n_q) - 1;
  const int key_end = row_key_limit(r, tok_last, a.causal_block);  // the last token attends the most
  const int n_tiles = (key_end + kKeys - 1) / kKeys;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = base + kOffQ;
  uint8_t* sKv = base + kOffKv;
  uint8_t* sP = base + kOffP;
  TcBars* bar = reinterpret_cast<TcBars*>(base + kOffBar);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&bar->kv_full[i], 1);
      mbar_init(&bar->kv_empty[i], 1);
    }
    mbar_init(&bar->q_ready, 4);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bar->s_full[i], 1);
      mbar_init(&bar->s_free[i], 4);
      mbar_init(&bar->p_full[i], 4);
      mbar_init(&bar->p_empty[i], 1);
      mbar_init(&bar->o_full[i], 1);
      mbar_init(&bar->o_free[i], 4);
    }
    mbar_fence_init();
  }
  if (warp == 1) {
    tmem_alloc(&bar->tmem, 512);
    tmem_relinquish();
  }
  tc_fence_before_sync();
  __syncthreads();
  tc_fence_after_sync();
  const uint32_t tmem = bar->tmem;

  const int layer_c = r.layer_stride != 0 ? a.layer : 0;  // a per-layer scratch holds one layer
  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer ----------------
      const CUtensorMap* mk = maps + 2 * req;
      const CUtensorMap* mv = mk + 1;
      tma_prefetch_map(mk);
      tma_prefetch_map(mv);
      const uint64_t pol = l2_policy_evict_last();  // K/V are re-read by the other query tiles
      int issued = 0;
      for (int j = 0; j < n_tiles; ++j) {
        const int st = j % kStages;
        if (!mbar_wait(&bar->kv_empty[st], ((j / kStages) & 1u) ^ 1u)) {
          report_wait(a.err, kErrTimeoutProducer, 21, a.m_total, 0);
          break;
        }
        mbar_arrive_expect_tx(&bar->kv_full[st], kKvStage);
        uint8_t* kvs = sKv + st * kKvStage;
        for (int h = 0; h < 2; ++h) {
          tma_load_3d(kvs + h * kKvHalf, mk, &bar->kv_full[st], kvh * a.hd + h * 64, j * kKeys, layer_c, pol);
          tma_load_3d(kvs + (2 + h) * kKvHalf, mv, &bar->kv_full[st], kvh * a.hd + h * 64, j * kKeys, layer_c, pol);
        }
        ++issued;
      }
      for (int j = max(0, issued - kStages); j < issued; ++j)  // every copy landed before leaving
        if (!mbar_wait(&bar->kv_full[j % kStages], (j / kStages) & 1u)) break;
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer ----------------
      constexpr uint32_t idesc_s = umma_idesc_bf16(kRows, kKeys);
      constexpr uint32_t idesc_o = umma_idesc_bf16_bmn(kRows, 128);
      bool ok = wait_or_report(&bar->q_ready, 0, a.err, 22, a.m_total);
      for (int j = 0; ok && j <= n_tiles; ++j) {
        if (j < n_tiles) {  // S_j = Q K_j^T
          const int st = j % kStages, sb = j & 1;
          if (!wait_or_report(&bar->kv_full[st], (j / kStages) & 1u, a.err, 23, a.m_total) ||
              !wait_or_report(&bar->s_free[sb], ((j >> 1) & 1u) ^ 1u, a.err, 24, a.m_total)) {
            ok = false;
            break;
          }
          tc_fence_after_sync();
          const uint8_t* kt = sKv + st * kKvStage;
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            const uint64_t ad = umma_desc_sw128(sQ + (kk >> 2) * (kRows * 128)) + 2 * (kk & 3);
            const uint64_t bd = umma_desc_sw128(kt + (kk >> 2) * kKvHalf) + 2 * (kk & 3);
            tc_mma_bf16(tmem + kTmemS + sb * kKeys, ad, bd, idesc_s, kk > 0 ? 1u : 0u);
          }
          tc_commit(&bar->s_full[sb]);
        }
        if (j >= 1) {  // O_i = P_i V_i, i = j - 1
          const int i = j - 1, st = i % kStages, pb = i & 1;
          if (!wait_or_report(&bar->p_full[pb], (i >> 1) & 1u, a.err, 25, a.m_total) ||
              !wait_or_report(&bar->o_free[pb], ((i >> 1) & 1u) ^ 1u, a.err, 26, a.m_total)) {
            ok = false;
            break;
          }
          tc_fence_after_sync();
          const uint8_t* vt = sKv + st * kKvStage + 2 * kKvHalf;
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            const uint64_t ad = umma_desc_sw128(sP + pb * kPBytes) + 2 * kk;
            // V rows are keys (the reduction), 64 head-dim columns per box: 16 keys per step are
            // two 8-row groups, 2048 B on; the second 64 columns sit one box (kKvHalf) further.
            const uint64_t bd = umma_desc_sw128_mn(vt + kk * 2048, kKvHalf, 1024);
            tc_mma_bf16(tmem + kTmemO + pb * 128, ad, bd, idesc_o, kk > 0 ? 1u : 0u);
          }
          tc_commit(&bar->o_full[pb]);
          tc_commit(&bar->p_empty[pb]);
          tc_commit(&bar->kv_empty[st]);
        }
      }
    }
  } else {
    // ---------------- softmax / output warps 2-5: one query row per thread ----------------
    const int q4 = warp & 3;
    const int row = q4 * 32 + lane;
    const uint32_t lane_base = static_cast<uint32_t>(q4 * 32) << 16;
    const int tl = tok0 + row / G;  // request-local token of this row
    const int head = kvh * G + row % G;
    const bool valid = row < tq * G && tl < r.n_q;
    const int lim = valid ? row_key_limit(r, tl, a.causal_block) : 0;
    const size_t qstride = static_cast<size_t>(a.hq) * a.hd;
    {  // Q row -> the two swizzled 64-column sub-tiles (zeros for padding rows)
      const uint4* src = reinterpret_cast<const uint4*>(static_cast<const bf16*>(a.q) +
                                                        static_cast<size_t>(r.q_tok0 + (valid ? tl : 0)) * qstride +
                                                        static_cast<size_t>(head) * a.hd);
      uint4 v[16];
#pragma unroll
      for (int c = 0; c < 16; ++c) v[c] = valid ? src[c] : make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
      for (int c = 0; c < 16; ++c)
        *reinterpret_cast<uint4*>(sQ + (c >> 3) * (kRows * 128) + row * 128 + (((c & 7) ^ (row & 7)) << 4)) = v[c];
    }
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) mbar_arrive(&bar->q_ready);

    const float sl2 = a.scale * kLog2e;
    float m_run = -INFINITY, l_run = 0.f, alpha_prev = 1.f;
    float o[128];
#pragma unroll
    for (int c = 0; c < 128; ++c) o[c] = 0.f;
    bool ok = true;

    for (int j = 0; j < n_tiles && ok; ++j) {
      const int sb = j & 1;
      if (!wait_or_report(&bar->s_full[sb], (j >> 1) & 1u, a.err, 28, a.m_total)) {
        ok = false;
        break;
      }
      tc_fence_after_sync();
      float s[kKeys];
      {
        uint32_t v[32];
        tmem_ld_32x32b_x32(tmem + lane_base + kTmemS + sb * kKeys, v);
        tmem_ld_wait();
#pragma unroll
        for (int c = 0; c < 32; ++c) s[c] = __uint_as_float(v[c]);
        tmem_ld_32x32b_x32(tmem + lane_base + kTmemS + sb * kKeys + 32, v);
        tmem_ld_wait();
#pragma unroll
        for (int c = 0; c < 32; ++c) s[32 + c] = __uint_as_float(v[c]);
      }
      tc_fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar->s_free[sb]);

      // mask and online softmax in the log2 domain (exp2 of scaled scores)
      const int key0 = j * kKeys;
      float mx = -INFINITY;
#pragma unroll
      for (int c = 0; c < kKeys; ++c) {
        s[c] = (key0 + c < lim) ? s[c] * sl2 : -INFINITY;
        mx = fmaxf(mx, s[c]);
      }
      const float m_new = fmaxf(m_run, mx);
      const float m_use = m_new == -INFINITY ? 0.f : m_new;
      const float alpha = exp2f(m_run - m_use);  // 0 while m_run is still -inf
      float psum = 0.f;
#pragma unroll
      for (int c = 0; c < kKeys; ++c) {
        s[c] = exp2f(s[c] - m_use);
        psum += s[c];
      }
      l_run = l_run * alpha + psum;
      m_run = m_new;

      // P_j (bf16) -> shared memory buffer j & 1, this row's 8 swizzled 16-byte chunks
      const int pb = j & 1;
      if (!wait_or_report(&bar->p_empty[pb], ((j >> 1) & 1u) ^ 1u, a.err, 29, a.m_total)) {
        ok = false;
        break;
      }
      uint8_t* prow = sP + pb * kPBytes + row * 128;
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        uint4 u;
        u.x = pack_bf16x2(s[8 * c + 0], s[8 * c + 1]);
        u.y = pack_bf16x2(s[8 * c + 2], s[8 * c + 3]);
        u.z = pack_bf16x2(s[8 * c + 4], s[8 * c + 5]);
        u.w = pack_bf16x2(s[8 * c + 6], s[8 * c + 7]);
        *reinterpret_cast<uint4*>(prow + ((c ^ (row & 7)) << 4)) = u;
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar->p_full[pb]);

      if (j >= 1 && !fold_o(o, j - 1, alpha_prev, bar, tmem + lane_base, lane, a.err, a.m_total)) {
        ok = false;
        break;
      }
      alpha_prev = alpha;
    }
    if (ok && n_tiles > 0) ok = fold_o(o, n_tiles - 1, alpha_prev, bar, tmem + lane_base, lane, a.err, a.m_total);
    if (valid) {
      const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
      uint4* dst = reinterpret_cast<uint4*>(static_cast<bf16*>(a.out) + static_cast<size_t>(r.q_tok0 + tl) * qstride +
                                            static_cast<size_t>(head) * a.hd);
#pragma unroll
      for (int c = 0; c < 16; ++c) {
        uint4 u;
        u.x = pack_bf16x2(o[8 * c + 0] * inv, o[8 * c + 1] * inv);
        u.y = pack_bf16x2(o[8 * c + 2] * inv, o[8 * c + 3] * inv);
        u.z = pack_bf16x2(o[8 * c + 4] * inv, o[8 * c + 5] * inv);
        u.w = pack_bf16x2(o[8 * c + 6] * inv, o[8 * c + 7] * inv);
        dst[c] = u;
      }
    }
  }
  __syncwarp();
  tc_fence_before_sync();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after_sync();
    tmem_dealloc(tmem, 512);
  }
  if (threadIdx.x == 0) ktrace_stamp<KT>(a.ktrace, 7);
}

int init_attention_tc_long_attributes();
int launch_attention_tc_long(const AttnArgs& a, const CUtensorMap* maps_dev, dim3 grid, int tq, int num_sms,
                             cudaStream_t s);

int init_attention_tc_attributes() {
  cudaError_t e = cudaFuncSetAttribute(attn_tc_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
  if (e == cudaSuccess) e = cudaFuncSetAttribute(attn_tc_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
  if (e == cudaSuccess) e = static_cast<cudaError_t>(init_attention_tc_long_attributes());
  return e;
}

// A grid that fits one CTA per SM (batched steps, short prefills) runs this kernel; a larger one
// runs the O-in-TMEM variant of attention_tc_long.cu at two CTAs per SM (4 x 2048-token prefill:
// 143 against 157 us a layer; 8 x 4096: 344 against 391 us; the 1024-row batched step keeps 20.4
// us here against 22.0 there, where most key tiles would rescale O in TMEM).
int launch_attention_tc(const AttnArgs& a, const CUtensorMap* maps_dev, int max_q, int num_sms, cudaStream_t s) {
  const int G = a.hq / a.hkv;
  if (a.hd != 128 || G < 1 || G > kRows / 8) return cudaErrorInvalidValue;
  const int tq = kRows / G;
  dim3 grid((max_q + tq - 1) / tq, a.hkv, a.n_reqs);
  if (a.n_splits > 1 || static_cast<long long>(grid.x) * grid.y * grid.z > num_sms)
    return launch_attention_tc_long(a, maps_dev, grid, tq, num_sms, s);  // key splits are that kernel's
  if (a.ktrace != nullptr) return launch_k(attn_tc_kernel<true>, grid, dim3(192), kSmem, s, a, maps_dev, tq);
  return launch_k(attn_tc_kernel<false>, grid, dim3(192), kSmem, s, a, maps_dev, tq);
}

}  // namespace fdllm
