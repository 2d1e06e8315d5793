// GQA attention on the 5th-generation tensor cores (tcgen05 / TMEM) for launches of more CTAs than
// SMs (long prefills): the variant of attention_tc.cu that keeps O in TMEM, so that two CTAs share
// an SM and one's softmax chain overlaps the other's.  Launched by launch_attention_tc.
//
// Reference semantics: fast_dllm_relax/model/cuda.py:401-466 (dense: scores * head_dim**-0.5, the
// block-causal mask q//bs >= k//bs, softmax, P.V) and runtime.py:63-73 (cached: every query row
// attends cache rows [0, prefix_len + attend_rel)); the arithmetic is the flash-attention one of
// the reference runtime's callback (runtime.py:30-48): fp32 scores and row maxima, the
// unnormalised probabilities rounded to bf16 for the P.V product, fp32 accumulation, one division
// by the fp32 row sum at the end.
//
// One CTA per (request, query tile, KV head), two CTAs per SM.  The query tile packs TQ = 128 / G
// tokens of the G query heads that share the KV head into the 128 rows of the MMA (row = token *
// G + head), so each K/V tile staged in shared memory serves the whole group.  Roles (192 threads):
//   warp 0, lane 0  TMA producer: K and V tiles of 64 keys (two 64-column boxes each, 128-byte
//                   swizzle) through a 2-stage ring, from per-request 3D tensor maps whose key
//                   extent is the attended length (keys past it read as zeros);
//   warp 1, lane 0  MMA issuer: S_j = Q K_j^T (M 128, N 64, K 128) into one of two TMEM buffers,
//                   then O += P_{j-1} V_{j-1} (M 128, N 128, K 64; V is the MN-major operand) into
//                   the one TMEM accumulator; warp 1 also owns the TMEM allocation (256 columns);
//   warps 2-5       one query row per thread (the TMEM lane quarter of warp % 4): stage Q, read
//                   S_j from TMEM, mask, online softmax, write P_j (bf16, swizzled) over K_j in the
//                   ring (S_j is done with it), and at the end read O once and divide by the row sum.
// O stays in TMEM.  When a row's maximum grows, the warp waits for the previous P.V to land and
// rescales its rows of O in TMEM by 2^(old - new) before P_j V_j adds, so the probabilities are
// the flash-attention ones (each row's running maximum).  With AttnArgs::lazy_log2 = x > 0 the
// base moves only when the maximum outgrows it by more than 2^x (the probabilities stay below 2^x
// in between, and far fewer tiles rescale): equal in exact arithmetic, rounded differently.
// Every wait is bounded (kWaitLimitNs): on expiry the thread records an error with its wait site
// and the CTA drains and leaves.  No thread-block cluster: every TMA load reads this GPU's
// own memory into this CTA only.
#include "common.cuh"
#include "kernels.h"

namespace fdllm {

namespace {

constexpr int kRows = 128;                    // MMA M: packed (token, head) query rows
constexpr int kKeys = 64;                     // keys per tile (S columns, P.V reduction)
constexpr int kMaxStages = 3;                 // K/V ring depth (P_j is written over K_j): 2 or 3
constexpr int kQBytes = kRows * 128 * 2;      // Q tile: two 64-column sub-tiles of 128 rows (32 KB)
constexpr int kKvHalf = kKeys * 64 * 2;       // one 64-column box of 64 keys (8 KB)
constexpr int kKvStage = 4 * kKvHalf;         // K (2 boxes) + V (2 boxes) = 32 KB
constexpr int kPBytes = kRows * kKeys * 2;    // P tile: 128 rows x 64 keys bf16 (16 KB) = the K boxes
static_assert(kPBytes == 2 * kKvHalf, "P_j replaces K_j in its stage");
constexpr int kOffQ = 0;
constexpr int kOffKv = kOffQ + kQBytes;
template <int STAGES>
struct RingCfg {
  static constexpr int kOffBar = kOffKv + STAGES * kKvStage;
  static constexpr int kSmem = 1024 + kOffBar + 256;  // + alignment slack, barriers, TMEM slot
};
constexpr uint32_t kTmemS = 0;                // S buffers: columns [0, 64), [64, 128)
constexpr uint32_t kTmemO = 128;              // O accumulator: columns [128, 256)
constexpr uint32_t kTmemCols = 256;
constexpr float kLog2e = 1.4426950408889634f;
static_assert(RingCfg<2>::kSmem <= 227 * 1024 / 2, "two CTAs per SM with two stages");
static_assert(RingCfg<3>::kSmem <= 227 * 1024, "shared memory budget");

struct TcBars {
  uint64_t kv_full[kMaxStages], kv_empty[kMaxStages];
  uint64_t q_ready;
  uint64_t s_full[2], s_free[2];
  uint64_t p_full[2];
  uint64_t o_done;   // one phase per P.V product (a rescale waits for the latest, never two behind)
  uint64_t o_final;  // one phase: every P.V product has landed
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

// The same for the 32 lanes of a softmax warp: the result is warp-uniform, so that the
// warp-collective TMEM accesses that follow are taken by all lanes or none.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, int* err, int site, int rows) {
  return __all_sync(0xffffffffu, wait_or_report(bar, parity, err, site, rows));
}

}  // namespace

template <bool KT, int STAGES>
__global__ void __launch_bounds__(192, 2) attn_tc_long_kernel(const AttnArgs a, const CUtensorMap* maps, int tq) {
  constexpr int kStages = STAGES;
  // The request table, Q and this layer's K/V rows come from kernels earlier in the stream (the
  // per-call prepare kernel among them): wait for them before reading anything.
  pdl_wait();
  pdl_trigger();
  if (threadIdx.x == 0) ktrace_stamp<KT>(a.ktrace, 1);
  const int G = a.hq / a.hkv;
  const int S = a.n_splits > 1 ? a.n_splits : 1;  // key splits (cached calls only)
  const int qtile = blockIdx.x, kvh = blockIdx.y, req = blockIdx.z / S, split = blockIdx.z % S;
  const ReqDesc r = a.reqs[req];
  const int tok0 = qtile * tq;  // first request-local token of this tile
  if (tok0 >= r.n_q) return;    // uniform over the CTA: nothing allocated yet
  const int tok_last = min(tok0 + tq, r.n_q) - 1;
  const int key_end = row_key_limit(r, tok_last, a.causal_block);  // the last token attends the most
  // this split's keys [kbeg, kend): equal 64-aligned shares of the request's own length (read on
  // the device), the last one shorter, trailing ones possibly empty
  int kbeg = 0, kend = key_end;
  if (S > 1) {
    const int share = ((key_end + S - 1) / S + kKeys - 1) / kKeys * kKeys;
    kbeg = min(key_end, split * share);
    kend = min(key_end, kbeg + share);
  }
  const int n_tiles = (kend - kbeg + kKeys - 1) / kKeys;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = base + kOffQ;
  uint8_t* sKv = base + kOffKv;
  TcBars* bar = reinterpret_cast<TcBars*>(base + RingCfg<STAGES>::kOffBar);
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
    }
    mbar_init(&bar->o_done, 1);
    mbar_init(&bar->o_final, 1);
    mbar_fence_init();
  }
  if (warp == 1) {
    tmem_alloc(&bar->tmem, kTmemCols);
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
          tma_load_3d(kvs + h * kKvHalf, mk, &bar->kv_full[st], kvh * a.hd + h * 64, kbeg + j * kKeys, layer_c, pol);
          tma_load_3d(kvs + (2 + h) * kKvHalf, mv, &bar->kv_full[st], kvh * a.hd + h * 64, kbeg + j * kKeys, layer_c,
                      pol);
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
        if (j >= 1) {  // O += P_i V_i, i = j - 1; P_i sits where K_i was
          const int i = j - 1, st = i % kStages;
          if (!wait_or_report(&bar->p_full[i & 1], (i >> 1) & 1u, a.err, 25, a.m_total)) {
            ok = false;
            break;
          }
          tc_fence_after_sync();
          const uint8_t* pt = sKv + st * kKvStage;
          const uint8_t* vt = pt + 2 * kKvHalf;
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            const uint64_t ad = umma_desc_sw128(pt) + 2 * kk;
            // V rows are keys (the reduction), 64 head-dim columns per box: 16 keys per step are
            // two 8-row groups, 2048 B on; the second 64 columns sit one box (kKvHalf) further.
            const uint64_t bd = umma_desc_sw128_mn(vt + kk * 2048, kKvHalf, 1024);
            tc_mma_bf16(tmem + kTmemO, ad, bd, idesc_o, (i > 0 || kk > 0) ? 1u : 0u);
          }
          tc_commit(&bar->o_done);
          tc_commit(&bar->kv_empty[st]);
          if (i == n_tiles - 1) tc_commit(&bar->o_final);
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
    const int lim = valid ? min(row_key_limit(r, tl, a.causal_block), kend) : 0;
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
    float m_base = -INFINITY, l_run = 0.f;  // exponent base of this row's probabilities and their sum
    bool ok = true;

    for (int j = 0; j < n_tiles && ok; ++j) {
      const int sb = j & 1;
      if (!(ok = warp_wait(&bar->s_full[sb], (j >> 1) & 1u, a.err, 28, a.m_total))) break;
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

      // mask, scale to the log2 domain, tile maximum
      const int key0 = kbeg + j * kKeys;
      float mx = -INFINITY;
#pragma unroll
      for (int c = 0; c < kKeys; ++c) {
        s[c] = (key0 + c < lim) ? s[c] * sl2 : -INFINITY;
        mx = fmaxf(mx, s[c]);
      }
      // The base moves on the first tile with keys and whenever the maximum outgrows it by > 2^8;
      // then O (the earlier tiles' P.V, in TMEM) is scaled by 2^(old - new) before P_j V_j adds.
      const bool move = mx > m_base + a.lazy_log2 || (m_base == -INFINITY && mx != -INFINITY);
      float alpha = 1.f;
      if (move) {
        alpha = m_base == -INFINITY ? 0.f : exp2f(m_base - mx);
        m_base = mx;
      }
      if (__any_sync(0xffffffffu, move && j > 0 && alpha != 0.f)) {
        // this warp's rows of O hold P_0..P_{j-1} V: the last of those products has to land first.
        // S_j's commit covered every MMA issued before it, P_{j-2} V among them, so o_done is at
        // phase j - 1 or j here and its parity names the right phase.
        if (!(ok = warp_wait(&bar->o_done, (j - 1) & 1u, a.err, 27, a.m_total))) break;
        tc_fence_after_sync();
#pragma unroll
        for (int c0 = 0; c0 < 128; c0 += 32) {
          uint32_t v[32];
          tmem_ld_32x32b_x32(tmem + lane_base + kTmemO + c0, v);
          tmem_ld_wait();
#pragma unroll
          for (int c = 0; c < 32; ++c) v[c] = __float_as_uint(__uint_as_float(v[c]) * alpha);
          tmem_st_32x32b_x32(tmem + lane_base + kTmemO + c0, v);
        }
        tmem_st_wait();
        tc_fence_before_sync();
      }
      const float m_use = m_base == -INFINITY ? 0.f : m_base;
      float psum = 0.f;
#pragma unroll
      for (int c = 0; c < kKeys; ++c) {
        s[c] = exp2f(s[c] - m_use);
        psum += s[c];
      }
      l_run = l_run * alpha + psum;

      // P_j (bf16) -> this row's 8 swizzled 16-byte chunks over K_j (S_j has finished with it)
      uint8_t* prow = sKv + (j % kStages) * kKvStage + row * 128;
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
      if (lane == 0) mbar_arrive(&bar->p_full[j & 1]);
    }
    // every P.V has landed (its own one-phase barrier: o_done may be two phases on by now): O / l
    if (ok && n_tiles > 0) ok = warp_wait(&bar->o_final, 0, a.err, 26, a.m_total);
    if (ok && S > 1) {
      // a split's partial: O / l in fp32 and the row's log2-sum-exp, for attn_split_merge_kernel
      const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
      const size_t prow = (static_cast<size_t>(split) * a.m_total + r.q_tok0 + (valid ? tl : 0)) * a.hq + head;
      float4* dst = reinterpret_cast<float4*>(a.part + prow * a.hd);
      tc_fence_after_sync();
#pragma unroll
      for (int c0 = 0; c0 < 128; c0 += 32) {
        uint32_t v[32];
        if (n_tiles > 0) {
          tmem_ld_32x32b_x32(tmem + lane_base + kTmemO + c0, v);
          tmem_ld_wait();
        } else {
#pragma unroll
          for (int c = 0; c < 32; ++c) v[c] = 0u;
        }
        if (valid) {
#pragma unroll
          for (int c = 0; c < 8; ++c)
            dst[c0 / 4 + c] = make_float4(__uint_as_float(v[4 * c]) * inv, __uint_as_float(v[4 * c + 1]) * inv,
                                          __uint_as_float(v[4 * c + 2]) * inv, __uint_as_float(v[4 * c + 3]) * inv);
        }
      }
      if (valid) a.part_lse[prow] = l_run > 0.f ? m_base + log2f(l_run) : -INFINITY;
      tc_fence_before_sync();
    } else if (ok) {
      const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
      uint4* dst = reinterpret_cast<uint4*>(static_cast<bf16*>(a.out) + static_cast<size_t>(r.q_tok0 + (valid ? tl : 0)) * qstride +
                                            static_cast<size_t>(head) * a.hd);
      tc_fence_after_sync();
#pragma unroll
      for (int c0 = 0; c0 < 128; c0 += 32) {
        uint32_t v[32];
        if (n_tiles > 0) {
          tmem_ld_32x32b_x32(tmem + lane_base + kTmemO + c0, v);
          tmem_ld_wait();
        } else {
#pragma unroll
          for (int c = 0; c < 32; ++c) v[c] = 0u;
        }
        if (valid) {
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            uint4 u;
            u.x = pack_bf16x2(__uint_as_float(v[8 * c + 0]) * inv, __uint_as_float(v[8 * c + 1]) * inv);
            u.y = pack_bf16x2(__uint_as_float(v[8 * c + 2]) * inv, __uint_as_float(v[8 * c + 3]) * inv);
            u.z = pack_bf16x2(__uint_as_float(v[8 * c + 4]) * inv, __uint_as_float(v[8 * c + 5]) * inv);
            u.w = pack_bf16x2(__uint_as_float(v[8 * c + 6]) * inv, __uint_as_float(v[8 * c + 7]) * inv);
            dst[c0 / 8 + c] = u;
          }
        }
      }
      tc_fence_before_sync();
    }
  }
  __syncwarp();
  tc_fence_before_sync();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after_sync();
    tmem_dealloc(tmem, kTmemCols);
  }
  if (threadIdx.x == 0) ktrace_stamp<KT>(a.ktrace, 7);
}

int init_attention_tc_long_attributes() {
  cudaError_t e = cudaSuccess;
  for (auto f : {attn_tc_long_kernel<false, 2>, attn_tc_long_kernel<true, 2>})
    if (e == cudaSuccess) e = cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, RingCfg<2>::kSmem);
  for (auto f : {attn_tc_long_kernel<false, 3>, attn_tc_long_kernel<true, 3>})
    if (e == cudaSuccess) e = cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, RingCfg<3>::kSmem);
  return e;
}

// Key-split merge: one warp per (token, query head); each lane merges 4 of the 128 columns over
// the S splits in split order: out = sum_s w_s o_s / sum_s w_s, w_s = 2^(lse_s - max lse).
__global__ void __launch_bounds__(256) attn_split_merge_kernel(const AttnArgs a) {
  pdl_wait();
  pdl_trigger();
  const int pair = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (pair >= a.m_total * a.hq) return;
  const int S = a.n_splits;
  const size_t plane = static_cast<size_t>(a.m_total) * a.hq;
  float l[kMaxAttnSplits];
  float mx = -INFINITY;
#pragma unroll
  for (int m = 0; m < kMaxAttnSplits; ++m) {
    l[m] = m < S ? a.part_lse[m * plane + pair] : -INFINITY;
    mx = fmaxf(mx, l[m]);
  }
  float4 v[kMaxAttnSplits];
#pragma unroll
  for (int m = 0; m < kMaxAttnSplits; ++m)
    v[m] = m < S ? reinterpret_cast<const float4*>(a.part + (m * plane + pair) * a.hd)[lane] : make_float4(0.f, 0.f, 0.f, 0.f);
  float den = 0.f;
  float4 num = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int m = 0; m < kMaxAttnSplits; ++m) {
    const float w = (m < S && l[m] != -INFINITY) ? exp2f(l[m] - mx) : 0.f;
    den += w;
    num.x += w * v[m].x;
    num.y += w * v[m].y;
    num.z += w * v[m].z;
    num.w += w * v[m].w;
  }
  const float inv = den > 0.f ? 1.f / den : 0.f;
  bf16* op = static_cast<bf16*>(a.out) + static_cast<size_t>(pair) * a.hd + lane * 4;
  *reinterpret_cast<uint2*>(op) = make_uint2(pack_bf16x2(num.x * inv, num.y * inv), pack_bf16x2(num.z * inv, num.w * inv));
}

// Two CTAs per SM (2-stage ring) for grids of more CTAs than SMs, else one with a 3-stage ring (two
// K/V tiles in flight ahead of the one being computed).
int launch_attention_tc_long(const AttnArgs& a, const CUtensorMap* maps_dev, dim3 grid, int tq, int num_sms,
                             cudaStream_t s) {
  const int S = a.n_splits > 1 ? a.n_splits : 1;
  grid.z *= S;
  const bool two = static_cast<long long>(grid.x) * grid.y * grid.z > num_sms;
  cudaError_t e;
  if (two)
    e = a.ktrace != nullptr ? launch_k(attn_tc_long_kernel<true, 2>, grid, dim3(192), RingCfg<2>::kSmem, s, a, maps_dev, tq)
                            : launch_k(attn_tc_long_kernel<false, 2>, grid, dim3(192), RingCfg<2>::kSmem, s, a, maps_dev, tq);
  else
    e = a.ktrace != nullptr ? launch_k(attn_tc_long_kernel<true, 3>, grid, dim3(192), RingCfg<3>::kSmem, s, a, maps_dev, tq)
                            : launch_k(attn_tc_long_kernel<false, 3>, grid, dim3(192), RingCfg<3>::kSmem, s, a, maps_dev, tq);
  if (e != cudaSuccess || S == 1) return e;
  const int pairs = a.m_total * a.hq;
  return launch_k(attn_split_merge_kernel, dim3((pairs + 7) / 8), dim3(256), 0, s, a);
}

}  // namespace fdllm
