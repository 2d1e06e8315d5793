// GQA attention over the in-place KV cache (cached steps) and over a block-causal biased window
// (prefill / forward_hidden).
//
// Reference semantics: fast_dllm_relax/runtime.py:63-73 (cached: write rows, then non-causal
// attention over cache rows [0, prefix_len + attend_rel)) and model/cuda.py:401-466 (dense: fp32
// scores * scale + bias, fp32 softmax, PV, one cast at the end).  The scale is head_dim**-0.5.
//
// bf16: one CTA per (request, 16-token query tile, KV head, key split).  The 16 tokens x G query
// heads that share a KV head form 16*G query rows, one m16 tile per warp, so each K/V byte staged in
// shared memory serves all G heads.  K/V tiles of 64 keys stream through a ring of three with
// cp.async into a XOR-swizzled layout and are read with ldmatrix; QK^T and PV run on mma.sync m16n8k16 (bf16 in,
// fp32 accumulate) with an online (flash) softmax in registers and quad shuffles for the row
// reductions.  Long key ranges are split across the CTAs of a thread-block cluster, which merge
// their partial outputs by log-sum-exp through distributed shared memory.
// fp32: a CUDA-core kernel, one warp per (token, head), online softmax with warp-shuffle dots.
#include <algorithm>

#include "common.cuh"
#include "kernels.h"

namespace fdllm {

constexpr int kQT = 16;  // query tokens per CTA
constexpr int kKT = 64;  // keys per shared-memory tile
constexpr int kKV = 3;   // K/V tile ring depth: two tiles in flight while one is computed
static_assert(kKV == 3, "the tail waits of the tile loop are written for a ring of three");
constexpr float kLog2e = 1.4426950408889634f;

__device__ __forceinline__ void mma_16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// Byte offset of 16-byte chunk `c` of key row `key` in a swizzled [kKT][HD] bf16 tile.
template <int HD>
__device__ __forceinline__ uint32_t tile_off(int key, int c) {
  return static_cast<uint32_t>(key * (HD * 2) + ((c ^ (key & 7)) << 4));
}

// At most 6 query heads per KV head (192 threads).  MINB = 2 (two CTAs per SM, <= 170 registers)
// for launches with more CTAs than SMs; MINB = 1 keeps every accumulator in registers.
template <int HD, int MINB, bool KT>
__global__ void __launch_bounds__(192, MINB) attn_mma_kernel(const AttnArgs a) {
  if (threadIdx.x == 0) ktrace_stamp<KT>(a.ktrace, 0);
  pdl_trigger();
  pdl_wait();
  if (threadIdx.x == 0) ktrace_stamp<KT>(a.ktrace, 1);
  constexpr int kChunks = HD / 8;          // 16-byte chunks per key row
  constexpr int kTileBytes = kKT * HD * 2;
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* Ks = smem;                        // [kKV][kKT][HD]
  uint8_t* Vs = smem + kKV * kTileBytes;     // [kKV][kKT][HD]

  const int G = a.hq / a.hkv;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g8 = lane >> 2, t4 = lane & 3;
  const int qtile = blockIdx.x, kvh = blockIdx.y;
  const int req = blockIdx.z / a.n_splits, split = blockIdx.z % a.n_splits;
  const ReqDesc r = a.reqs[req];
  const int tq0 = qtile * kQT;
  if (tq0 >= r.n_q) return;
  const int L = r.attend_len;
  // Keys split evenly over this request's own length (read on the device, so a captured graph
  // adapts as the prefix grows); a.split_len is a lower bound.
  const int split_len = a.n_splits == 1 ? L : max(a.split_len, ((L + a.n_splits - 1) / a.n_splits + 63) / 64 * 64);
  const int key0 = split * split_len;
  int key1 = min(L, key0 + split_len);
  const bool implicit_mask = (a.bias == nullptr && a.causal_block > 0);
  if (implicit_mask) {  // keys past the last query's block are masked for every row of this tile
    const int tq_last = min(tq0 + kQT, r.n_q) - 1;
    key1 = min(key1, (tq_last / a.causal_block + 1) * a.causal_block);
  }
  const size_t kv_row = static_cast<size_t>(a.hkv) * HD;
  const bf16* kg = static_cast<const bf16*>(r.k) + static_cast<size_t>(a.layer) * r.layer_stride + kvh * HD;
  const bf16* vg = static_cast<const bf16*>(r.v) + static_cast<size_t>(a.layer) * r.layer_stride + kvh * HD;
  const bf16* qg = static_cast<const bf16*>(a.q);

  // Query rows of this thread: ra = 16*warp + g8 and rb = ra + 8; row -> (token, head in group).
  int tok_row[2], qh_row[2];
  bool valid_row[2];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int rr = warp * 16 + g8 + h * 8;
    const int tq = tq0 + rr / G;
    valid_row[h] = (rr < kQT * G) && (tq < r.n_q);
    tok_row[h] = r.q_tok0 + (valid_row[h] ? tq : 0);
    qh_row[h] = kvh * G + rr % G;
  }
  uint32_t qf[HD / 16][4];
#pragma unroll
  for (int kk = 0; kk < HD / 16; ++kk) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const bf16* qp = qg + static_cast<size_t>(tok_row[h]) * (a.hq * HD) + qh_row[h] * HD + kk * 16 + 2 * t4;
      qf[kk][h] = valid_row[h] ? *reinterpret_cast<const uint32_t*>(qp) : 0u;
      qf[kk][h + 2] = valid_row[h] ? *reinterpret_cast<const uint32_t*>(qp + 8) : 0u;
    }
  }

  float o[HD / 8][4];
#pragma unroll
  for (int n = 0; n < HD / 8; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
  float m_run[2] = {-INFINITY, -INFINITY};
  float l_run[2] = {0.f, 0.f};

  const int n_tiles = (key1 > key0) ? (key1 - key0 + kKT - 1) / kKT : 0;
  auto load_tile = [&](int it, int buf) {
    const int kt0 = key0 + it * kKT;
    for (int idx = threadIdx.x; idx < kKT * kChunks; idx += blockDim.x) {
      const int key = idx / kChunks, c = idx % kChunks;
      const bool ok = kt0 + key < key1;
      const size_t src = static_cast<size_t>(ok ? kt0 + key : 0) * kv_row + c * 8;
      cp_async_16(Ks + buf * kTileBytes + tile_off<HD>(key, c), kg + src, ok);
      cp_async_16(Vs + buf * kTileBytes + tile_off<HD>(key, c), vg + src, ok);
    }
    cp_async_commit();
  };

  for (int p = 0; p < kKV - 1 && p < n_tiles; ++p) load_tile(p, p);
  for (int it = 0; it < n_tiles; ++it) {
    const int buf = it % kKV;
    // tile it must have landed: the groups still pending may only be the later tiles issued
    if (it + kKV - 1 < n_tiles) {
      load_tile(it + kKV - 1, (it + kKV - 1) % kKV);  // into the buffer tile it-1 used
      cp_async_wait<kKV - 1>();
    } else if (it + 1 < n_tiles) {
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const uint32_t kb = smem_addr(Ks + buf * kTileBytes);
    const uint32_t vb = smem_addr(Vs + buf * kTileBytes);
    const int kt0 = key0 + it * kKT;

    float s[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < HD / 16; ++kk) {
#pragma unroll
      for (int jp = 0; jp < 4; ++jp) {
        const int m = lane >> 3, i = lane & 7;
        const int key = (2 * jp + (m >> 1)) * 8 + i;
        uint32_t b[4];
        ldsm_x4(b, kb + tile_off<HD>(key, kk * 2 + (m & 1)));
        mma_16816(s[2 * jp], qf[kk], b[0], b[1]);
        mma_16816(s[2 * jp + 1], qf[kk], b[2], b[3]);
      }
    }
    // scale, bias, mask; online softmax per row half
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      float mx = -INFINITY;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int key = kt0 + j * 8 + 2 * t4 + e;
          float v = s[j][2 * h + e] * a.scale;
          if (a.bias != nullptr) {
            const int brow = tok_row[h] - r.q_tok0;
            v += (key < key1) ? a.bias[static_cast<size_t>(brow) * a.ld_bias + key] : 0.f;
          } else if (implicit_mask) {
            const int tq = tok_row[h] - r.q_tok0;
            if (key / a.causal_block > tq / a.causal_block) v = -INFINITY;
          }
          if (key >= key1) v = -INFINITY;
          s[j][2 * h + e] = v;
          mx = fmaxf(mx, v);
        }
      }
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      const float m_new = fmaxf(m_run[h], mx);
      const float m_use = (m_new == -INFINITY) ? 0.f : m_new;
      const float alpha = exp2f((m_run[h] - m_use) * kLog2e);
      float psum = 0.f;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const float p = exp2f((s[j][2 * h + e] - m_use) * kLog2e);
          s[j][2 * h + e] = p;
          psum += p;
        }
      }
      l_run[h] = l_run[h] * alpha + psum;
      m_run[h] = m_new;
#pragma unroll
      for (int n = 0; n < HD / 8; ++n) {
        o[n][2 * h] *= alpha;
        o[n][2 * h + 1] *= alpha;
      }
    }
    // O += P V
#pragma unroll
    for (int kc = 0; kc < 4; ++kc) {
      uint32_t pa[4];
      pa[0] = pack_bf16(s[2 * kc][0], s[2 * kc][1]);
      pa[1] = pack_bf16(s[2 * kc][2], s[2 * kc][3]);
      pa[2] = pack_bf16(s[2 * kc + 1][0], s[2 * kc + 1][1]);
      pa[3] = pack_bf16(s[2 * kc + 1][2], s[2 * kc + 1][3]);
#pragma unroll
      for (int np = 0; np < HD / 16; ++np) {
        const int m = lane >> 3, i = lane & 7;
        const int key = kc * 16 + (m & 1) * 8 + i;
        uint32_t b[4];
        ldsm_x4_t(b, vb + tile_off<HD>(key, 2 * np + (m >> 1)));
        mma_16816(o[2 * np], pa, b[0], b[1]);
        mma_16816(o[2 * np + 1], pa, b[2], b[3]);
      }
    }
    __syncthreads();
  }

#pragma unroll
  for (int h = 0; h < 2; ++h) {
    l_run[h] += __shfl_xor_sync(0xffffffffu, l_run[h], 1);
    l_run[h] += __shfl_xor_sync(0xffffffffu, l_run[h], 2);
  }
  if (threadIdx.x == 0) ktrace_stamp<KT>(a.ktrace, 2);
  if (a.n_splits == 1) {
    bf16* out = static_cast<bf16*>(a.out);
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      if (!valid_row[h]) continue;
      const float inv = l_run[h] > 0.f ? 1.f / l_run[h] : 0.f;
      bf16* op = out + static_cast<size_t>(tok_row[h]) * (a.hq * HD) + qh_row[h] * HD;
#pragma unroll
      for (int n = 0; n < HD / 8; ++n) {
        *reinterpret_cast<__nv_bfloat162*>(op + n * 8 + 2 * t4) =
            __floats2bfloat162_rn(o[n][2 * h] * inv, o[n][2 * h + 1] * inv);
      }
    }
  } else {
    // Key splits of one (request, query tile, KV head) form a thread-block cluster.  Each member
    // leaves its normalized partial O and log-sum-exp in shared memory (the K/V tiles are no longer
    // needed); member r then merges query rows [r*R/S, (r+1)*R/S) over all members through
    // distributed shared memory: out = sum_s w_s o_s / sum_s w_s, w_s = exp(lse_s - max lse).
    __shared__ float s_lse[kQT * 8];
    __shared__ float s_w[kQT * 4][kMaxAttnSplits + 1];  // merge weights of this member's rows, 1/sum
    constexpr int kOP = HD + 4;  // padded fp32 partial rows: the float2 writes hit distinct banks
    float* o_s = reinterpret_cast<float*>(smem);  // [16 * G][kOP] fp32
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int rr = warp * 16 + g8 + h * 8;
      const float inv = l_run[h] > 0.f ? 1.f / l_run[h] : 0.f;
#pragma unroll
      for (int n = 0; n < HD / 8; ++n)
        *reinterpret_cast<float2*>(o_s + rr * kOP + n * 8 + 2 * t4) = make_float2(o[n][2 * h] * inv, o[n][2 * h + 1] * inv);
      if (t4 == 0) s_lse[rr] = (valid_row[h] && l_run[h] > 0.f) ? m_run[h] + logf(l_run[h]) : -INFINITY;
    }
    cluster_sync();  // every member's partial is in its shared memory
    if (threadIdx.x == 0) ktrace_stamp<KT>(a.ktrace, 3);
    constexpr int kMaxS = kMaxAttnSplits;
    const uint32_t S = static_cast<uint32_t>(a.n_splits);
    const uint32_t rank = cluster_ctarank();
    const int rows = kQT * G;
    const int r0 = static_cast<int>(rank * rows / S), r1 = static_cast<int>((rank + 1) * rows / S);
    const uint32_t o_addr = smem_addr(o_s), lse_addr = smem_addr(s_lse);
    for (int rr = r0 + threadIdx.x; rr < r1; rr += blockDim.x) {  // per-row member weights, once
      float l[kMaxS];
      float mx = -INFINITY;
#pragma unroll
      for (int m = 0; m < kMaxS; ++m) {
        l[m] = (static_cast<uint32_t>(m) < S) ? ld_dsmem_f32(map_shared_rank(lse_addr + rr * 4, m)) : -INFINITY;
        mx = fmaxf(mx, l[m]);
      }
      float den = 0.f;
#pragma unroll
      for (int m = 0; m < kMaxS; ++m) {
        const float w = (static_cast<uint32_t>(m) < S && l[m] != -INFINITY) ? expf(l[m] - mx) : 0.f;
        s_w[rr - r0][m] = w;
        den += w;
      }
      s_w[rr - r0][kMaxS] = den > 0.f ? 1.f / den : 0.f;
    }
    __syncthreads();
    if (threadIdx.x == 0) ktrace_stamp<KT>(a.ktrace, 4);
    bf16* out = static_cast<bf16*>(a.out);
    for (int idx = threadIdx.x; idx < (r1 - r0) * (HD / 4); idx += blockDim.x) {
      const int rr = r0 + idx / (HD / 4), c4 = idx % (HD / 4);
      const int tq = tq0 + rr / G;
      if (tq >= r.n_q) continue;
      float4 v[kMaxS];
#pragma unroll
      for (int m = 0; m < kMaxS; ++m)  // all members' chunks in flight at once
        v[m] = (static_cast<uint32_t>(m) < S) ? ld_dsmem_f4(map_shared_rank(o_addr + (rr * kOP + c4 * 4) * 4, m))
                                              : make_float4(0.f, 0.f, 0.f, 0.f);
      float4 num = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int m = 0; m < kMaxS; ++m) {
        const float w = s_w[rr - r0][m];
        num.x += w * v[m].x;
        num.y += w * v[m].y;
        num.z += w * v[m].z;
        num.w += w * v[m].w;
      }
      const float inv = s_w[rr - r0][kMaxS];
      bf16* op = out + static_cast<size_t>(r.q_tok0 + tq) * (a.hq * HD) + (kvh * G + rr % G) * HD + c4 * 4;
      *reinterpret_cast<__nv_bfloat162*>(op) = __floats2bfloat162_rn(num.x * inv, num.y * inv);
      *reinterpret_cast<__nv_bfloat162*>(op + 2) = __floats2bfloat162_rn(num.z * inv, num.w * inv);
    }
    if (threadIdx.x == 0) ktrace_stamp<KT>(a.ktrace, 5);
    cluster_sync();  // no member leaves while another may still read its shared memory
  }
  if (threadIdx.x == 0) ktrace_stamp<KT>(a.ktrace, 7);
}

// CUDA-core attention: one warp per (token, query head); dims split over lanes (hd <= 128).
template <typename T>
__global__ void attn_simt_kernel(const AttnArgs a) {
  pdl_trigger();
  pdl_wait();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int req = blockIdx.z;
  const ReqDesc r = a.reqs[req];
  const int gid = blockIdx.x * (blockDim.x >> 5) + warp;
  const int tq = gid / a.hq, qh = gid % a.hq;
  if (tq >= r.n_q) return;
  const int G = a.hq / a.hkv;
  const int kvh = qh / G;
  const int tok = r.q_tok0 + tq;
  const int nd = a.hd / 32;
  const T* q = static_cast<const T*>(a.q) + static_cast<size_t>(tok) * a.hq * a.hd + qh * a.hd;
  const T* kg = static_cast<const T*>(r.k) + static_cast<size_t>(a.layer) * r.layer_stride + kvh * a.hd;
  const T* vg = static_cast<const T*>(r.v) + static_cast<size_t>(a.layer) * r.layer_stride + kvh * a.hd;
  const size_t kv_row = static_cast<size_t>(a.hkv) * a.hd;
  float qv[4], ov[4] = {0.f, 0.f, 0.f, 0.f};
  for (int i = 0; i < 4; ++i) qv[i] = (i < nd) ? to_f<T>(q[lane + 32 * i]) : 0.f;
  float m = -INFINITY, l = 0.f;
  const int L = r.attend_len;
  for (int key = 0; key < L; ++key) {
    const T* kp = kg + key * kv_row;
    float dot = 0.f;
    for (int i = 0; i < nd; ++i) dot = fmaf(qv[i], to_f<T>(kp[lane + 32 * i]), dot);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, off);
    float sc = dot * a.scale;
    if (a.bias != nullptr) sc += a.bias[static_cast<size_t>(tq) * a.ld_bias + key];
    else if (a.causal_block > 0 && key / a.causal_block > tq / a.causal_block) continue;  // exp -> 0
    const float m_new = fmaxf(m, sc);
    const float alpha = (m == -INFINITY) ? 0.f : expf(m - m_new);
    const float p = expf(sc - m_new);
    l = l * alpha + p;
    const T* vp = vg + key * kv_row;
    for (int i = 0; i < nd; ++i) ov[i] = ov[i] * alpha + p * to_f<T>(vp[lane + 32 * i]);
    m = m_new;
  }
  T* out = static_cast<T*>(a.out) + static_cast<size_t>(tok) * a.hq * a.hd + qh * a.hd;
  const float inv = l > 0.f ? 1.f / l : 0.f;
  for (int i = 0; i < nd; ++i) out[lane + 32 * i] = from_f<T>(ov[i] * inv);
}

template <int HD>
static int launch_mma(const AttnArgs& a, int max_q, cudaStream_t s) {
  const int G = a.hq / a.hkv;
  constexpr int smem = 2 * kKV * kKT * HD * 2;
  cudaError_t e;
  dim3 grid((max_q + kQT - 1) / kQT, a.hkv, a.n_reqs * a.n_splits);
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const bool many = static_cast<long long>(grid.x) * grid.y * grid.z > sms;
  if (a.ktrace != nullptr)
    e = many ? launch_kc(attn_mma_kernel<HD, 2, true>, grid, dim3(G * 32), smem, s, a.n_splits, a)
             : launch_kc(attn_mma_kernel<HD, 1, true>, grid, dim3(G * 32), smem, s, a.n_splits, a);
  else
    e = many ? launch_kc(attn_mma_kernel<HD, 2, false>, grid, dim3(G * 32), smem, s, a.n_splits, a)
             : launch_kc(attn_mma_kernel<HD, 1, false>, grid, dim3(G * 32), smem, s, a.n_splits, a);
  return e;
}

int init_gemm_tc_attributes();

template <int HD, int MINB, bool KT>
static cudaError_t attn_attrs1() {
  cudaError_t e = cudaFuncSetAttribute(attn_mma_kernel<HD, MINB, KT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       2 * kKV * kKT * HD * 2);
  if (e == cudaSuccess) e = cudaFuncSetAttribute(attn_mma_kernel<HD, MINB, KT>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
  return e;
}

template <int HD, int MINB>
static cudaError_t attn_attrs() {
  cudaError_t e = attn_attrs1<HD, MINB, false>();
  if (e == cudaSuccess) e = attn_attrs1<HD, MINB, true>();
  return e;
}

int init_kernel_attributes() {
  cudaError_t e = attn_attrs<128, 1>();
  if (e == cudaSuccess) e = attn_attrs<128, 2>();
  if (e == cudaSuccess) e = attn_attrs<64, 1>();
  if (e == cudaSuccess) e = attn_attrs<64, 2>();
  if (e == cudaSuccess) e = static_cast<cudaError_t>(init_gemm_tc_attributes());
  if (e == cudaSuccess) e = static_cast<cudaError_t>(init_attention_tc_attributes());
  return e;
}

int launch_attention(const AttnArgs& a, int max_q, int dtype, cudaStream_t s) {
  if (a.hq % a.hkv != 0 || a.hd % 32 != 0 || a.hd > 128) return cudaErrorInvalidValue;
  const int G = a.hq / a.hkv;
  if (dtype == 1 && (a.hd == 128 || a.hd == 64) && G <= 6) {
    return a.hd == 128 ? launch_mma<128>(a, max_q, s) : launch_mma<64>(a, max_q, s);
  }
  AttnArgs b = a;
  b.n_splits = 1;
  const int per_block = 4;
  dim3 grid((max_q * a.hq + per_block - 1) / per_block, 1, a.n_reqs);
  if (dtype == 1) return launch_k(attn_simt_kernel<bf16>, grid, dim3(per_block * 32), 0, s, b);
  return launch_k(attn_simt_kernel<float>, grid, dim3(per_block * 32), 0, s, b);
}

}  // namespace fdllm
