// Small kernels around the projections and attention: embedding gather, RMSNorm, RoPE tables,
// per-call request preparation, confidence / log-softmax reductions and the unmask decision.
#include <math.h>

#include <atomic>
#include <cstdlib>

#include "common.cuh"
#include "kernels.h"

namespace fdllm {

static std::atomic<long long> g_launches{0};
void count_launch(int n) { g_launches.fetch_add(n, std::memory_order_relaxed); }
long long launch_count() { return g_launches.load(std::memory_order_relaxed); }

// ---- embed (model/cuda.py:698-699) ----------------------------------------------------------
template <typename T>
__global__ void embed_kernel(const int* __restrict__ ids, const T* __restrict__ table, int vocab, int hidden,
                             T* __restrict__ out, int* err) {
  pdl_trigger();
  pdl_wait();
  const int i = blockIdx.x;
  const int id = ids[i];
  const bool ok = id >= 0 && id < vocab;
  if (!ok && threadIdx.x == 0) report_error(err, kErrTokenRange);
  const T* src = table + static_cast<size_t>(ok ? id : 0) * hidden;
  T* dst = out + static_cast<size_t>(i) * hidden;
  for (int j = threadIdx.x; j < hidden; j += blockDim.x) dst[j] = ok ? src[j] : from_f<T>(0.f);
}

int launch_embed(const int* ids, int n, const void* table, int vocab, int hidden, void* out, int dtype, int* err,
                 cudaStream_t s) {
  if (n <= 0) return cudaSuccess;
  if (dtype == 1)
    return launch_k(embed_kernel<bf16>, dim3(n), dim3(256), 0, s, ids, static_cast<const bf16*>(table), vocab, hidden,
                    static_cast<bf16*>(out), err);
  return launch_k(embed_kernel<float>, dim3(n), dim3(256), 0, s, ids, static_cast<const float*>(table), vocab, hidden,
                  static_cast<float*>(out), err);
}

// ---- RMSNorm (model/cuda.py:269-275): fp32 mean square, rsqrt, cast, then x weight ------------
__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = 0.f;
  for (int w = 0; w < nw; ++w) t += red[w];  // fixed order: deterministic
  __syncthreads();
  return t;
}

template <typename T>
__global__ void rmsnorm_kernel(const T* __restrict__ x, const T* __restrict__ w, T* __restrict__ out, int hidden,
                               float eps, T* __restrict__ copy_to) {
  __shared__ float red[32];
  pdl_trigger();
  pdl_wait();

  const T* xr = x + static_cast<size_t>(blockIdx.x) * hidden;
  T* orow = out + static_cast<size_t>(blockIdx.x) * hidden;
  float ss = 0.f;
  for (int j = threadIdx.x; j < hidden; j += blockDim.x) {
    const float v = to_f<T>(xr[j]);
    ss = fmaf(v, v, ss);
  }
  const float var = block_sum(ss, red) / static_cast<float>(hidden);
  const float rs = rsqrtf(var + eps);
  T* crow = copy_to ? copy_to + static_cast<size_t>(blockIdx.x) * hidden : nullptr;
  for (int j = threadIdx.x; j < hidden; j += blockDim.x) {
    const T xv = xr[j];
    const float xn = round_t<T>(to_f<T>(xv) * rs);
    orow[j] = from_f<T>(to_f<T>(w[j]) * xn);
    if (crow) crow[j] = xv;  // the residual stream starts as a copy of the input
  }
}

// bf16 rows of hidden % 8 == 0 features (<= 8192): 16-byte chunks held in registers between the
// statistics and the normalisation, so each row is read once and every load of a thread is in
// flight at once.
constexpr int kNormChunks = 4;  // chunks per thread (256 threads x 4 x 8 = 8192 features)
__global__ void __launch_bounds__(256) rmsnorm_bf16_vec_kernel(const bf16* __restrict__ x, const bf16* __restrict__ w,
                                                               bf16* __restrict__ out, int hidden, float eps,
                                                               bf16* __restrict__ copy_to) {
  __shared__ float red[32];
  pdl_trigger();
  const int nch = hidden / 8;
  // the weights do not depend on the previous kernel: load them while it finishes
  const uint4* w4 = reinterpret_cast<const uint4*>(w);
  uint4 wv[kNormChunks];
#pragma unroll
  for (int k = 0; k < kNormChunks; ++k) {
    const int c = threadIdx.x + k * blockDim.x;
    if (c < nch) wv[k] = __ldg(w4 + c);
  }
  pdl_wait();
  const uint4* xr = reinterpret_cast<const uint4*>(x + static_cast<size_t>(blockIdx.x) * hidden);
  uint4 xv[kNormChunks];
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < kNormChunks; ++k) {
    const int c = threadIdx.x + k * blockDim.x;
    if (c < nch) xv[k] = xr[c];
  }
#pragma unroll
  for (int k = 0; k < kNormChunks; ++k) {
    if (threadIdx.x + k * blockDim.x >= nch) continue;
    const __nv_bfloat162* x2 = reinterpret_cast<const __nv_bfloat162*>(&xv[k]);
#pragma unroll
    for (int v = 0; v < 4; ++v) {
      const float2 f = __bfloat1622float2(x2[v]);
      ss = fmaf(f.x, f.x, ss);
      ss = fmaf(f.y, f.y, ss);
    }
  }
  const float rs = rsqrtf(block_sum(ss, red) / static_cast<float>(hidden) + eps);
  uint4* orow = reinterpret_cast<uint4*>(out + static_cast<size_t>(blockIdx.x) * hidden);
  uint4* crow = copy_to ? reinterpret_cast<uint4*>(copy_to + static_cast<size_t>(blockIdx.x) * hidden) : nullptr;
#pragma unroll
  for (int k = 0; k < kNormChunks; ++k) {
    const int c = threadIdx.x + k * blockDim.x;
    if (c >= nch) continue;
    const __nv_bfloat162* x2 = reinterpret_cast<const __nv_bfloat162*>(&xv[k]);
    const __nv_bfloat162* w2 = reinterpret_cast<const __nv_bfloat162*>(&wv[k]);
    uint4 o;
    __nv_bfloat162* o2 = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
    for (int v = 0; v < 4; ++v) {
      const float2 f = __bfloat1622float2(x2[v]);
      const float2 xn = round2_bf16(f.x * rs, f.y * rs);
      const float2 wf = __bfloat1622float2(w2[v]);
      o2[v] = __floats2bfloat162_rn(wf.x * xn.x, wf.y * xn.y);
    }
    orow[c] = o;
    if (crow) crow[c] = xv[k];  // the residual stream starts as a copy of the input
  }
}

int launch_rmsnorm(const void* x, const void* w, void* out, int rows, int hidden, float eps, int dtype,
                   cudaStream_t s, void* copy_x_to) {
  if (rows <= 0) return cudaSuccess;
  auto a16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  if (dtype == 1 && hidden % 8 == 0 && hidden <= 8 * 256 * kNormChunks && a16(x) && a16(w) && a16(out) &&
      a16(copy_x_to))
    return launch_k(rmsnorm_bf16_vec_kernel, dim3(rows), dim3(256), 0, s, static_cast<const bf16*>(x),
                    static_cast<const bf16*>(w), static_cast<bf16*>(out), hidden, eps, static_cast<bf16*>(copy_x_to));
  if (dtype == 1)
    return launch_k(rmsnorm_kernel<bf16>, dim3(rows), dim3(256), 0, s, static_cast<const bf16*>(x),
                    static_cast<const bf16*>(w), static_cast<bf16*>(out), hidden, eps, static_cast<bf16*>(copy_x_to));
  return launch_k(rmsnorm_kernel<float>, dim3(rows), dim3(256), 0, s, static_cast<const float*>(x),
                  static_cast<const float*>(w), static_cast<float*>(out), hidden, eps, static_cast<float*>(copy_x_to));
}

// ---- RoPE tables (model/cuda.py:278-300): inv_freq = exp(-ln(theta) * i / half) in fp32 ----------
template <typename T>
__global__ void rope_table_kernel(T* cos_t, T* sin_t, int max_pos, int half, float neg_log_theta) {
  const size_t idx = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= static_cast<size_t>(max_pos) * half) return;
  const int pos = static_cast<int>(idx / half), i = static_cast<int>(idx % half);
  const float exponent = (neg_log_theta * static_cast<float>(i)) / static_cast<float>(half);
  const float inv_freq = expf(exponent);
  const float f = static_cast<float>(pos) * inv_freq;
  cos_t[idx] = from_f<T>(cosf(f));
  sin_t[idx] = from_f<T>(sinf(f));
}

int launch_rope_tables(void* cos_t, void* sin_t, int max_pos, int hd, float theta, int dtype, cudaStream_t s) {
  const int half = hd / 2;
  const size_t n = static_cast<size_t>(max_pos) * half;
  const int blocks = static_cast<int>((n + 255) / 256);
  const float nl = static_cast<float>(-log(static_cast<double>(theta)));
  if (dtype == 1)
    rope_table_kernel<bf16><<<blocks, 256, 0, s>>>(static_cast<bf16*>(cos_t), static_cast<bf16*>(sin_t), max_pos, half, nl);
  else
    rope_table_kernel<float><<<blocks, 256, 0, s>>>(static_cast<float*>(cos_t), static_cast<float*>(sin_t), max_pos, half, nl);
  count_launch();
  return cudaGetLastError();
}

// ---- per-call request preparation --------------------------------------------------------------
__global__ void prepare_kernel(const ReqBatch b, ReqDesc* table, TokenMaps tok, int max_pos, int* err) {
  pdl_trigger();
  pdl_wait();
  const int i = blockIdx.x;
  if (i >= b.n) return;
  ReqDesc r = b.r[i];
  if (r.plen_dev != nullptr) {
    const int P = *r.plen_dev;
    r.write_start = P + r.write_rel;
    r.attend_len = P + r.attend_rel;
    if (r.rope_off == nullptr) r.rope_base = P + r.write_rel;
    if (P < 0 || r.attend_len > r.cap || r.write_start + r.n_q > r.cap) {
      if (threadIdx.x == 0) report_error(err, kErrCacheRange);
      r.attend_len = min(max(r.attend_len, 0), r.cap);
    }
  }
  if (threadIdx.x == 0) table[b.first + i] = r;
  const int p0 = (r.rope_off != nullptr) ? *r.rope_off : r.rope_base;
  for (int j = threadIdx.x; j < r.n_q; j += blockDim.x) {
    const int t = r.q_tok0 + j;
    int pos = p0 + j;
    if (pos < 0 || pos >= max_pos) {
      report_error(err, kErrPositionRange);
      pos = pos < 0 ? 0 : max_pos - 1;
    }
    const int row = r.write_start + j;
    if (row < 0 || row >= r.cap) report_error(err, kErrCacheRange);
    tok.req[t] = b.first + i;
    tok.pos[t] = pos;
    tok.row[t] = row;
  }
}

int launch_prepare(const ReqBatch& b, ReqDesc* dev_table, TokenMaps tok, int max_pos, int* err, cudaStream_t s) {
  if (b.n <= 0) return cudaSuccess;
  return launch_k(prepare_kernel, dim3(b.n), dim3(128), 0, s, b, dev_table, tok, max_pos, err);
}

// ---- confidence (model/metal.py:316-374): first-index argmax, maxp = 1 / sum exp(l - max) -------
struct Top {
  float m;
  int i;
  float s;
};

__device__ __forceinline__ Top merge_top(Top a, Top b) {
  Top r;
  r.m = fmaxf(a.m, b.m);
  r.i = (a.m > b.m) ? a.i : ((b.m > a.m) ? b.i : min(a.i, b.i));
  const float sa = (a.m == -INFINITY) ? 0.f : a.s * expf(a.m - r.m);
  const float sb = (b.m == -INFINITY) ? 0.f : b.s * expf(b.m - r.m);
  r.s = sa + sb;
  return r;
}

__device__ __forceinline__ Top warp_merge(Top t) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    Top o;
    o.m = __shfl_xor_sync(0xffffffffu, t.m, off);
    o.i = __shfl_xor_sync(0xffffffffu, t.i, off);
    o.s = __shfl_xor_sync(0xffffffffu, t.s, off);
    t = merge_top(t, o);
  }
  return t;
}

// Partials from the fused lm_head epilogue: [rows, n_slabs, 4] = (max, argmax bits, sum exp,
// target logit).  One CTA per row: each thread merges the slabs tid + 256 j with every load of a
// batch in flight first (a one-warp loop over 37 slabs serialised a memory round trip and two
// exponentials per slab), the warps merge by shuffles and thread 0 merges the warps' results in
// warp order -- a fixed order, so the result is deterministic.
constexpr int kTopThreads = 256;
constexpr int kTopPer = 8;  // slabs per thread and batch (vocab 151936: 1187 slabs, one batch)

template <bool kLse>
__global__ void __launch_bounds__(kTopThreads) top_combine_kernel(const float* __restrict__ part, int n_slabs,
                                                                  int* ids, float* maxp, float* logprob) {
  pdl_trigger();
  pdl_wait();
  const int row = blockIdx.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const float4* p4 = reinterpret_cast<const float4*>(part) + static_cast<size_t>(row) * n_slabs;
  Top t{-INFINITY, 0x7fffffff, 0.f};
  float tgt = 0.f;  // exactly one slab holds the target's logit, the others hold 0
  for (int s0 = tid; s0 < n_slabs; s0 += kTopThreads * kTopPer) {
    float4 v[kTopPer];
#pragma unroll
    for (int j = 0; j < kTopPer; ++j)
      if (s0 + j * kTopThreads < n_slabs) v[j] = p4[s0 + j * kTopThreads];
#pragma unroll
    for (int j = 0; j < kTopPer; ++j) {
      if (s0 + j * kTopThreads >= n_slabs) continue;
      t = merge_top(t, Top{v[j].x, __float_as_int(v[j].y), v[j].z});
      if (kLse) tgt += v[j].w;
    }
  }
  t = warp_merge(t);
  if (kLse) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) tgt += __shfl_xor_sync(0xffffffffu, tgt, off);
  }
  __shared__ Top s_t[kTopThreads / 32];
  __shared__ float s_g[kTopThreads / 32];
  if (lane == 0) {
    s_t[warp] = t;
    s_g[warp] = tgt;
  }
  __syncthreads();
  if (tid == 0) {
    Top r = s_t[0];
    float g = s_g[0];
    for (int w = 1; w < kTopThreads / 32; ++w) {
      r = merge_top(r, s_t[w]);
      g += s_g[w];
    }
    if (kLse) {
      logprob[row] = g - (r.m + logf(r.s));
    } else {
      ids[row] = r.i;
      maxp[row] = 1.0f / r.s;
    }
  }
}

int launch_conf_combine(const float* part, int rows, int n_slabs, int* ids, float* maxp, cudaStream_t s) {
  if (rows <= 0) return cudaSuccess;
  return launch_k(top_combine_kernel<false>, dim3(rows), dim3(kTopThreads), 0, s, part, n_slabs, ids, maxp,
                  static_cast<float*>(nullptr));
}

// The same reduction over materialised fp32 logits [rows, vocab] (three passes per row).
__global__ void conf_logits_kernel(const float* __restrict__ logits, int vocab, int* ids, float* maxp) {
  pdl_trigger();
  pdl_wait();
  __shared__ float red_m[32];
  __shared__ int red_i[32];
  __shared__ float red_s[32];
  const float* l = logits + static_cast<size_t>(blockIdx.x) * vocab;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  float m = -INFINITY;
  int mi = 0x7fffffff;
  for (int j = threadIdx.x; j < vocab; j += blockDim.x) {
    const float v = l[j];
    if (v > m) { m = v; mi = j; }  // ascending j per thread: first index kept on ties
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    const float om = __shfl_xor_sync(0xffffffffu, m, off);
    const int oi = __shfl_xor_sync(0xffffffffu, mi, off);
    if (om > m || (om == m && oi < mi)) { m = om; mi = oi; }
  }
  if (lane == 0) { red_m[warp] = m; red_i[warp] = mi; }
  __syncthreads();
  m = red_m[0];
  mi = red_i[0];
  for (int w = 1; w < nw; ++w)
    if (red_m[w] > m || (red_m[w] == m && red_i[w] < mi)) { m = red_m[w]; mi = red_i[w]; }
  float s = 0.f;
  for (int j = threadIdx.x; j < vocab; j += blockDim.x) s += expf(l[j] - m);
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
  if (lane == 0) red_s[warp] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    float tot = 0.f;
    for (int w = 0; w < nw; ++w) tot += red_s[w];
    ids[blockIdx.x] = mi;
    maxp[blockIdx.x] = 1.0f / tot;
  }
}

int launch_conf_from_logits(const float* logits, int rows, int vocab, int* ids, float* maxp, cudaStream_t s) {
  if (rows <= 0) return cudaSuccess;
  return launch_k(conf_logits_kernel, dim3(rows), dim3(512), 0, s, logits, vocab, ids, maxp);
}

// log_softmax(logits)[target] per row from the fused partials (runners.py:877-881 on the device).
int launch_lse_combine(const float* part, int rows, int n_slabs, float* logprob, cudaStream_t s) {
  if (rows <= 0) return cudaSuccess;
  return launch_k(top_combine_kernel<true>, dim3(rows), dim3(kTopThreads), 0, s, part, n_slabs,
                  static_cast<int*>(nullptr), static_cast<float*>(nullptr), logprob);
}

// ---- unmask decision (runtime.py:158-181 shift, 794-805 rule), one warp ------------------------
// ids / maxp: unshifted per-row argmax and confidence of `rows` hidden rows.  Row i of the block
// window takes row i-1's prediction (row 0 its own).  Full steps read the window
// [sub_start, sub_start+sub_len) of the shifted rows; partial steps use all `rows` (= sub_len).
// Masked positions whose confidence exceeds the threshold are unmasked; if none does, the first
// masked position with the largest confidence is.  `block` (the active block's token ids) is
// updated in place.  status[0] = masks left in the window, status[1] = positions unmasked.
__global__ void unmask_kernel(const int* __restrict__ ids, const float* __restrict__ maxp, int rows, int* block,
                              int sub_start, int sub_len, int partial, int mask_id, double threshold, int* out_tok,
                              float* out_conf, int* out_unmask, int* status) {
  pdl_trigger();
  pdl_wait();
  const int j = threadIdx.x;  // window position
  const bool in = j < sub_len;
  int tok = 0;
  float conf = -INFINITY;
  bool masked = false;
  if (in) {
    const int src_row = partial ? j : sub_start + j;       // row of the shifted array
    const int row = src_row > 0 ? src_row - 1 : 0;          // its unshifted source row
    if (row < rows) {
      tok = ids[row];
      conf = maxp[row];
    }
    masked = block[sub_start + j] == mask_id;
  }
  const bool above = masked && static_cast<double>(conf) > threshold;
  const unsigned any_above = __ballot_sync(0xffffffffu, above);
  bool take = above;
  if (any_above == 0u) {
    // first masked position with the largest confidence (np.argmax over the masked list)
    float best = masked ? conf : -INFINITY;
    int best_j = masked ? j : 0x7fffffff;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      const float ob = __shfl_xor_sync(0xffffffffu, best, off);
      const int oj = __shfl_xor_sync(0xffffffffu, best_j, off);
      if (ob > best || (ob == best && oj < best_j)) { best = ob; best_j = oj; }
    }
    take = masked && (j == best_j);
  }
  if (in) {
    if (take) block[sub_start + j] = tok;
    if (out_tok) out_tok[j] = tok;
    if (out_conf) out_conf[j] = conf;
    if (out_unmask) out_unmask[j] = take ? 1 : 0;
  }
  const unsigned left = __ballot_sync(0xffffffffu, masked && !take);
  const unsigned took = __ballot_sync(0xffffffffu, take);
  if (j == 0 && status) {
    status[0] = __popc(left);
    status[1] = __popc(took);
  }
}

int launch_unmask(const int* ids, const float* maxp, int rows, int* block, int sub_start, int sub_len, int partial,
                  int mask_id, double threshold, int* out_tok, float* out_conf, int* out_unmask, int* status,
                  cudaStream_t s) {
  if (sub_len <= 0 || sub_len > 32) return cudaErrorInvalidValue;
  return launch_k(unmask_kernel, dim3(1), dim3(32), 0, s, ids, maxp, rows, block, sub_start, sub_len, partial, mask_id,
                  threshold, out_tok, out_conf, out_unmask, status);
}

// ---- unmask decisions of a batched step, one warp per request ---------------------------------
// The rule of unmask_kernel for many requests whose rows share one ids / maxp array.  desc[5 i ..]:
// row0, rows (the request's rows in ids / maxp), base (window row 0 takes shifted row `base`: 0 for
// a partial step, the sub-block start for a full one), win (window length, 0 = no decision: a block
// append) and the bit mask of the window rows still masked.  out[34 i ..]: the bit mask of the rows
// unmasked, the last row's unshifted argmax (the token after the block, runtime.py:181), then the
// shifted token of each window row.  The block itself stays on the host, which applies the bits.
__global__ void unmask_batch_kernel(const int* __restrict__ ids, const float* __restrict__ maxp,
                                    const int* __restrict__ desc, int n, double threshold, int* __restrict__ out) {
  pdl_trigger();
  pdl_wait();
  const int i = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int j = threadIdx.x & 31;
  if (i >= n) return;
  const int row0 = desc[5 * i], rows = desc[5 * i + 1], base = desc[5 * i + 2], win = desc[5 * i + 3];
  const unsigned bits = static_cast<unsigned>(desc[5 * i + 4]);
  int tok = 0;
  float conf = -INFINITY;
  bool masked = false;
  if (j < win) {
    const int src_row = base + j;
    const int row = src_row > 0 ? src_row - 1 : 0;
    if (row < rows) {
      tok = ids[row0 + row];
      conf = maxp[row0 + row];
    }
    masked = (bits >> j) & 1u;
  }
  const bool above = masked && static_cast<double>(conf) > threshold;
  bool take = above;
  if (__ballot_sync(0xffffffffu, above) == 0u) {
    float best = masked ? conf : -INFINITY;
    int best_j = masked ? j : 0x7fffffff;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      const float ob = __shfl_xor_sync(0xffffffffu, best, off);
      const int oj = __shfl_xor_sync(0xffffffffu, best_j, off);
      if (ob > best || (ob == best && oj < best_j)) {
        best = ob;
        best_j = oj;
      }
    }
    take = masked && j == best_j;
  }
  const unsigned took = __ballot_sync(0xffffffffu, take);
  int* o = out + 34 * i;
  if (j == 0) {
    o[0] = static_cast<int>(took);
    o[1] = rows > 0 ? ids[row0 + rows - 1] : 0;
  }
  if (j < win) o[2 + j] = tok;
}

int launch_unmask_batch(const int* ids, const float* maxp, const int* desc, int n, double threshold, int* out,
                        cudaStream_t s) {
  if (n <= 0) return cudaSuccess;
  return launch_k(unmask_batch_kernel, dim3((n + 7) / 8), dim3(256), 0, s, ids, maxp, desc, n, threshold, out);
}

// ---- bounded-wait self test: spin on a flag that nothing sets; give up and report ----------
__global__ void wait_test_kernel(const volatile int* flag, int* err, unsigned long long limit_ns) {
  const uint64_t t0 = global_timer_ns();
  while (*flag == 0) {
    if (global_timer_ns() - t0 > limit_ns) {
      report_error(err, kErrTimeoutTest);
      return;
    }
    __nanosleep(1000);
  }
}

int launch_wait_test(int* flag, int* err, unsigned long long limit_ns, cudaStream_t s) {
  wait_test_kernel<<<1, 1, 0, s>>>(flag, err, limit_ns);
  count_launch();
  return cudaGetLastError();
}

}  // namespace fdllm
