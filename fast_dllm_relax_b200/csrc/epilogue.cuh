// GEMM epilogues shared by the tcgen05 kernel (bf16) and the SIMT kernel (fp32).
//
// Both kernels first gather one output tile into shared memory as fp32 `acc[t][f]`
// (t = token within the tile, f = one of the 128 weight rows of slab `slab`), then call
// gemm_epilogue<T>, which applies the op that follows the projection in the reference graph with
// the reference's rounding order (each bf16 op computed in fp32 and rounded back):
//   qkv_proj + bias -> RoPE on q and k -> KV-cache append   model/cuda.py:389-399, 303-316; runtime.py:51-60
//   o_proj / down_proj + residual add                        model/cuda.py:546-547, 577-578
//   gate_up_proj -> SiLU(gate) (fp32) * up                   model/cuda.py:319-328, 343-347
//   lm_head -> fp32 logits                                   model/cuda.py:704-711
//   lm_head -> per-slab (max, first argmax, sum exp)          model/metal.py:316-374 (confidence)
//
// Memory access shape: every thread works on 16-byte chunks (8 bf16 / 4 fp32 consecutive features
// of one token) and issues the global loads of a batch of chunks before any of that batch's stores,
// so a thread pays one memory latency per batch instead of one per element.
#pragma once

#include "common.cuh"
#include "kernels.h"

namespace fdllm {

template <typename T>
struct Chunk {
  static constexpr int V = 16 / sizeof(T);  // elements per 16-byte chunk
  union {
    uint4 u;
    T e[V];
  };
};

// L2-only load (ld.global.cg): the persistent layer-stack kernel re-reads buffers that other CTAs
// rewrite between its phases, so no epilogue may be served a stale line from this SM's L1.
template <typename T>
__device__ __forceinline__ Chunk<T> ld_chunk(const T* p) {
  Chunk<T> c;
  c.u = __ldcg(reinterpret_cast<const uint4*>(p));
  return c;
}

// Read-only-path load (ld.global.nc) for tables that no kernel writes (bias, RoPE): the chunks
// that several tokens share stay in L1.
template <typename T>
__device__ __forceinline__ Chunk<T> ld_const_chunk(const T* p) {
  Chunk<T> c;
  c.u = __ldg(reinterpret_cast<const uint4*>(p));
  return c;
}

template <typename T>
__device__ __forceinline__ void st_chunk(T* p, const Chunk<T>& c) {
  *reinterpret_cast<uint4*>(p) = c.u;
}

// Two values rounded to the model dtype and widened back (one packed conversion for bf16).
template <typename T> __device__ __forceinline__ float2 round_pair(float a, float b);
template <> __device__ __forceinline__ float2 round_pair<float>(float a, float b) { return make_float2(a, b); }
template <> __device__ __forceinline__ float2 round_pair<bf16>(float a, float b) { return round2_bf16(a, b); }

// dst[0], dst[1] = T(a), T(b) (one packed conversion for bf16).
template <typename T> __device__ __forceinline__ void set_pair(T* dst, float a, float b);
template <> __device__ __forceinline__ void set_pair<float>(float* dst, float a, float b) {
  dst[0] = a;
  dst[1] = b;
}
template <> __device__ __forceinline__ void set_pair<bf16>(bf16* dst, float a, float b) {
  *reinterpret_cast<__nv_bfloat162*>(dst) = __floats2bfloat162_rn(a, b);
}

constexpr int kEpiBatch = 4;  // chunks in flight per thread

// SiLU(g) = g * sigmoid(g) in fp32 (model/cuda.py:319-328).  bf16: the approximate exponential and
// reciprocal (a few ulp of fp32, far below the bf16 rounding that follows) -- the IEEE division's
// special-case branch serialises the independent element chains of a chunk.  fp32 keeps IEEE.
template <typename T> __device__ __forceinline__ float silu_f(float g);
template <> __device__ __forceinline__ float silu_f<float>(float g) { return g * (1.0f / (1.0f + expf(-g))); }
template <> __device__ __forceinline__ float silu_f<bf16>(float g) { return g * __fdividef(1.0f, 1.0f + __expf(-g)); }

// V consecutive fp32 accumulator values (16-byte aligned) with 16-byte shared-memory loads: the
// chunk pattern of the epilogues (8 chunks of one token row per 8 lanes) costs a 2-way bank
// conflict per 128-bit load instead of an 8-way conflict per scalar load.
template <int V>
__device__ __forceinline__ void ld_acc(const float* p, float (&x)[V]) {
  static_assert(V % 4 == 0, "whole float4s");
#pragma unroll
  for (int i = 0; i < V / 4; ++i) {
    const float4 q = reinterpret_cast<const float4*>(p)[i];
    x[4 * i] = q.x;
    x[4 * i + 1] = q.y;
    x[4 * i + 2] = q.z;
    x[4 * i + 3] = q.w;
  }
}

// Epilogue inputs that do not depend on the accumulator, loaded before it is ready so that their
// latency overlaps the main loop's tail and the split-K reduction.  Only when each thread owns at
// most kEpiPre chunks (chunks cbeg + tid + b * nthr, b < kEpiPre); n = 0 otherwise.  One chunk
// covers every decode-sized split-K tile and keeps the GEMM at its former register count: a GEMM
// CTA must still fit beside an attention CTA on an SM for programmatic launch to overlap them.
constexpr int kEpiPre = 1;
template <typename T>
struct EpiPre {
  int n = 0;
  Chunk<T> a[kEpiPre];                // residual: resid chunk; qkv: bias chunk
  Chunk<T> b[kEpiPre];                // qkv: bias chunk of the RoPE partner features
  Chunk<T> cs[kEpiPre], sn[kEpiPre];  // qkv: RoPE tables at the token's position
  T* dst[kEpiPre];                    // qkv: q row, or the request's K / V cache row (null: none)
};

template <typename T>
__device__ void epi_prefetch(const GemmArgs& g, int tok0, int slab, int row0, int row1, int tid, int nthr,
                             EpiPre<T>& p) {
  const Epilogue& e = g.epi;
  constexpr int V = Chunk<T>::V;
  constexpr int CPR = 128 / V;
  const int cbeg = row0 * CPR, cend = row1 * CPR;
  p.n = 0;
  if (cend - cbeg > nthr * kEpiPre) return;
  if (e.kind == kEpiResidual) {
    const T* hs = e.resid_src ? static_cast<const T*>(e.resid_src) : static_cast<const T*>(e.resid);
#pragma unroll
    for (int b = 0; b < kEpiPre; ++b) {
      const int c = cbeg + tid + b * nthr;
      const int t = c / CPR, f0 = (c % CPR) * V, tok = tok0 + t, F0 = slab * 128 + f0;
      if (c < cend && tok < g.M && F0 < g.N) p.a[b] = ld_chunk(hs + (size_t)tok * e.ld_resid + F0);
    }
    p.n = kEpiPre;
  } else if (e.kind == kEpiQkvRope) {
    const T* bias = static_cast<const T*>(e.bias);
    const int hd = e.hd, half = e.hd >> 1;
#pragma unroll
    for (int b = 0; b < kEpiPre; ++b) {
      p.dst[b] = nullptr;
      const int c = cbeg + tid + b * nthr;
      const int t = c / CPR, f0 = (c % CPR) * V, tok = tok0 + t, F0 = slab * 128 + f0;
      if (c >= cend || tok >= g.M || F0 >= g.N) continue;
      const int head = F0 / hd, d0 = F0 - head * hd;
      p.a[b] = ld_const_chunk(bias + F0);
      if (head < e.hq + e.hkv) {
        int pos = e.tok.pos[tok];
        pos = pos < 0 ? 0 : (pos >= e.max_pos ? e.max_pos - 1 : pos);  // range checked in prepare
        const bool lo = d0 < half;
        p.b[b] = ld_const_chunk(bias + (lo ? F0 + half : F0 - half));
        const size_t ti = (size_t)pos * half + (lo ? d0 : d0 - half);
        p.cs[b] = ld_const_chunk(static_cast<const T*>(e.rope_cos) + ti);
        p.sn[b] = ld_const_chunk(static_cast<const T*>(e.rope_sin) + ti);
      }
      if (head < e.hq) {
        p.dst[b] = static_cast<T*>(e.qout) + (size_t)tok * (e.hq * hd) + F0;
      } else {
        const ReqDesc& r = e.reqs[e.tok.req[tok]];
        const int row = e.tok.row[tok];
        if (row >= 0 && row < r.cap) {
          const size_t off = (size_t)e.layer * r.layer_stride + (size_t)row * e.hkv * hd;
          p.dst[b] = head < e.hq + e.hkv ? static_cast<T*>(r.k) + off + (head - e.hq) * hd + d0
                                         : static_cast<T*>(r.v) + off + (head - e.hq - e.hkv) * hd + d0;
        }
      }
    }
    p.n = kEpiPre;
  }
}

// Per-token destinations of a qkv tile's rows [t0, t1) into s_epi (RoPE position, the K and V
// cache row bases of this layer, null where the token has no cache row), so that the element loop
// of the epilogue carries no dependent global loads.  l2: also prefetch each token's K and V rows
// into L2, for a caller that builds them while the main loop still runs: the epilogue's stores
// then find their lines and address translations warm (one step of 32 requests scatters each
// layer's rows over 64 cache allocations).
template <typename T>
__device__ void qkv_dest_setup(const GemmArgs& g, int tok0, int t0, int t1, unsigned char* s_epi, int tid, int nthr,
                               bool l2) {
  const Epilogue& e = g.epi;
  int* s_pos = reinterpret_cast<int*>(s_epi);              // [256]
  T** s_kb = reinterpret_cast<T**>(s_epi + 1024);         // [256]
  T** s_vb = reinterpret_cast<T**>(s_epi + 1024 + 2048);  // [256]
  for (int t = t0 + tid; t < t1; t += nthr) {
    const int tok = tok0 + t;
    T* kb = nullptr;
    T* vb = nullptr;
    int pos = 0;
    if (tok < g.M) {
      pos = e.tok.pos[tok];
      pos = pos < 0 ? 0 : (pos >= e.max_pos ? e.max_pos - 1 : pos);  // range checked in prepare
      const ReqDesc& r = e.reqs[e.tok.req[tok]];
      const int row = e.tok.row[tok];
      if (row >= 0 && row < r.cap) {
        const size_t off = (size_t)e.layer * r.layer_stride + (size_t)row * e.hkv * e.hd;
        kb = static_cast<T*>(r.k) + off;
        vb = static_cast<T*>(r.v) + off;
        if (l2) {
          const int bytes = e.hkv * e.hd * static_cast<int>(sizeof(T));
          for (int o = 0; o < bytes; o += 128) {
            asm volatile("prefetch.global.L2 [%0];" ::"l"(reinterpret_cast<const char*>(kb) + o));
            asm volatile("prefetch.global.L2 [%0];" ::"l"(reinterpret_cast<const char*>(vb) + o));
          }
        }
      }
    }
    s_pos[t] = pos;
    s_kb[t] = kb;
    s_vb[t] = vb;
  }
}

// Rows [row0, row1) of the tile are processed (a split-K cluster member owns a share of the rows).
// s_epi: 5120 bytes of shared scratch owned by the calling kernel.  The calling threads are
// tid = 0..nthr-1 (a multiple of 32); they synchronise with named barrier `bar_id` (0 with
// nthr == blockDim.x is __syncthreads()).
// pre: inputs loaded by epi_prefetch for the same rows and threads, or null.
// setup0 / setup1 (QkvRope): the tile rows whose per-token destinations are (re)built into s_epi
// by this call; -1 (default) = [row0, row1).  A caller that walks one tile in chunks builds them
// for the whole tile with its first chunk and passes an empty range afterwards.
template <typename T>
__device__ void gemm_epilogue(const GemmArgs& g, float* acc, int nt, int tok0, int slab, int row0, int row1,
                              unsigned char* s_epi, int tid, int nthr, int bar_id, const EpiPre<T>* pre = nullptr,
                              int setup0 = -1, int setup1 = -1) {
  const Epilogue& e = g.epi;
  const bool have_pre = pre != nullptr && pre->n > 0;
  constexpr int V = Chunk<T>::V;
  constexpr int CPR = 128 / V;  // chunks per 128-feature row of the tile
  const int cbeg = row0 * CPR, cend = row1 * CPR;

  switch (e.kind) {
    case kEpiStore: {
      T* out = static_cast<T*>(e.out);
      for (int c = cbeg + tid; c < cend; c += nthr) {
        const int t = c / CPR, f0 = (c % CPR) * V, tok = tok0 + t, F0 = slab * 128 + f0;
        if (tok >= g.M || F0 >= g.N) continue;
        Chunk<T> o;
        float x[V];
        ld_acc<V>(acc + t * 128 + f0, x);
#pragma unroll
        for (int v = 0; v < V; v += 2) set_pair<T>(&o.e[v], x[v], x[v + 1]);
        st_chunk(out + (size_t)tok * e.ld_out + F0, o);
      }
      break;
    }
    case kEpiLogitsF32: {
      float* out = static_cast<float*>(e.out);
      for (int c = row0 * 32 + tid; c < row1 * 32; c += nthr) {  // float4 chunks
        const int t = c >> 5, f0 = (c & 31) * 4, tok = tok0 + t, F0 = slab * 128 + f0;
        if (tok >= g.M || F0 >= g.N) continue;
        const float* a = acc + t * 128 + f0;
        const float2 lo = round_pair<T>(a[0], a[1]), hi = round_pair<T>(a[2], a[3]);
        *reinterpret_cast<float4*>(out + (size_t)tok * e.ld_out + F0) = make_float4(lo.x, lo.y, hi.x, hi.y);
      }
      break;
    }
    case kEpiResidual: {
      T* h = static_cast<T*>(e.resid);
      const T* hs = e.resid_src ? static_cast<const T*>(e.resid_src) : h;
      float* s_ss = reinterpret_cast<float*>(s_epi);  // [nt <= 64][CPR] chunk sums of squares
      const bool want_ss = e.ss_out != nullptr && nt <= 64;
      // the chunk's residual add, rounded as the reference rounds it, and its sum of squares
      auto finish = [&](int c, const Chunk<T>& r) {
        const int t = c / CPR, f0 = (c % CPR) * V, tok = tok0 + t, F0 = slab * 128 + f0;
        Chunk<T> o;
        float ss = 0.f;
        float x[V];
        ld_acc<V>(acc + t * 128 + f0, x);
#pragma unroll
        for (int v = 0; v < V; v += 2) {
          const float2 y = round_pair<T>(x[v], x[v + 1]);
          const float2 z = round_pair<T>(to_f<T>(r.e[v]) + y.x, to_f<T>(r.e[v + 1]) + y.y);
          set_pair<T>(&o.e[v], z.x, z.y);
          ss = fmaf(z.x, z.x, ss);
          ss = fmaf(z.y, z.y, ss);
        }
        st_chunk(h + (size_t)tok * e.ld_resid + F0, o);
        if (want_ss) s_ss[t * CPR + (c % CPR)] = ss;
      };
      // prefetched (decode): each thread owns at most kEpiPre chunks, so no batch loop -- a short
      // code path for a latency-bound launch whose instructions arrive cold
      for (int b = 0; have_pre && b < kEpiPre; ++b) {
        const int c = cbeg + tid + b * nthr;
        const int t = c / CPR, F0 = slab * 128 + (c % CPR) * V;
        if (c < cend && tok0 + t < g.M && F0 < g.N) finish(c, pre->a[b]);
      }
      // otherwise a rolled loop over the thread's chunks with the next two chunks' residual loads
      // in flight: one chunk of code, whose instructions a large call fetches cold
      if (!have_pre) {
        auto load = [&](int c, Chunk<T>& r) {
          const int t = c / CPR, tok = tok0 + t, F0 = slab * 128 + (c % CPR) * V;
          if (c < cend && tok < g.M && F0 < g.N) r = ld_chunk(hs + (size_t)tok * e.ld_resid + F0);
        };
        Chunk<T> r1, r2;
        r1.u = r2.u = make_uint4(0u, 0u, 0u, 0u);
        load(cbeg + tid, r1);
        load(cbeg + tid + nthr, r2);
#pragma unroll 1
        for (int c = cbeg + tid; c < cend; c += nthr) {
          const Chunk<T> r = r1;
          r1 = r2;
          load(c + 2 * nthr, r2);
          const int t = c / CPR, F0 = slab * 128 + (c % CPR) * V;
          if (tok0 + t < g.M && F0 < g.N) finish(c, r);
        }
      }
      if (want_ss) {  // per-row sum over this slab's 128 features, in chunk order (deterministic)
        named_sync(bar_id, nthr);
        for (int t = row0 + tid; t < row1; t += nthr) {
          const int tok = tok0 + t;
          if (tok >= g.M) continue;
          float ss = 0.f;
          for (int j = 0; j < CPR; ++j) ss += s_ss[t * CPR + j];
          e.ss_out[(size_t)tok * e.ss_ld + slab] = ss;
        }
      }
      break;
    }
    case kEpiSiluMul: {
      T* out = static_cast<T*>(e.out);
      const int inter = g.N / 2;
      constexpr int CPH = 64 / V;  // chunks per 64-feature half
      for (int c = row0 * CPH + tid; c < row1 * CPH; c += nthr) {
        const int t = c / CPH, f0 = (c % CPH) * V, tok = tok0 + t, j0 = slab * 64 + f0;
        if (tok >= g.M || j0 >= inter) continue;
        Chunk<T> o;
        float gx[V], ux[V];
        ld_acc<V>(acc + t * 128 + f0, gx);
        ld_acc<V>(acc + t * 128 + 64 + f0, ux);
#pragma unroll
        for (int v = 0; v < V; v += 2) {
          const float2 gate = round_pair<T>(gx[v], gx[v + 1]);
          const float2 up = round_pair<T>(ux[v], ux[v + 1]);
          const float2 act = round_pair<T>(silu_f<T>(gate.x), silu_f<T>(gate.y));
          set_pair<T>(&o.e[v], act.x * up.x, act.y * up.y);
        }
        st_chunk(out + (size_t)tok * e.ld_out + j0, o);
      }
      break;
    }
    case kEpiQkvRope: {
      if (have_pre) {  // one pass: the partner features' biased values are recomputed, no barrier
        const int hd = e.hd, half = e.hd >> 1;
#pragma unroll
        for (int b = 0; b < kEpiPre; ++b) {
          const int c = cbeg + tid + b * nthr;
          const int t = c / CPR, f0 = (c % CPR) * V, tok = tok0 + t, F0 = slab * 128 + f0;
          if (c >= cend || tok >= g.M || F0 >= g.N || pre->dst[b] == nullptr) continue;
          const int head = F0 / hd, d0 = F0 - head * hd;
          float x[V];
          ld_acc<V>(acc + t * 128 + f0, x);
          Chunk<T> o;
          if (head < e.hq + e.hkv) {
            const bool lo = d0 < half;
            float xp[V];
            ld_acc<V>(acc + t * 128 + (lo ? f0 + half : f0 - half), xp);
#pragma unroll
            for (int v = 0; v < V; v += 2) {
              const float2 y = round_pair<T>(x[v] + to_f<T>(pre->a[b].e[v]), x[v + 1] + to_f<T>(pre->a[b].e[v + 1]));
              const float2 yp = round_pair<T>(xp[v] + to_f<T>(pre->b[b].e[v]), xp[v + 1] + to_f<T>(pre->b[b].e[v + 1]));
              const float r0 = lo ? -yp.x : yp.x, r1 = lo ? -yp.y : yp.y;
              const float2 cv = round_pair<T>(y.x * to_f<T>(pre->cs[b].e[v]), y.y * to_f<T>(pre->cs[b].e[v + 1]));
              const float2 sv = round_pair<T>(r0 * to_f<T>(pre->sn[b].e[v]), r1 * to_f<T>(pre->sn[b].e[v + 1]));
              set_pair<T>(&o.e[v], cv.x + sv.x, cv.y + sv.y);  // T(round(c + s)) == T(c + s)
            }
          } else {
#pragma unroll
            for (int v = 0; v < V; v += 2) {
              const float2 y = round_pair<T>(x[v] + to_f<T>(pre->a[b].e[v]), x[v + 1] + to_f<T>(pre->a[b].e[v + 1]));
              set_pair<T>(&o.e[v], y.x, y.y);
            }
          }
          st_chunk(pre->dst[b], o);
        }
        break;
      }
      if (setup0 < 0) {
        setup0 = row0;
        setup1 = row1;
      }
      qkv_dest_setup<T>(g, tok0, setup0, setup1, s_epi, tid, nthr, false);
      int* s_pos = reinterpret_cast<int*>(s_epi);
      T** s_kb = reinterpret_cast<T**>(s_epi + 1024);
      T** s_vb = reinterpret_cast<T**>(s_epi + 1024 + 2048);
      const T* bias = static_cast<const T*>(e.bias);
      if (setup1 > setup0) named_sync(bar_id, nthr);  // the destinations are visible
      // One pass over the chunks: a chunk's bias, and its RoPE partner's, are added and rounded
      // here (the partner's value recomputed from the accumulator, as the prefetched path above
      // does), so the tile needs neither a rounding pass nor a barrier between the two.  When nthr
      // is a multiple of CPR (the tcgen05 kernels' 128 and 256 threads) every chunk of a thread
      // covers the same 8 features, and its two bias chunks are loaded once.
      const int hd = e.hd, half = e.hd >> 1, hq = e.hq, hkv = e.hkv;
      const T* cos_t = static_cast<const T*>(e.rope_cos);
      const T* sin_t = static_cast<const T*>(e.rope_sin);
      T* q = static_cast<T*>(e.qout);
      auto load_bias = [&](int c, Chunk<T>& a, Chunk<T>& bp) {
        const int F0 = slab * 128 + (c % CPR) * V;
        if (F0 >= g.N) return;
        const int head = F0 / hd, d0 = F0 - head * hd;
        a = ld_const_chunk(bias + F0);
        if (head < hq + hkv) bp = ld_const_chunk(bias + (d0 < half ? F0 + half : F0 - half));
      };
      const bool fixed = nthr % CPR == 0;
      Chunk<T> ba, bb;
      ba.u = bb.u = make_uint4(0u, 0u, 0u, 0u);
      if (fixed) load_bias(cbeg + tid, ba, bb);
      // A rolled loop, the next chunk's table loads issued before this chunk's arithmetic: the body
      // is one chunk of code.  (A batch of chunks unrolled is several KB of straight-line code that
      // a large call fetches cold into the instruction cache, the other kernels of a layer having
      // run in between: its first batch took 7 of a 10 us epilogue at 1024 rows.)
      auto load_tables = [&](int c, Chunk<T>& cs, Chunk<T>& sn) {
        const int t = c / CPR, f0 = (c % CPR) * V, F0 = slab * 128 + f0;
        if (c >= cend || tok0 + t >= g.M || F0 >= g.N) return;
        const int head = F0 / hd, d0 = F0 - head * hd;
        if (head < hq + hkv) {
          const size_t ti = (size_t)s_pos[t] * half + (d0 < half ? d0 : d0 - half);
          cs = ld_const_chunk(cos_t + ti);
          sn = ld_const_chunk(sin_t + ti);
        }
      };
      Chunk<T> cs_n, sn_n;
      cs_n.u = sn_n.u = make_uint4(0u, 0u, 0u, 0u);
      load_tables(cbeg + tid, cs_n, sn_n);
#pragma unroll 1
      for (int c = cbeg + tid; c < cend; c += nthr) {
        const Chunk<T> cs = cs_n, sn = sn_n;
        load_tables(c + nthr, cs_n, sn_n);
        const int t = c / CPR, f0 = (c % CPR) * V, tok = tok0 + t, F0 = slab * 128 + f0;
        if (tok >= g.M || F0 >= g.N) continue;
        const int head = F0 / hd, d0 = F0 - head * hd;
        Chunk<T> a = ba, bp = bb;
        if (!fixed) load_bias(c, a, bp);
        float x[V];
        ld_acc<V>(acc + t * 128 + f0, x);
        Chunk<T> o;
        if (head < hq + hkv) {
          const bool lo = d0 < half;
          float xp[V];
          ld_acc<V>(acc + t * 128 + (lo ? f0 + half : f0 - half), xp);
#pragma unroll
          for (int v = 0; v < V; v += 2) {
            const float2 y = round_pair<T>(x[v] + to_f<T>(a.e[v]), x[v + 1] + to_f<T>(a.e[v + 1]));
            const float2 yp = round_pair<T>(xp[v] + to_f<T>(bp.e[v]), xp[v + 1] + to_f<T>(bp.e[v + 1]));
            const float r0 = lo ? -yp.x : yp.x, r1 = lo ? -yp.y : yp.y;
            const float2 cv = round_pair<T>(y.x * to_f<T>(cs.e[v]), y.y * to_f<T>(cs.e[v + 1]));
            const float2 sv = round_pair<T>(r0 * to_f<T>(sn.e[v]), r1 * to_f<T>(sn.e[v + 1]));
            set_pair<T>(&o.e[v], cv.x + sv.x, cv.y + sv.y);  // T(round(c + s)) == T(c + s)
          }
          if (head < hq) {
            st_chunk(q + (size_t)tok * (hq * hd) + F0, o);
          } else if (s_kb[t] != nullptr) {
            st_chunk(s_kb[t] + (head - hq) * hd + d0, o);
          }
        } else if (s_vb[t] != nullptr) {
#pragma unroll
          for (int v = 0; v < V; v += 2) {
            const float2 y = round_pair<T>(x[v] + to_f<T>(a.e[v]), x[v + 1] + to_f<T>(a.e[v + 1]));
            set_pair<T>(&o.e[v], y.x, y.y);
          }
          st_chunk(s_vb[t] + (head - hq - hkv) * hd + d0, o);
        }
      }
      break;
    }
    case kEpiConf:
    case kEpiLseGather: {
      const int warp = tid >> 5, lane = tid & 31, nwarps = nthr >> 5;
      for (int t = row0 + warp; t < row1; t += nwarps) {
        const int tok = tok0 + t;
        if (tok >= g.M) continue;
        float best = -INFINITY;
        int best_i = 0x7fffffff;
        float vals[4];
        {
          const float2 p0 = round_pair<T>(acc[t * 128 + lane], acc[t * 128 + lane + 32]);
          const float2 p1 = round_pair<T>(acc[t * 128 + lane + 64], acc[t * 128 + lane + 96]);
          vals[0] = p0.x;
          vals[1] = p0.y;
          vals[2] = p1.x;
          vals[3] = p1.y;
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int f = lane + 32 * i;
          const int F = slab * 128 + f;
          if (F < g.N) {
            const float v = vals[i];
            if (v > best || (v == best && F < best_i)) { best = v; best_i = F; }
          }
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
          const float ob = __shfl_xor_sync(0xffffffffu, best, off);
          const int oi = __shfl_xor_sync(0xffffffffu, best_i, off);
          if (ob > best || (ob == best && oi < best_i)) { best = ob; best_i = oi; }
        }
        float sum = 0.f;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int f = lane + 32 * i;
          if (slab * 128 + f < g.N) sum += expf(vals[i] - best);
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
        if (lane == 0) {
          float tv = 0.f;
          if (e.kind == kEpiLseGather) {
            const int tg = e.target[tok] - slab * 128;
            tv = (tg >= 0 && tg < 128) ? round_t<T>(acc[t * 128 + tg]) : 0.f;
          }
          *reinterpret_cast<float4*>(e.part + ((size_t)tok * g.n_slabs + slab) * 4) =
              make_float4(best, __int_as_float(best_i), sum, tv);
        }
      }
      break;
    }
    default:
      break;
  }
}

template <typename T>
__device__ __forceinline__ void gemm_epilogue(const GemmArgs& g, float* acc, int nt, int tok0, int slab, int row0,
                                              int row1, unsigned char* s_epi) {
  gemm_epilogue<T>(g, acc, nt, tok0, slab, row0, row1, s_epi, static_cast<int>(threadIdx.x),
                   static_cast<int>(blockDim.x), 0);
}

}  // namespace fdllm
