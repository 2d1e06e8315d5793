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

template <typename T>
__device__ __forceinline__ Chunk<T> ld_chunk(const T* p) {
  Chunk<T> c;
  c.u = *reinterpret_cast<const uint4*>(p);
  return c;
}

template <typename T>
__device__ __forceinline__ void st_chunk(T* p, const Chunk<T>& c) {
  *reinterpret_cast<uint4*>(p) = c.u;
}

constexpr int kEpiBatch = 4;  // chunks in flight per thread

// Rows [row0, row1) of the tile are processed (a split-K cluster member owns a share of the rows).
template <typename T>
// s_epi: 5120 bytes of shared scratch owned by the calling kernel.
__device__ void gemm_epilogue(const GemmArgs& g, float* acc, int nt, int tok0, int slab, int row0, int row1,
                              unsigned char* s_epi) {
  const Epilogue& e = g.epi;
  const int nthr = blockDim.x;
  const int tid = threadIdx.x;
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
#pragma unroll
        for (int v = 0; v < V; ++v) o.e[v] = from_f<T>(acc[t * 128 + f0 + v]);
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
        *reinterpret_cast<float4*>(out + (size_t)tok * e.ld_out + F0) =
            make_float4(round_t<T>(a[0]), round_t<T>(a[1]), round_t<T>(a[2]), round_t<T>(a[3]));
      }
      break;
    }
    case kEpiResidual: {
      T* h = static_cast<T*>(e.resid);
      const T* hs = e.resid_src ? static_cast<const T*>(e.resid_src) : h;
      float* s_ss = reinterpret_cast<float*>(s_epi);  // [nt <= 64][CPR] chunk sums of squares
      const bool want_ss = e.ss_out != nullptr && nt <= 64;
      for (int c0 = cbeg + tid; c0 < cend; c0 += nthr * kEpiBatch) {
        Chunk<T> r[kEpiBatch];
#pragma unroll
        for (int b = 0; b < kEpiBatch; ++b) {  // loads first
          const int c = c0 + b * nthr;
          const int t = c / CPR, f0 = (c % CPR) * V, tok = tok0 + t, F0 = slab * 128 + f0;
          if (c < cend && tok < g.M && F0 < g.N) r[b] = ld_chunk(hs + (size_t)tok * e.ld_resid + F0);
        }
#pragma unroll
        for (int b = 0; b < kEpiBatch; ++b) {
          const int c = c0 + b * nthr;
          const int t = c / CPR, f0 = (c % CPR) * V, tok = tok0 + t, F0 = slab * 128 + f0;
          if (c >= cend || tok >= g.M || F0 >= g.N) continue;
          Chunk<T> o;
          float ss = 0.f;
#pragma unroll
          for (int v = 0; v < V; ++v) {
            o.e[v] = from_f<T>(to_f<T>(r[b].e[v]) + round_t<T>(acc[t * 128 + f0 + v]));
            const float f = to_f<T>(o.e[v]);
            ss = fmaf(f, f, ss);
          }
          st_chunk(h + (size_t)tok * e.ld_resid + F0, o);
          if (want_ss) s_ss[t * CPR + (c % CPR)] = ss;
        }
      }
      if (want_ss) {  // per-row sum over this slab's 128 features, in chunk order (deterministic)
        __syncthreads();
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
#pragma unroll
        for (int v = 0; v < V; ++v) {
          const float gate = round_t<T>(acc[t * 128 + f0 + v]);
          const float up = round_t<T>(acc[t * 128 + 64 + f0 + v]);
          const float act = round_t<T>(gate * (1.0f / (1.0f + expf(-gate))));
          o.e[v] = from_f<T>(act * up);
        }
        st_chunk(out + (size_t)tok * e.ld_out + j0, o);
      }
      break;
    }
    case kEpiQkvRope: {
      // Per-token destinations (RoPE position, cache row, K / V bases) once per tile, in shared
      // memory, so the element loop below carries no dependent global loads.
      int* s_pos = reinterpret_cast<int*>(s_epi);                 // [256]
      T** s_kb = reinterpret_cast<T**>(s_epi + 1024);            // [256]
      T** s_vb = reinterpret_cast<T**>(s_epi + 1024 + 2048);     // [256]
      const T* bias = static_cast<const T*>(e.bias);
      for (int t = row0 + tid; t < row1; t += nthr) {
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
          }
        }
        s_pos[t] = pos;
        s_kb[t] = kb;
        s_vb[t] = vb;
      }
      // Phase 1: projection + bias, rounded to the model dtype (the op's output tensor).
      for (int idx = row0 * 128 + tid; idx < row1 * 128; idx += nthr) {
        const int F = slab * 128 + (idx & 127);
        if (F < g.N) acc[idx] = round_t<T>(acc[idx] + to_f<T>(bias[F]));
      }
      __syncthreads();
      // Phase 2: rotate q and k (partner element d +- hd/2 of the same head, inside this slab),
      // scatter q to qout and k / v to the request's cache row.
      const int hd = e.hd, half = e.hd >> 1, hq = e.hq, hkv = e.hkv;
      const T* cos_t = static_cast<const T*>(e.rope_cos);
      const T* sin_t = static_cast<const T*>(e.rope_sin);
      T* q = static_cast<T*>(e.qout);
      for (int c0 = cbeg + tid; c0 < cend; c0 += nthr * kEpiBatch) {
        Chunk<T> cs[kEpiBatch], sn[kEpiBatch];
#pragma unroll
        for (int b = 0; b < kEpiBatch; ++b) {  // table loads first
          const int c = c0 + b * nthr;
          const int t = c / CPR, f0 = (c % CPR) * V, F0 = slab * 128 + f0;
          if (c >= cend || tok0 + t >= g.M || F0 >= g.N) continue;
          const int head = F0 / hd, d0 = F0 - head * hd;
          if (head < hq + hkv) {
            const size_t ti = (size_t)s_pos[t] * half + (d0 < half ? d0 : d0 - half);
            cs[b] = ld_chunk(cos_t + ti);
            sn[b] = ld_chunk(sin_t + ti);
          }
        }
#pragma unroll
        for (int b = 0; b < kEpiBatch; ++b) {
          const int c = c0 + b * nthr;
          const int t = c / CPR, f0 = (c % CPR) * V, tok = tok0 + t, F0 = slab * 128 + f0;
          if (c >= cend || tok >= g.M || F0 >= g.N) continue;
          const int head = F0 / hd, d0 = F0 - head * hd;
          const float* x = acc + t * 128 + f0;
          Chunk<T> o;
          if (head < hq + hkv) {
            const bool lo = d0 < half;
            const float* xp = lo ? x + half : x - half;
#pragma unroll
            for (int v = 0; v < V; ++v) {
              const float rot = lo ? -xp[v] : xp[v];
              o.e[v] = from_f<T>(round_t<T>(round_t<T>(x[v] * to_f<T>(cs[b].e[v])) +
                                            round_t<T>(rot * to_f<T>(sn[b].e[v]))));
            }
            if (head < hq) {
              st_chunk(q + (size_t)tok * (hq * hd) + F0, o);
            } else if (s_kb[t] != nullptr) {
              st_chunk(s_kb[t] + (head - hq) * hd + d0, o);
            }
          } else if (s_vb[t] != nullptr) {
#pragma unroll
            for (int v = 0; v < V; ++v) o.e[v] = from_f<T>(x[v]);
            st_chunk(s_vb[t] + (head - hq - hkv) * hd + d0, o);
          }
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
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int f = lane + 32 * i;
          const int F = slab * 128 + f;
          if (F < g.N) {
            const float v = round_t<T>(acc[t * 128 + f]);
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
          if (slab * 128 + f < g.N) sum += expf(round_t<T>(acc[t * 128 + f]) - best);
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

}  // namespace fdllm
