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
#pragma once

#include "common.cuh"
#include "kernels.h"

namespace fdllm {

template <typename T>
__device__ void gemm_epilogue(const GemmArgs& g, float* acc, int nt, int tok0, int slab) {
  const Epilogue& e = g.epi;
  const int nthr = blockDim.x;
  const int tid = threadIdx.x;

  switch (e.kind) {
    case kEpiStore: {
      T* out = static_cast<T*>(e.out);
      for (int idx = tid; idx < nt * 128; idx += nthr) {
        const int t = idx >> 7, f = idx & 127, tok = tok0 + t, F = slab * 128 + f;
        if (tok < g.M && F < g.N) out[(size_t)tok * e.ld_out + F] = from_f<T>(acc[idx]);
      }
      break;
    }
    case kEpiLogitsF32: {
      float* out = static_cast<float*>(e.out);
      for (int idx = tid; idx < nt * 128; idx += nthr) {
        const int t = idx >> 7, f = idx & 127, tok = tok0 + t, F = slab * 128 + f;
        if (tok < g.M && F < g.N) out[(size_t)tok * e.ld_out + F] = round_t<T>(acc[idx]);
      }
      break;
    }
    case kEpiResidual: {
      T* h = static_cast<T*>(e.resid);
      for (int idx = tid; idx < nt * 128; idx += nthr) {
        const int t = idx >> 7, f = idx & 127, tok = tok0 + t, F = slab * 128 + f;
        if (tok < g.M && F < g.N) {
          T* p = h + (size_t)tok * e.ld_resid + F;
          *p = from_f<T>(to_f<T>(*p) + round_t<T>(acc[idx]));
        }
      }
      break;
    }
    case kEpiSiluMul: {
      T* out = static_cast<T*>(e.out);
      const int inter = g.N / 2;
      for (int idx = tid; idx < nt * 64; idx += nthr) {
        const int t = idx >> 6, f = idx & 63, tok = tok0 + t, j = slab * 64 + f;
        if (tok < g.M && j < inter) {
          const float gate = round_t<T>(acc[t * 128 + f]);
          const float up = round_t<T>(acc[t * 128 + 64 + f]);
          const float act = round_t<T>(gate * (1.0f / (1.0f + expf(-gate))));
          out[(size_t)tok * e.ld_out + j] = from_f<T>(act * up);
        }
      }
      break;
    }
    case kEpiQkvRope: {
      const T* bias = static_cast<const T*>(e.bias);
      // Phase 1: projection + bias, rounded to the model dtype (the op's output tensor).
      for (int idx = tid; idx < nt * 128; idx += nthr) {
        const int F = slab * 128 + (idx & 127);
        if (F < g.N) acc[idx] = round_t<T>(acc[idx] + to_f<T>(bias[F]));
      }
      __syncthreads();
      // Phase 2: rotate q and k (partner element d +- hd/2 of the same head, inside this slab),
      // scatter q to qout and k / v to the request's cache rows.
      const int hd = e.hd, half = e.hd >> 1, hq = e.hq, hkv = e.hkv;
      const T* cos_t = static_cast<const T*>(e.rope_cos);
      const T* sin_t = static_cast<const T*>(e.rope_sin);
      T* q = static_cast<T*>(e.qout);
      for (int idx = tid; idx < nt * 128; idx += nthr) {
        const int t = idx >> 7, f = idx & 127, tok = tok0 + t, F = slab * 128 + f;
        if (tok >= g.M || F >= g.N) continue;
        const int head = F / hd, d = F - head * hd;
        const float x = acc[idx];
        if (head < hq + hkv) {
          const float partner = (d < half) ? acc[idx + half] : acc[idx - half];
          const float rot = (d < half) ? -partner : partner;
          int pos = e.tok.pos[tok];
          pos = pos < 0 ? 0 : (pos >= e.max_pos ? e.max_pos - 1 : pos);  // range checked in prepare
          const int di = (d < half) ? d : d - half;
          const float c = to_f<T>(cos_t[(size_t)pos * half + di]);
          const float s = to_f<T>(sin_t[(size_t)pos * half + di]);
          const float y = round_t<T>(round_t<T>(x * c) + round_t<T>(rot * s));
          if (head < hq) {
            q[(size_t)tok * (hq * hd) + F] = from_f<T>(y);
          } else {
            const ReqDesc& r = e.reqs[e.tok.req[tok]];
            const int row = e.tok.row[tok];
            if (row >= 0 && row < r.cap) {
              T* k = static_cast<T*>(r.k) + (size_t)e.layer * r.layer_stride;
              k[((size_t)row * hkv + (head - hq)) * hd + d] = from_f<T>(y);
            }
          }
        } else {
          const ReqDesc& r = e.reqs[e.tok.req[tok]];
          const int row = e.tok.row[tok];
          if (row >= 0 && row < r.cap) {
            T* v = static_cast<T*>(r.v) + (size_t)e.layer * r.layer_stride;
            v[((size_t)row * hkv + (head - hq - hkv)) * hd + d] = from_f<T>(x);
          }
        }
      }
      break;
    }
    case kEpiConf:
    case kEpiLseGather: {
      const int warp = tid >> 5, lane = tid & 31, nwarps = nthr >> 5;
      for (int t = warp; t < nt; t += nwarps) {
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
          float* p = e.part + ((size_t)tok * g.n_slabs + slab) * 4;
          float tv = 0.f;
          if (e.kind == kEpiLseGather) {
            const int tg = e.target[tok] - slab * 128;
            tv = (tg >= 0 && tg < 128) ? round_t<T>(acc[t * 128 + tg]) : 0.f;
          }
          p[0] = best;
          p[1] = __int_as_float(best_i);
          p[2] = sum;
          p[3] = tv;
        }
      }
      break;
    }
    default:
      break;
  }
}

}  // namespace fdllm
