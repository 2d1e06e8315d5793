// fp32 projection GEMM on the CUDA cores (no TF32), for fp32 artifacts.
//
// fp32 mode exists so that decoded sequences can be compared token for token with the fp32
// oracle (the tiny config); tensor cores would round the inputs to TF32.  One CTA computes the
// same 128-weight-row x 32-token tile as the tcgen05 kernel, including the gate/up slab pairing,
// and hands it to the shared epilogue.  The K loop accumulates in ascending order.
#include "common.cuh"
#include "epilogue.cuh"
#include "kernels.h"

namespace fdllm {

constexpr int kSimtTok = 32;
constexpr int kSimtK = 32;

__global__ void __launch_bounds__(256) gemm_simt_f32_kernel(const float* __restrict__ W,
                                                            const float* __restrict__ X, const GemmArgs g) {
  __shared__ float ws[kSimtK][128 + 1];
  __shared__ float xs[kSimtK][kSimtTok + 1];
  __shared__ __align__(16) float acc[kSimtTok * 128];
  __shared__ __align__(16) unsigned char s_epi[5120];
  pdl_trigger();
  pdl_wait();
  const int slab = blockIdx.x, tile = blockIdx.y;
  const int tok0 = tile * kSimtTok;
  const int tid = threadIdx.x;
  const int tf = tid & 31;  // features tf*4 .. tf*4+3
  const int tt = tid >> 5;  // tokens   tt*4 .. tt*4+3
  const int inter = g.N / 2;
  float c[4][4] = {};
  for (int k0 = 0; k0 < g.K; k0 += kSimtK) {
    for (int idx = tid; idx < 128 * kSimtK; idx += blockDim.x) {
      const int f = idx / kSimtK, kk = idx % kSimtK;
      int row;
      if (g.paired) row = (f < 64) ? slab * 64 + f : inter + slab * 64 + (f - 64);
      else row = slab * 128 + f;
      const bool ok = g.paired ? (slab * 64 + (f & 63) < inter) : (row < g.N);
      ws[kk][f] = ok ? W[(size_t)row * g.K + k0 + kk] : 0.f;
    }
    for (int idx = tid; idx < kSimtTok * kSimtK; idx += blockDim.x) {
      const int t = idx / kSimtK, kk = idx % kSimtK;
      xs[kk][t] = (tok0 + t < g.M) ? X[(size_t)(tok0 + t) * g.K + k0 + kk] : 0.f;
    }
    __syncthreads();
#pragma unroll 8
    for (int kk = 0; kk < kSimtK; ++kk) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = ws[kk][tf * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) b[j] = xs[kk][tt * 4 + j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) c[i][j] = fmaf(a[i], b[j], c[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[(tt * 4 + j) * 128 + tf * 4 + i] = c[i][j];
  __syncthreads();
  gemm_epilogue<float>(g, acc, kSimtTok, tok0, slab, 0, kSimtTok, s_epi);
}

int launch_gemm_simt_f32(const GemmArgs& a, const float* W, const float* X, cudaStream_t s) {
  if (a.K % kSimtK != 0) return cudaErrorInvalidValue;
  dim3 grid(a.n_slabs, (a.M + kSimtTok - 1) / kSimtTok, 1);
  return launch_k(gemm_simt_f32_kernel, grid, dim3(256), 0, s, W, X, a);
}

}  // namespace fdllm
