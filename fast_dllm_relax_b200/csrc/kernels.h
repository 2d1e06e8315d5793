// Kernel-facing structures and launcher declarations shared by the .cu files of the library.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace fdllm {

// One request of a (possibly batched) forward call, as the device sees it.  Token rows of all
// requests are concatenated: request r owns activation rows [q_tok0, q_tok0 + n_q).
struct ReqDesc {
  void* k;                  // KV cache base [layers, 1, cap, kv_heads, head_dim] (or a per-layer scratch)
  void* v;
  long long layer_stride;   // elements between consecutive layers of k / v (0 for a per-layer scratch)
  int cap;                  // cache rows
  int q_tok0;               // first activation row of this request
  int n_q;                  // activation rows (tokens) of this request
  int write_start;          // cache row that receives token 0's K/V
  int attend_len;           // attention keys are cache rows [0, attend_len)
  int rope_base;            // RoPE position of token 0 when rope_off is null
  const int* rope_off;      // device int32 position of token 0 (the reference's cache_offset), or null
  // When plen_dev is set, the prepare kernel derives write_start / attend_len / rope_base from the
  // device prefix length (a captured CUDA graph replays unchanged while the prefix grows).
  const int* plen_dev;
  int write_rel;
  int attend_rel;
};

constexpr int kMaxAttnSplits = 8;  // key splits = attention cluster size (portable)
constexpr int kMaxReqsPerLaunch = 48;  // keeps ReqBatch under the classic 4 KB parameter limit

struct ReqBatch {
  ReqDesc r[kMaxReqsPerLaunch];
  int n;
  int first;  // index of r[0] in the device request table
};

// Per-token data derived from the requests once per forward call (prepare kernel).
struct TokenMaps {
  int* req;    // [M] request index
  int* pos;    // [M] RoPE position
  int* row;    // [M] cache row receiving this token's K/V
};

enum EpiKind : int {
  kEpiStore = 0,      // out[t, f] = T(acc)
  kEpiQkvRope = 1,    // + bias, RoPE on q/k, q -> qout, k/v -> caches (per-token rows)
  kEpiResidual = 2,   // resid[t, f] = T(resid + T(acc))
  kEpiSiluMul = 3,    // paired gate/up slab: out[t, j] = T(T(silu(T(gate))) * T(up))
  kEpiLogitsF32 = 4,  // out_f32[t, f] = float(T(acc))
  kEpiConf = 5,       // per (token, slab): max, first argmax, sum exp(v - max) of float(T(acc))
  kEpiLseGather = 6,  // kEpiConf plus the logit of a per-token target id
};

struct Epilogue {
  int kind;
  int layer;
  void* out;                // Store / SiluMul: [M, ld_out] in T; LogitsF32: float [M, ld_out]
  int ld_out;
  const void* bias;         // QkvRope: [N] in T
  void* resid;              // Residual: [M, ld_resid] in T
  const void* resid_src;    // Residual: optional source of the residual (else resid); same layout
  float* ss_out;            // Residual: optional [M, ss_ld] sum of squares of each new row's 128-feature
  int ss_ld;                //   slab (the next RMSNorm's statistics, consumed by a fused-norm GEMM)
  int ld_resid;
  // QkvRope
  void* qout;               // [M, hq*hd] in T
  const void* rope_cos;     // [max_pos, hd/2] in T
  const void* rope_sin;
  int max_pos;
  int hq, hkv, hd;
  const ReqDesc* reqs;      // device request table
  TokenMaps tok;
  // Conf / LseGather
  float* part;              // [M, n_slabs, 4]: max, argmax (as int bits), sum exp, target logit
  const int* target;        // LseGather: [M] target ids
};

// GemmArgs::tune bits (decode-sized tiles, NT <= 64): load the epilogue's inputs before the
// accumulator is ready; bits 8-15: weight k blocks prefetched into L2 ahead of the shared-memory
// ring (more bytes in flight per SM than the ring holds).
constexpr int kGemmTunePrefetch = 1;
constexpr int kGemmTuneL2Shift = 8;
constexpr int kGemmTunePersistL2Shift = 16;  // bits 16-23: the persistent GEMM's L2 prefetch distance

struct GemmArgs {
  int M, N, K;              // tokens, output features (weight rows), reduction
  int paired;               // gate/up pairing (N = 2*I; slab s covers rows [64s, 64s+64) and I + same)
  int n_slabs;              // N / 128 (or I / 64 when paired)
  int n_tok_tiles;
  int tile_n;               // persistent GEMM: token rows per tile (128 or 256; the B map's box height)
  int tile_major;           // per-tile GEMM: grid (token tiles, slabs, splits) instead of (slabs, tiles, splits)
  int splits;               // split-K factor = cluster size (<= 16)
  int kb_per_split;         // 64-wide k blocks per split
  // Fused RMSNorm of the activations (tcgen05 path): when norm_x is set the B operand is
  // rmsnorm(norm_x) * norm_w computed inside the GEMM (model/cuda.py:269-275) instead of TMA-loaded.
  const void* norm_x;       // [M, K] in T
  const void* norm_w;       // [K] in T
  const float* norm_ss;     // [M, norm_ss_ld] per-128-feature sums of squares of norm_x rows
  int norm_ss_ld;
  float norm_eps;
  // persistent GEMM split-K (splits <= 4): fp32 partial tiles [tiles][splits][NT][128] and per-tile
  // arrival counters (zero between launches; the last split resets its tile's counter)
  float* ppart;
  unsigned* pctr;           // [2][tiles]: partials arrived, splits done (pmerge_all)
  int pmerge_all;           // every split merges its share (only when each CTA holds <= 1 unit)
  // persistent GEMM (tile_n 256), confidence / log-softmax-gather epilogues only: 128 token rows on
  // the MMA's M side and two 128-row weight slabs on N, so TMEM lane = token; n_tok_tiles counts
  // 128-token tiles and the B map's box is 128 rows
  int conf_t;
  unsigned long long* ktrace;  // phase stamps of this launch (kernel trace), or null
  int tune;                 // kGemmTune* bits
  int* err;
  Epilogue epi;
};

struct AttnArgs {
  const void* q;            // [M, hq*hd] in T
  void* out;                // [M, hq*hd] in T
  const ReqDesc* reqs;      // device request table
  int n_reqs;
  int layer;
  int hq, hkv, hd;
  float scale;
  const float* bias;        // dense path: [n_q, ld_bias] fp32 additive bias of request 0, or null
  int ld_bias;
  int causal_block;         // > 0 and bias null: implicit block-causal mask (query block >= key block)
  int n_splits;             // key splits per (request, kv head, q tile) = cluster size
  int split_len;            // minimum keys per split (multiple of 64)
  int m_total;              // M: activation rows of all requests
  float lazy_log2;          // tcgen05 kernel: a row's exponent base moves when its maximum grows by
                            //   more than 2^lazy_log2 (0: whenever it grows)
  float* part;              // tcgen05 key splits: [n_splits][m_total][hq][hd] fp32 partial O / l
  float* part_lse;          //   [n_splits][m_total][hq] log2-sum-exp of each partial row
  unsigned long long* ktrace;  // phase stamps of this launch (kernel trace), or null
  int* err;
};

// ---- launch accounting / programmatic dependent launch -------------------------------------
void count_launch(int n = 1);
long long launch_count();

// Launch `kernel` with the programmatic-stream-serialization attribute: it may start while its
// predecessor in the stream drains (see pdl_wait / pdl_trigger).
template <typename... KArgs, typename... Args>
cudaError_t launch_k(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, Args&&... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  count_launch();
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

// launch_k with a (1, 1, cluster_z) thread-block cluster (cluster_z == 1: no cluster).
template <typename... KArgs, typename... Args>
cudaError_t launch_kc(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, int cluster_z,
                      Args&&... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  int n = 0;
  attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[n].val.programmaticStreamSerializationAllowed = 1;
  ++n;
  if (cluster_z > 1) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = 1;
    attr[n].val.clusterDim.y = 1;
    attr[n].val.clusterDim.z = static_cast<unsigned>(cluster_z);
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  count_launch();
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

// ---- launchers (return a cudaError_t) --------------------------------------------------------
int launch_gemm_tc(const GemmArgs& a, const CUtensorMap& tmA, const CUtensorMap& tmB, int nt, cudaStream_t s);
// Persistent 256-token-tile variant (grid CTAs walk all slab x token tiles; no split-K).
int launch_gemm_tc_persist(const GemmArgs& a, const CUtensorMap& tmA, const CUtensorMap& tmB, int nt, int grid,
                           cudaStream_t s);
int launch_gemm_simt_f32(const GemmArgs& a, const float* W, const float* X, cudaStream_t s);

int launch_attention(const AttnArgs& a, int max_q, int dtype, cudaStream_t s);
// tcgen05 attention (bf16, head_dim 128, no explicit bias): maps_dev holds two 3D tensor maps per
// request (K then V: {kv_heads * head_dim, attended keys, layers}, box {64, 64, 1}, 128-byte swizzle).
int launch_attention_tc(const AttnArgs& a, const CUtensorMap* maps_dev, int max_q, int num_sms, cudaStream_t s);
int init_attention_tc_attributes();
int init_kernel_attributes();  // opt-in shared memory sizes; once per device, before any capture

int launch_embed(const int* ids, int n, const void* table, int vocab, int hidden, void* out, int dtype, int* err,
                 cudaStream_t s);
int launch_rmsnorm(const void* x, const void* w, void* out, int rows, int hidden, float eps, int dtype,
                   cudaStream_t s, void* copy_x_to = nullptr);
int launch_rope_tables(void* cos_t, void* sin_t, int max_pos, int hd, float theta, int dtype, cudaStream_t s);
int launch_prepare(const ReqBatch& b, ReqDesc* dev_table, TokenMaps tok, int max_pos, int* err, cudaStream_t s);
int launch_conf_combine(const float* part, int rows, int n_slabs, int* ids, float* maxp, cudaStream_t s);
int launch_conf_from_logits(const float* logits, int rows, int vocab, int* ids, float* maxp, cudaStream_t s);
int launch_lse_combine(const float* part, int rows, int n_slabs, float* logprob, cudaStream_t s);
int launch_unmask(const int* ids, const float* maxp, int rows, int* block, int sub_start, int sub_len,
                  int partial, int mask_id, double threshold, int* out_tok, float* out_conf, int* out_unmask,
                  int* status, cudaStream_t s);
int launch_unmask_batch(const int* ids, const float* maxp, const int* desc, int n, double threshold, int* out,
                        cudaStream_t s);
int launch_wait_test(int* flag, int* err, unsigned long long limit_ns, cudaStream_t s);
}  // namespace fdllm
