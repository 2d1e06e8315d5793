/* fdllm_sm100.h -- C ABI of the sm_100a (B200) Fast-dLLM v2 block-diffusion decode library.
 *
 * This library replaces the compiled TVM Relax module of longthangvu/fast-dllm-relax
 * (artifact fast_dllm_relax_nn.so; entry points declared in fast_dllm_relax/model/cuda.py:799-842,
 * listed in fast_dllm_relax/export_utils.py:13-17).  Each entry point below names the reference
 * interface it replaces.  Conventions:
 *   - every pointer argument is device memory unless its comment says "host";
 *   - every buffer is caller-owned; the handle owns only its workspace;
 *   - calls are asynchronous on `stream` (a cudaStream_t; NULL = legacy default stream) and are
 *     serialised per handle (one handle per device and host thread is the intended use);
 *   - the return value is FDLLM_OK (0) or a negative FDLLM_ERR_* code; fdllm_last_error() gives the
 *     calling thread's last message.  No C++ exception crosses this ABI.
 *   - activations and weights are in the handle's dtype (bf16 or fp32); logits are fp32.
 */
#ifndef FDLLM_SM100_H_
#define FDLLM_SM100_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define FDLLM_ABI_VERSION 1

#if defined(__GNUC__)
#define FDLLM_API __attribute__((visibility("default")))
#else
#define FDLLM_API
#endif

enum {
  FDLLM_OK = 0,
  FDLLM_ERR_INVALID = -1,   /* bad argument / window (the reference raises ValueError) */
  FDLLM_ERR_CUDA = -2,      /* a CUDA runtime or driver call failed */
  FDLLM_ERR_UNBOUND = -3,   /* fdllm_bind_params has not been called */
  FDLLM_ERR_UNSUPPORTED = -4,
  FDLLM_ERR_DEVICE = -5     /* a kernel recorded an error (fdllm_device_error gives the code) */
};

enum { FDLLM_FLOAT32 = 0, FDLLM_BFLOAT16 = 1 };

typedef struct fdllm_handle fdllm_handle;

/* FastDLLMRelaxConfig (fast_dllm_relax/model/cuda.py:15-29) plus the artifact dtype. */
typedef struct fdllm_config {
  int32_t vocab_size;
  int32_t hidden_size;
  int32_t intermediate_size;
  int32_t num_hidden_layers;
  int32_t num_attention_heads;
  int32_t num_key_value_heads;
  int32_t head_dim;
  float rms_norm_eps;
  float rope_theta;
  int32_t tie_word_embeddings;
  int32_t bd_size;
  int32_t max_positions;      /* RoPE table length (context_window_size) */
  int32_t dtype;              /* FDLLM_FLOAT32 or FDLLM_BFLOAT16 */
} fdllm_config;

/* One request of a batched cached forward (the per-request arguments of forward_cached). */
typedef struct fdllm_request {
  void* k_cache;                     /* [layers, 1, cap, kv_heads, head_dim] */
  void* v_cache;
  int32_t cap;
  int32_t rows;                      /* active rows of this request (8 or 32 in decoding) */
  int32_t prefix_len;                /* committed cache rows */
  int32_t write_rel;                 /* K/V rows written: [prefix_len + write_rel, + rows) */
  int32_t attend_rel;                /* keys attended:    [0, prefix_len + attend_rel) */
  int32_t cache_offset_host;         /* RoPE position of row 0 when cache_offset_dev is NULL */
  const int32_t* cache_offset_dev;   /* device int32 RoPE position of row 0, or NULL */
} fdllm_request;

FDLLM_API int fdllm_abi_version(void);
FDLLM_API const char* fdllm_last_error(void);

/* Create / destroy a handle on CUDA device `device` (replaces runtime.load_module +
 * relax.VirtualMachine, fast_dllm_relax/runners.py:614-615). */
FDLLM_API int fdllm_create(const fdllm_config* cfg, int device, fdllm_handle** out);
FDLLM_API int fdllm_destroy(fdllm_handle* h);

/* Bind the parameter list, `n` device pointers in fast_dllm_relax_nn_param_names.txt order
 * (the `params` argument of every vm[...] call, fast_dllm_relax/runners.py:947-972). */
FDLLM_API int fdllm_bind_params(fdllm_handle* h, const void* const* ptrs, int n);

/* vm["embed"](input_ids) -- model/cuda.py:698-699, spec :810-813.  ids int32[n] -> out [n, hidden]. */
FDLLM_API int fdllm_embed(fdllm_handle* h, const int32_t* ids, int n, void* out, void* stream);

/* vm["forward_hidden"](input_embed, attention_bias) -- model/cuda.py:701-702, 604-608; spec :814-818.
 * x [T, hidden], bias fp32 [T, T] -> out [T, hidden]. */
FDLLM_API int fdllm_forward_hidden(fdllm_handle* h, const void* x, const float* bias, int T, void* out, void* stream);

/* vm["get_logits"](hidden_states) -- model/cuda.py:704-711, spec :819-822.
 * hidden [rows, hidden] -> fp32 logits [rows, vocab] (rounded to the model dtype first). */
FDLLM_API int fdllm_get_logits(fdllm_handle* h, const void* hidden, int rows, float* logits, void* stream);

/* vm["build_prefix_cache"](prefix_embed, prefix_bias, k_cache, v_cache) -- model/cuda.py:713-721,
 * 610-637; spec :823-829.  Writes post-RoPE K/V rows [0, P) of every layer in place. */
FDLLM_API int fdllm_build_prefix_cache(fdllm_handle* h, const void* x, const float* bias, int P, void* k_cache,
                             void* v_cache, int cap, void* stream);

/* fdllm_build_prefix_cache for n requests in one forward (no counterpart in the reference, which
 * builds one prefix per call): request i's prefix is rows [sum(rows[<i]), + rows[i]) of x, under
 * the implicit block-causal mask (block = bd_size) within the request, written to its own cache
 * rows [0, rows[i]).  Only k_cache, v_cache, cap and rows of each descriptor are read.  Results
 * match n single calls up to the bf16 rounding of the larger GEMM tiles. */
FDLLM_API int fdllm_build_prefix_cache_batch(fdllm_handle* h, const fdllm_request* reqs, int n, const void* x,
                                             void* stream);

/* vm["forward_cached"] (write_rel 0, attend_rel rows) and vm["forward_block_partial_rp{0,8,16,24}"]
 * (write_rel = rp, attend_rel = bd_size) -- model/cuda.py:723-788, 639-666; callback semantics
 * runtime.py:63-73.  cache_offset_dev is the reference's 0-d int32 device tensor, prefix_len its
 * host ShapeTuple.  x [rows, hidden] -> out [rows, hidden] (after the final norm). */
FDLLM_API int fdllm_forward_cached(fdllm_handle* h, const void* x, int rows, void* k_cache, void* v_cache, int cap,
                         const int32_t* cache_offset_dev, int prefix_len, int write_rel, int attend_rel,
                         void* out, void* stream);

/* Batched forward_cached: requests' rows are concatenated in x / out (no reference counterpart:
 * the reference runs one request at a time; each request follows runtime.py:63-73). */
FDLLM_API int fdllm_forward_cached_batch(fdllm_handle* h, const fdllm_request* reqs_host, int n, const void* x, void* out,
                               void* stream);

/* vm["get_confidence_m{rows}"] -- runtime.py:131-174, semantics model/metal.py:513-528 and the
 * kernel model/metal.py:316-374: lm_head fused with the per-row first-index argmax and
 * maxp = 1 / sum(exp(logit - max)).  Unshifted.  ids int32[rows], maxp fp32[rows]. */
FDLLM_API int fdllm_confidence(fdllm_handle* h, const void* hidden, int rows, int32_t* ids, float* maxp, void* stream);

/* The same reduction over fp32 logits [rows, vocab] (model/metal.py:316-374). */
FDLLM_API int fdllm_confidence_from_logits(fdllm_handle* h, const float* logits, int rows, int32_t* ids, float* maxp,
                                 void* stream);

/* The unmask decision of runtime.py:794-805 with the shift of runtime.py:172-173, on the device.
 * ids / maxp: unshifted results of fdllm_confidence for `rows` rows.  block_tokens: int32[bd_size]
 * ids of the active block, updated in place.  Full steps (partial = 0) use shifted rows
 * [sub_start, sub_start + sub_len); partial steps (partial = 1, rows == sub_len) use all rows.
 * Outputs per window position (each may be NULL): token, confidence, unmask flag; status int32[2]:
 * masks left in the window, positions unmasked. */
FDLLM_API int fdllm_unmask(fdllm_handle* h, const int32_t* ids, const float* maxp, int rows, int32_t* block_tokens,
                 int sub_start, int sub_len, int partial, int mask_id, double threshold, int32_t* out_tokens,
                 float* out_conf, int32_t* out_unmask, int32_t* status, void* stream);

/* fdllm_unmask for every request of a batched step at once (runtime.py:158-181 shift, 794-805
 * rule, per request; the reference decides one request at a time on the host).  ids / maxp: the
 * unshifted fdllm_confidence results of all rows of the step.  desc int32[5 n] (device), per
 * request: row0, rows (its rows in ids / maxp), base (window row 0 takes shifted row `base`: 0 for
 * a partial step, the sub-block start for a full one), win (window length <= 32; 0: no decision,
 * a block append) and the bit mask of the window rows still masked.  out int32[34 n] (device), per
 * request: the bit mask of the window rows unmasked, the last row's unshifted argmax (the token
 * after the block), then win shifted tokens.  The caller applies the bits to its block. */
FDLLM_API int fdllm_unmask_batch(fdllm_handle* h, const int32_t* ids, const float* maxp, const int32_t* desc, int n,
                                 double threshold, int32_t* out, void* stream);

/* log_softmax(get_logits(hidden))[row, target[row]] per row, fused with the lm_head
 * (the host reduction of runners.py:877-881).  targets int32[rows] -> logprob fp32[rows]. */
FDLLM_API int fdllm_token_logprob(fdllm_handle* h, const void* hidden, int rows, const int32_t* targets, float* logprob,
                        void* stream);

/* Device-resident greedy block-diffusion generation of one request (runtime.py:591-880 for
 * block-aligned prompts, temperature 0): prefill, refinement steps, threshold unmasking and
 * block-append on the device; one small status read per step.  prompt and out_tokens are host
 * int32 arrays; *n_out receives the continuation length (trimmed as runtime.py:664-669).
 * stats (host int32[4], may be NULL): unmask_updates, block_recomputes, partial_recomputes,
 * block_appends.  timing_ms (host float[2], may be NULL): CUDA-event time of the prefill (up to the
 * first refinement step, the reference's prefill boundary runtime.py:741-746) and of the whole call.
 * Returns FDLLM_ERR_UNSUPPORTED for prompts shorter than one block. */
FDLLM_API int fdllm_generate(fdllm_handle* h, const int32_t* prompt, int prompt_len, int max_new_tokens, int block_size,
                   int small_block_size, double threshold, int use_block_cache, int mask_id, int stop_token,
                   int32_t* out_tokens, int* n_out, int32_t* stats, float* timing_ms, void* stream);

/* Read and clear the handle's device error word (synchronises the device).  *code = 0 if none. */
FDLLM_API int fdllm_device_error(fdllm_handle* h, int* code);

/* fdllm_device_error with where an expired wait gave up (diagnostics; no counterpart in the
 * reference): out[0] the code, and for a wait timeout out[1] the wait site (1-5 the per-tile
 * projection GEMM's producer, drain, normaliser, MMA issuer and epilogue; 11-15 the persistent
 * GEMM's producer, drain, MMA accumulator, MMA operand and epilogue waits), out[2] the call's token
 * rows, out[3] the CTA's block index | split count << 16.  Clears all four words. */
FDLLM_API int fdllm_device_error_detail(fdllm_handle* h, int32_t* out4);

/* Failure-detection self test: launch a kernel that waits on a flag nothing sets, with a bounded
 * wait of limit_ns; it must give up, record its error code and leave the context usable. */
FDLLM_API int fdllm_wait_selftest(fdllm_handle* h, unsigned long long limit_ns, int* code);

/* Kernel launches issued by the library since it was loaded (all handles). */
FDLLM_API long long fdllm_kernel_launches(void);

/* Per-launch CUDA-event timing of the projection GEMM kernel (the dominant kernel): enable, then
 * read and reset the totals (synchronises).  out[0] = total ms, out[1] = algorithmic bytes
 * (weights + activations in + outputs), out[2] = launches, out[3] = flops. */
FDLLM_API int fdllm_profile_enable(fdllm_handle* h, int enable);
FDLLM_API int fdllm_profile_read(fdllm_handle* h, double* out4);

/* Bytes of device workspace the handle currently holds. */
FDLLM_API long long fdllm_workspace_bytes(fdllm_handle* h);

/* Kernel trace (diagnostics; no counterpart in the reference).  While enabled, every projection
 * GEMM and attention launch issued outside stream capture records the earliest and latest
 * %globaltimer value (ns) at which any of its CTAs reached phase p: out[24*i + 2p] and
 * out[24*i + 2p + 1] for launch i and p = 0..11 (UINT64_MAX / 0: not reached; the large-tile
 * persistent GEMM records nothing).  Always recorded: phase 1 (dependency wait passed) and 7 (exit);
 * the span from the earliest phase-1 stamp to the latest exit is the launch's share of the step's
 * critical path under programmatic dependent launch.  A build with
 * `python -m fast_dllm_relax_b200.build --ktrace` also records 0 entry, 2 main loop done;
 * projection 3 accumulator drained from TMEM, 4 split-K partials summed, 5 epilogue done,
 * 8 TMEM released; attention 3 partials published, 4 merge weights, 5 merge done (those stamps
 * slow every launch).  kinds[i]: 1 attention (mma.sync), 2 attention (tcgen05); 100 + epilogue kind
 * for a projection, +2000 with the fused input norm.  Enabling, and every read, clears the
 * record; at most 512 launches (1280 CTAs each) are kept.  Both calls synchronise the device.
 * With out == NULL only *n is written. */
FDLLM_API int fdllm_kernel_trace_enable(fdllm_handle* h, int enable);
FDLLM_API int fdllm_kernel_trace_read(fdllm_handle* h, uint64_t* out, int32_t* kinds, int cap, int32_t* n);

/* fdllm_confidence without any device allocation (no counterpart in the reference).  For callers
 * that may not allocate device memory inside their step: an external memory pool or a fixed
 * arena owns the device, or the step must never grow the handle's workspace.  The lm_head
 * partials live in one fixed 4 MiB module-scope device array per device, shared by every handle
 * on that device, so rows must satisfy rows * ceil(vocab / 128) * 16 <= 4 MiB (220 rows at vocab
 * 151936); larger calls return FDLLM_ERR_INVALID with the limit in fdllm_last_error.
 * - The first call on each device looks up the array's address (cudaGetSymbolAddress, which may
 *   load the module); make that first call before any stream capture.  The address is kept per
 *   device together with the CUDA context it belongs to; a call made after that context was torn
 *   down and recreated (cudaDeviceReset) looks it up again, so that call too belongs before any
 *   capture.
 * - The array keeps the previous call's contents; nothing in it needs to start at zero, because
 *   every entry a call reads is written earlier in that same call.
 * - Calls whose kernels can overlap on one device (different streams, or different handles on the
 *   same device) race on the shared array: order them on one stream or with events.
 * Results are identical to fdllm_confidence. */
FDLLM_API int fdllm_confidence_static(fdllm_handle* h, const void* hidden, int rows, int32_t* ids, float* maxp,
                                      void* stream);

#ifdef __cplusplus
}
#endif

#endif /* FDLLM_SM100_H_ */
