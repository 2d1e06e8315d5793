// Internal host-side state of a library handle, shared by model.cu and decode.cu.
#pragma once

#include <algorithm>
#include <atomic>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/fdllm_sm100.h"
#include "common.cuh"
#include "kernels.h"

namespace fdllm {

int fail(int code, const std::string& msg);

#define CUDA_TRY(expr)                                                                       \
  do {                                                                                       \
    cudaError_t _e = static_cast<cudaError_t>(expr);                                         \
    if (_e != cudaSuccess)                                                                   \
      return ::fdllm::fail(FDLLM_ERR_CUDA, std::string(#expr) + ": " + cudaGetErrorString(_e)); \
  } while (0)

#define FDLLM_TRY(expr)            \
  do {                             \
    int _r = (expr);               \
    if (_r != FDLLM_OK) return _r; \
  } while (0)

// ---- tuning --------------------------------------------------------------------------------
// Parameters of the kernel plans, fixed per handle at fdllm_create.  The defaults are the
// measured best on B200; the environment variable FDLLM_TUNING ("key=value,...", read by
// fdllm_create) overrides them for experiments without rebuilding.
struct Tuning {
  int nt_max = 128;            // largest token tile of the per-tile projection GEMM: 64, 128 or 256
                               // (224-row prefill: 2.62 ms at 128 against 3.71 at 256)
  int split_target = 0;        // CTAs per SM the split-K plan aims for (0: 2 at <= 32 rows, else 1)
  int split_max = 16;          // largest split-K cluster of the per-tile GEMM
  int short_split_max = 8;     // ... of projections with K <= 2048 (qkv, o, gate_up; 0: split_max):
                               // qkv and o of a decode step in clusters of 8 instead of 12, each CTA's
                               // 3 weight k blocks still in its ring before the dependency wait
                               // (8-row step 1.3225 -> 1.3077 ms, 32-row 1.503 -> 1.4996; 6 and 4 slower)
  int gemm_tune = kGemmTunePrefetch | (2 << kGemmTuneL2Shift);  // kGemmTune* bits
  int persist_min_rows = 65;   // token rows from which projections run on the persistent GEMM (0:
                               // never); prefix builds of 96 / 160 / 224 rows: 2.17 / 2.38 / 2.44 ->
                               // 1.95 / 2.33 / 2.39 ms against 256 (64 rows: 1.53 -> 1.84, so not below)
  int persist_splitk = 3;      // split K inside the persistent GEMM (bits): 1 while its tiles leave
                               // half the SMs idle; 2 for long-K few-slab projections on 256-token
                               // tiles (down at 1024 rows: 46.6 -> 45.2 us, 32.0 with merge_all)
  int short_k_nt = 64;         // per-tile token tile of short-K few-slab projections of calls the
                               // persistent kernel covers with <= 1 tile per CTA (0: persistent)
  int persist_nt96 = 1;        // 96-token persistent tiles where they balance the SMs better
                               // (o, down at 1024 rows; batched step 4.666 -> 4.470 ms with the two above)
  int persist_l2_ahead = 0;    // weight k blocks the persistent GEMM prefetches into L2 ahead of its ring
                               // (8: 8 x 4096 prefill 142.5 -> 139.5 ms, 1024-row step +1.3%)
  int persist_merge_all = 1;   // persistent split-K in one wave: every split waits for the tile's
                               // partials and merges its share (down at 1024 rows 44.7 -> 32.0 us)
                               // instead of the last split merging the whole tile
  int persist_conf_t = 1;      // the persistent lm_head + confidence / log-softmax-gather GEMM puts
                               // 128 tokens on the MMA's M side, so each epilogue thread reduces one
                               // token's 128-logit slab in registers (0: tokens on N, lane-tree
                               // reductions through shared memory)
  int attn_splits = 0;        // attention key splits of decode-sized calls (0: planned)
  int gu_fused_rows = 16;      // gate_up normalises its own B tiles up to this many token rows
  int block_graph = 1;         // fdllm_generate runs whole blocks as device-looped CUDA graphs
  int attn_tc_min_q = 64;      // tcgen05 attention from this many query tokens per request (0: never)
  int attn_tc_min_ctas = 64;   // ... or from this many (request, KV head, query tile) CTAs
  int attn_lazy_log2 = 0;      // tcgen05 attention: exponent base moves when a row's max grows by > 2^x
  int attn_tc_split_min_keys = 1024;  // cached calls from this many keys whose tcgen05 grid leaves SMs
                               // idle: the keys split over CTAs and merged (8 x 32 rows at 4096 keys:
                               // 3.28 -> 2.92 ms a forward; 512 slows the 32 x 32-row step at 768 keys)
  int attn_tc_split_target = 1;  // ... as many splits as give this many CTAs per SM (1: a 3-stage ring
                               // each, 2.92 ms; 2: two CTAs per SM on 2 stages, 2.97 ms)
};
int parse_tuning(const char* spec, Tuning* t);

// ---- handle ------------------------------------------------------------------------------
struct Weight {
  const void* ptr = nullptr;
  int rows = 0, cols = 0;
  bool paired = false;
  CUtensorMap map{};
};

struct BMapEntry {  // an encoded 2D activation tensor map and what it was encoded for
  const void* base;
  int rows, cols, box_rows;
  CUtensorMap map;
};

struct LayerW {
  Weight qkv, o, gu, down;
  const void* qkv_b = nullptr;
  const void* ln1 = nullptr;
  const void* ln2 = nullptr;
};

// Bumped whenever any workspace buffer is reallocated: captured graphs recorded before a bump hold
// stale pointers and are recaptured.
extern std::atomic<unsigned long long> g_ws_generation;

template <typename P>
struct DevBuf {
  P* p = nullptr;
  size_t n = 0;  // elements
  int ensure(size_t want, bool zero = false) {
    if (want <= n) return FDLLM_OK;
    g_ws_generation.fetch_add(1);
    if (p) cudaFree(p);
    p = nullptr;
    n = 0;
    size_t cap = std::max<size_t>(want, 256);
    cudaError_t e = cudaMalloc(&p, cap * sizeof(P));
    if (e != cudaSuccess) return fail(FDLLM_ERR_CUDA, std::string("cudaMalloc: ") + cudaGetErrorString(e));
    if (zero) {
      e = cudaMemset(p, 0, cap * sizeof(P));
      if (e != cudaSuccess) return fail(FDLLM_ERR_CUDA, std::string("cudaMemset: ") + cudaGetErrorString(e));
    }
    n = cap;
    return FDLLM_OK;
  }
  void release() {
    if (p) cudaFree(p);
    p = nullptr;
    n = 0;
  }
  size_t bytes() const { return n * sizeof(P); }
};

struct ProfPair {
  cudaEvent_t e0 = nullptr, e1 = nullptr;
  double bytes = 0.0, flops = 0.0;
};

// One captured decode step (see decode.cu).
struct StepGraph {
  cudaGraphExec_t exec = nullptr;
  unsigned long long gen = 0;  // g_ws_generation at capture
  int mask_id = 0;             // unmask parameters baked into the captured launch
  double thr = 0.0;
  int n_kernels = 0;           // kernel nodes, counted as launches at every replay
  std::vector<ProfPair> prof;
};

// One captured decode block (see decode.cu): every refinement step of the block's sub-blocks run
// by device-side WHILE / IF-ELSE graph nodes, then the block-append forward.
struct BlockGraph {
  cudaGraphExec_t exec = nullptr;
  unsigned long long gen = 0;
  int mask_id = 0;
  double thr = 0.0;
  int use_block_cache = 0, sbs = 0;
  int n_full = 0, n_partial = 0, n_append = 0;  // kernels of one full / partial step and of the append
};

struct DecodeState {
  DevBuf<uint8_t> k, v;        // caches of the native driver
  BlockGraph block_graph;      // the device-looped block (when the block fits its conditions)
  DevBuf<int> loop;            // device loop state of the block graph
  DevBuf<int> ids;             // prefill / block token ids
  DevBuf<int> block;           // active block ids (bd_size)
  DevBuf<uint8_t> x, hid;      // embeddings in / hidden out
  DevBuf<int> cids;            // confidence ids
  DevBuf<float> cmax;          // confidence values
  DevBuf<int> out;             // [0..1] status, [2..] window tokens, then unmask flags
  int* host = nullptr;         // pinned read-back buffer
  int* host_params = nullptr;  // pinned step parameters (prefix length)
  DevBuf<int> plen;            // device prefix length read by the captured steps
  cudaStream_t stream = nullptr;
  std::vector<std::pair<long long, StepGraph>> graphs;  // keyed step graphs
  const void* graph_cache_ptr = nullptr;                // caches the graphs were captured against
  int graph_cap = 0;
};

}  // namespace fdllm

using fdllm::DecodeState;
using fdllm::DevBuf;
using fdllm::LayerW;
using fdllm::ReqDesc;
using fdllm::Weight;

struct fdllm_handle {
  fdllm_config cfg{};
  int device = 0;
  int dtype = FDLLM_BFLOAT16;
  size_t esz = 2;
  int num_sms = 148;
  bool bound = false;
  fdllm::Tuning tune;
  std::mutex mu;

  const void* embed = nullptr;
  const void* final_norm = nullptr;
  Weight lm;
  std::vector<LayerW> layers;

  DevBuf<uint8_t> rope_cos, rope_sin;
  DevBuf<int> err;

  // workspace (grown on demand; never inside a captured region)
  DevBuf<uint8_t> h, xn, q, attn, act, scratch_k, scratch_v;
  DevBuf<int> tok_req, tok_pos, tok_row, tmp_ids, targets;
  DevBuf<ReqDesc> reqs;
  DevBuf<float> conf_part, tmp_maxp, ss;  // ss: per-slab row sums of squares
  DevBuf<CUtensorMap> attn_maps;          // tcgen05 attention: K and V tensor maps per request
  std::vector<long long> attn_maps_key;   // the requests whose maps attn_maps holds
  std::vector<fdllm::BMapEntry> bmaps;    // encoded activation maps of the projections
  DevBuf<float> attn_part, attn_part_lse;  // tcgen05 key-split partials
  DevBuf<float> persist_part;               // persistent-GEMM split-K partial tiles
  DevBuf<unsigned> persist_ctr;             // persistent-GEMM per-tile split counters (zero between launches)
  // kernel trace (fdllm_kernel_trace_enable / _read): phase stamps of every projection and
  // attention launch issued outside stream capture while enabled, 8 per launch, and their kinds
  bool ktrace_on = false;
  DevBuf<unsigned long long> ktrace;
  std::vector<int32_t> ktrace_kind;
  DecodeState dec;

  // per-launch CUDA-event timing of the projection GEMM (fdllm_profile_enable / _read)
  bool prof = false;
  std::vector<cudaEvent_t> prof_ev;
  size_t prof_used = 0;
  double prof_bytes = 0.0, prof_flops = 0.0;
  double prof_ms_extra = 0.0;       // accumulated from replayed graphs
  long long prof_launch_extra = 0;
  // stream capture in progress: profiled launches get graph-owned events
  bool capturing = false;
  std::vector<fdllm::ProfPair> cap_prof;
};


namespace fdllm {

size_t round_up(size_t x, size_t m);
long long layer_stride(const fdllm_handle* h, int cap);
int check_handle(fdllm_handle* h);
int forward_core(fdllm_handle* h, const void* x, int M, std::vector<ReqDesc>& reqs, const float* bias, int ld_bias,
                 int causal_block, void* out, cudaStream_t s, int max_l_hint = 0);
int reserve_workspace(fdllm_handle* h, int M, int nreq, int max_l);
void release_step_graphs(fdllm_handle* h);
int dense_forward(fdllm_handle* h, const void* x, const float* bias, int T, void* k, void* v, int cap, bool scratch,
                  void* out, cudaStream_t s);
int cached_desc(fdllm_handle* h, const fdllm_request& r, int q_tok0, ReqDesc* d);
int confidence_locked(fdllm_handle* h, const void* hidden, int rows, int32_t* ids, float* maxp,
                      const int32_t* targets, float* logprob, cudaStream_t s);

}  // namespace fdllm
