// Host runtime of the sm_100a library: the handle (device, config, bound parameters, TMA
// descriptors, RoPE tables, workspace), the layer schedule of the nine entry points, the batched
// cached forward, the device-side confidence / unmask path, the device-resident decode driver and
// the C ABI declared in include/fdllm_sm100.h.
//
// Layer schedule (model/cuda.py:545-579, 639-666), one launch each:
//   rmsnorm(h) -> qkv GEMM [+bias, RoPE, K/V append] -> attention -> o GEMM [+= h]
//   -> rmsnorm(h) -> gate_up GEMM [SiLU * up] -> down GEMM [+= h]
// then the final rmsnorm.  Nothing returns to the host between layers.
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "handle.h"

using namespace fdllm;

std::atomic<unsigned long long> fdllm::g_ws_generation{0};

// ---- error plumbing ------------------------------------------------------------------------
static thread_local std::string g_last_error;

int fdllm::fail(int code, const std::string& msg) {
  g_last_error = msg;
  // Consume the runtime's per-thread error state so that a failed call is not reported again by the
  // next launch's cudaGetLastError() (sticky device faults stay visible regardless).
  if (code == FDLLM_ERR_CUDA) (void)cudaGetLastError();
  return code;
}

// ---- TMA descriptor encoding (driver entry point fetched through the runtime) ----------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// 2D bf16 [rows, cols] row-major tensor, box of box_rows x 64 columns, 128-byte swizzle.
static int make_map(CUtensorMap* map, const void* base, int rows, int cols, int box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return fail(FDLLM_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0) return fail(FDLLM_ERR_INVALID, "TMA base must be 16-byte aligned");
  if (cols % 64 != 0) return fail(FDLLM_ERR_UNSUPPORTED, "GEMM reduction dim must be a multiple of 64");
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(cols) * 2};
  cuuint32_t box[2] = {64, static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(FDLLM_ERR_CUDA, "cuTensorMapEncodeTiled failed (" + std::to_string(r) + ")");
  return FDLLM_OK;
}

// make_map through the handle's cache of activation maps: the projections of a forward read the
// same few workspace buffers at the same sizes in every layer, so each map is encoded once.
static int cached_map(fdllm_handle* h, CUtensorMap* map, const void* base, int rows, int cols, int box_rows) {
  for (const BMapEntry& e : h->bmaps)
    if (e.base == base && e.rows == rows && e.cols == cols && e.box_rows == box_rows) {
      *map = e.map;
      return FDLLM_OK;
    }
  FDLLM_TRY(make_map(map, base, rows, cols, box_rows));
  if (h->bmaps.size() >= 64) h->bmaps.erase(h->bmaps.begin());
  h->bmaps.push_back(BMapEntry{base, rows, cols, box_rows, *map});
  return FDLLM_OK;
}

// K or V cache of one request as a 3D bf16 tensor {kv_heads * head_dim, keys, layers} (row stride
// row_bytes, layer stride layer_bytes), box {64, 64, 1}, 128-byte swizzle.  `keys` is the attended
// length, so keys past it read as zeros whatever the cache rows beyond it hold.
static int make_kv_map(CUtensorMap* map, const void* base, int cols, int keys, int layers, size_t row_bytes,
                       size_t layer_bytes) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return fail(FDLLM_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0) return fail(FDLLM_ERR_INVALID, "KV cache must be 16-byte aligned");
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(keys), static_cast<cuuint64_t>(layers)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(row_bytes), static_cast<cuuint64_t>(layer_bytes)};
  cuuint32_t box[3] = {64, 64, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(FDLLM_ERR_CUDA, "cuTensorMapEncodeTiled (KV) failed (" + std::to_string(r) + ")");
  return FDLLM_OK;
}

size_t fdllm::round_up(size_t x, size_t m) { return (x + m - 1) / m * m; }

// "key=value,key=value" over the Tuning fields; unknown keys or values out of range fail.
int fdllm::parse_tuning(const char* spec, Tuning* t) {
  if (spec == nullptr || spec[0] == '\0') return FDLLM_OK;
  const std::string all(spec);
  size_t pos = 0;
  while (pos <= all.size()) {
    const size_t end = std::min(all.find(',', pos), all.size());
    const std::string item = all.substr(pos, end - pos);
    pos = end + 1;
    if (item.empty()) continue;
    const size_t eq = item.find('=');
    if (eq == std::string::npos) return fail(FDLLM_ERR_INVALID, "tuning item without '=': " + item);
    const std::string key = item.substr(0, eq);
    char* stop = nullptr;
    const long v = std::strtol(item.c_str() + eq + 1, &stop, 0);
    if (stop == item.c_str() + eq + 1 || *stop != '\0') return fail(FDLLM_ERR_INVALID, "bad tuning value: " + item);
    const int x = static_cast<int>(v);
    if (key == "nt_max" && (x == 64 || x == 128 || x == 256)) t->nt_max = x;
    else if (key == "split_target" && x >= 0 && x <= 4) t->split_target = x;
    else if (key == "split_max" && x >= 1 && x <= 16) t->split_max = x;
    else if (key == "short_split_max" && x >= 0 && x <= 16) t->short_split_max = x;
    else if (key == "gemm_tune" && x >= 0) t->gemm_tune = x;
    else if (key == "persist_min_rows" && x >= 0) t->persist_min_rows = x;
    else if (key == "persist_splitk" && x >= 0 && x <= 3) t->persist_splitk = x;
    else if (key == "short_k_nt" && (x == 0 || x == 64 || x == 128)) t->short_k_nt = x;
    else if (key == "attn_splits" && x >= 0 && x <= kMaxAttnSplits) t->attn_splits = x;
    else if (key == "gu_fused_rows" && x >= 0 && x <= 64) t->gu_fused_rows = x;
    else if (key == "block_graph" && (x == 0 || x == 1)) t->block_graph = x;
    else if (key == "attn_tc_min_q" && x >= 0) t->attn_tc_min_q = x;
    else if (key == "attn_tc_min_ctas" && x >= 0) t->attn_tc_min_ctas = x;
    else if (key == "persist_nt96" && (x == 0 || x == 1)) t->persist_nt96 = x;
    else if (key == "persist_l2_ahead" && x >= 0 && x <= 64) t->persist_l2_ahead = x;
    else if (key == "persist_merge_all" && (x == 0 || x == 1)) t->persist_merge_all = x;
    else if (key == "persist_conf_t" && (x == 0 || x == 1)) t->persist_conf_t = x;
    else if (key == "attn_lazy_log2" && x >= 0 && x <= 16) t->attn_lazy_log2 = x;
    else if (key == "attn_tc_split_min_keys" && x >= 0) t->attn_tc_split_min_keys = x;
    else if (key == "attn_tc_split_target" && (x == 1 || x == 2)) t->attn_tc_split_target = x;
    else return fail(FDLLM_ERR_INVALID, "unknown tuning key or value out of range: " + item);
  }
  return FDLLM_OK;
}

// ---- GEMM dispatch -------------------------------------------------------------------------
static int pick_nt(const fdllm_handle* h, int M) {
  const int nt_max = h->tune.nt_max;
  if (M <= 16) return 16;
  if (M <= 32) return 32;
  if (M <= 64 || nt_max == 64) return 64;
  if (M <= 128 || nt_max == 128) return 128;
  return 256;
}

// Events for one profiled launch (reused across reads).
static int prof_events(fdllm_handle* h, cudaEvent_t* e0, cudaEvent_t* e1) {
  while (h->prof_ev.size() < h->prof_used + 2) {
    cudaEvent_t e;
    CUDA_TRY(cudaEventCreate(&e));
    h->prof_ev.push_back(e);
  }
  *e0 = h->prof_ev[h->prof_used];
  *e1 = h->prof_ev[h->prof_used + 1];
  h->prof_used += 2;
  return FDLLM_OK;
}

// Algorithmic HBM bytes of one projection launch: weights + activations in + outputs.
static double gemm_bytes(const fdllm_handle* h, const GemmArgs& g) {
  const double e = static_cast<double>(h->esz);
  double out = 0.0;
  switch (g.epi.kind) {
    case kEpiSiluMul: out = static_cast<double>(g.M) * (g.N / 2) * e; break;
    case kEpiResidual: out = 2.0 * g.M * g.N * e; break;
    case kEpiLogitsF32: out = 4.0 * g.M * g.N; break;
    case kEpiConf:
    case kEpiLseGather: out = 16.0 * g.M * g.n_slabs; break;
    default: out = static_cast<double>(g.M) * g.N * e; break;
  }
  return static_cast<double>(g.N) * g.K * e + static_cast<double>(g.M) * g.K * e + out;
}

static int timed_launch(fdllm_handle* h, const GemmArgs& g, cudaStream_t s, int (*launch)(const GemmArgs&, const void*, const void*, int, cudaStream_t),
                        const void* a0, const void* a1, int nt) {
  cudaEvent_t e0 = nullptr, e1 = nullptr;
  if (h->prof) {
    if (h->capturing) {  // the graph owns these events; its replays re-record them
      ProfPair pp;
      CUDA_TRY(cudaEventCreate(&pp.e0));
      CUDA_TRY(cudaEventCreate(&pp.e1));
      pp.bytes = gemm_bytes(h, g);
      pp.flops = 2.0 * g.M * static_cast<double>(g.N) * g.K;
      h->cap_prof.push_back(pp);
      e0 = pp.e0;
      e1 = pp.e1;
    } else {
      FDLLM_TRY(prof_events(h, &e0, &e1));
    }
    // While capturing, only an "external" record becomes a real event-record node of the graph.
    CUDA_TRY(cudaEventRecordWithFlags(e0, s, h->capturing ? cudaEventRecordExternal : cudaEventRecordDefault));
  }
  CUDA_TRY(launch(g, a0, a1, nt, s));
  if (h->prof) {
    CUDA_TRY(cudaEventRecordWithFlags(e1, s, h->capturing ? cudaEventRecordExternal : cudaEventRecordDefault));
    if (!h->capturing) {
      h->prof_bytes += gemm_bytes(h, g);
      h->prof_flops += 2.0 * g.M * static_cast<double>(g.N) * g.K;
    }
  }
  return FDLLM_OK;
}

static int launch_tc_thunk(const GemmArgs& g, const void* a, const void* b, int nt, cudaStream_t s) {
  return launch_gemm_tc(g, *static_cast<const CUtensorMap*>(a), *static_cast<const CUtensorMap*>(b), nt, s);
}

static int launch_persist_thunk(const GemmArgs& g, const void* a, const void* b, int grid, cudaStream_t s) {
  // the token tile is the one the B tensor map was encoded with (its box height)
  return launch_gemm_tc_persist(g, *static_cast<const CUtensorMap*>(a), *static_cast<const CUtensorMap*>(b), g.tile_n,
                                grid, s);
}

// The persistent large-tile GEMM from tune.persist_min_rows token rows (prefill, batched serving).
static bool use_persist(const fdllm_handle* h, int M) {
  return h->tune.persist_min_rows > 0 && h->dtype == FDLLM_BFLOAT16 && M >= h->tune.persist_min_rows;
}

static int launch_simt_thunk(const GemmArgs& g, const void* w, const void* x, int, cudaStream_t s) {
  return launch_gemm_simt_f32(g, static_cast<const float*>(w), static_cast<const float*>(x), s);
}

// Grid, token tile and split-K plan of one projection (no side effects).  nt_cap > 0 caps the
// token tile.
static int plan_gemm(const fdllm_handle* h, const Weight& w, int M, GemmArgs* g, int nt_cap = 0) {
  g->M = M;
  g->N = w.rows;
  g->K = w.cols;
  g->paired = w.paired ? 1 : 0;
  if (h->dtype == FDLLM_FLOAT32) {
    g->n_slabs = w.paired ? (g->N / 2 + 63) / 64 : (g->N + 127) / 128;
    g->n_tok_tiles = (M + 31) / 32;
    g->splits = 1;
    g->kb_per_split = 0;
    return 32;
  }
  const int nt = nt_cap > 0 ? std::min(pick_nt(h, M), nt_cap) : pick_nt(h, M);
  g->n_tok_tiles = (M + nt - 1) / nt;
  g->n_slabs = w.paired ? (g->N / 2) / 64 : g->N / 128;
  const int kblocks = g->K / 64;
  const int tiles = g->n_slabs * g->n_tok_tiles;
  int splits = 1;
  // CTAs per SM the split-K plan aims for: 2 at <= 32 token rows (the 8-row partial step: 1.348 ->
  // 1.329 ms at prefix 384; the 32-row block step 1.517 -> 1.511 ms, 700 -> 707 tokens/s; 3 or 4
  // slower at both), else 1.
  const int target = h->tune.split_target > 0 ? h->tune.split_target : (M <= 32 ? 2 : 1);
  const int split_max = h->tune.short_split_max > 0 && g->K <= 2048 ? std::min(h->tune.split_max, h->tune.short_split_max)
                                                                   : h->tune.split_max;
  if (tiles < target * h->num_sms) {  // split K over a cluster of at most 16 CTAs
    splits = std::max(1, std::min({kblocks, target * h->num_sms / tiles, split_max}));
    const int kpb = (kblocks + splits - 1) / splits;
    splits = (kblocks + kpb - 1) / kpb;
  }
  g->splits = splits;
  g->kb_per_split = (kblocks + splits - 1) / splits;
  g->tile_major = (splits == 1 && g->n_tok_tiles > 1) ? 1 : 0;
  return nt;
}

// Kernel trace slot of the next launch (null when tracing is off, capturing, or full): one
// [kKtraceMaxCta][kKtracePhases] record per launch, zeroed (= not reached) between reads.
constexpr size_t kKtraceMax = 512;
constexpr size_t kKtraceRec = static_cast<size_t>(kKtraceMaxCta) * kKtracePhases;
static unsigned long long* ktrace_slot(fdllm_handle* h, int kind) {
  if (!h->ktrace_on || h->capturing || h->ktrace_kind.size() >= kKtraceMax) return nullptr;
  const size_t i = h->ktrace_kind.size();
  h->ktrace_kind.push_back(kind);
  return h->ktrace.p + kKtraceRec * i;
}

static int ktrace_reset(fdllm_handle* h) {
  h->ktrace_kind.clear();
  FDLLM_TRY(h->ktrace.ensure(kKtraceRec * kKtraceMax));
  CUDA_TRY(cudaMemset(h->ktrace.p, 0, kKtraceRec * kKtraceMax * sizeof(unsigned long long)));
  return FDLLM_OK;
}

// norm_w set (tcgen05 path only): X is the un-normalized input and the kernel applies RMSNorm
// with weight norm_w while building its B operand.
static int run_gemm(fdllm_handle* h, const Weight& w, const void* X, int M, Epilogue epi, cudaStream_t s,
                    const void* norm_w = nullptr) {
  if (M <= 0) return FDLLM_OK;
  // Short-K few-slab projections (qkv, o: K = 1536, <= 16 slabs) of a call the persistent kernel
  // would cover with at most one 128-token tile per CTA (256-1152 rows) stay on the per-tile kernel
  // with tune.short_k_nt-token tiles: the persistent kernel cannot overlap a lone tile's short
  // main loop with another tile's epilogue (1024 rows: qkv 24.2 -> 20.3 us, o 13.4 -> 12.4 us).
  const bool short_k = h->dtype == FDLLM_BFLOAT16 && h->tune.short_k_nt > 0 && norm_w == nullptr &&
                       use_persist(h, M) && !w.paired && w.cols <= 2048 && w.rows / 128 <= 16 &&
                       (w.rows / 128) * ((M + 127) / 128) <= h->num_sms;
  GemmArgs g{};
  const int nt = plan_gemm(h, w, M, &g, short_k ? h->tune.short_k_nt : 0);
  g.err = h->err.p;
  g.epi = epi;
  if (norm_w != nullptr) {
    g.norm_x = X;
    g.norm_w = norm_w;
    g.norm_ss = h->ss.p;
    g.norm_ss_ld = h->cfg.hidden_size / 128;
    g.norm_eps = h->cfg.rms_norm_eps;
  }
  if (h->dtype == FDLLM_FLOAT32) return timed_launch(h, g, s, launch_simt_thunk, w.ptr, X, 0);
  g.ktrace = ktrace_slot(h, 100 + epi.kind + (norm_w ? 2000 : 0));
  g.tune = h->tune.gemm_tune;
  if (norm_w == nullptr && use_persist(h, M) && !short_k) {
    g.tune |= (h->tune.persist_l2_ahead & 0xff) << kGemmTunePersistL2Shift;
    if (h->tune.persist_conf_t && !w.paired && (epi.kind == kEpiConf || epi.kind == kEpiLseGather)) {
      // lm_head + confidence: 128-token tiles on the MMA's M side against slab pairs, each
      // epilogue thread reducing one token's slab in registers (1024 rows: 0.80 ms with the
      // tokens on N and the reductions across lanes)
      g.conf_t = 1;
      g.n_slabs = g.N / 128;
      g.n_tok_tiles = (M + 127) / 128;
      g.tile_n = 256;
      g.splits = 1;
      g.kb_per_split = g.K / 64;
      const int tiles = (g.n_slabs + 1) / 2 * g.n_tok_tiles;
      CUtensorMap tmB;
      FDLLM_TRY(cached_map(h, &tmB, X, M, g.K, 128));
      return timed_launch(h, g, s, launch_persist_thunk, &w.map, &tmB, std::min(h->num_sms, tiles));
    }
    g.n_slabs = w.paired ? (g.N / 2) / 64 : g.N / 128;
    // 256-token tiles when they cover half the SMs, else 128 (twice the tiles for few-slab weights).
    // 96-token tiles where they shorten the busiest SM's share (rounds of tiles x tile height) by
    // at least 15%: the few-slab projections of a 1024-row step (o, down: 132 tiles in one round
    // instead of 96 of 128 rows).
    int pnt = 2 * g.n_slabs * ((M + 255) / 256) >= h->num_sms ? 256 : 128;
    auto share = [&](int nt) {
      const long long tiles = static_cast<long long>(g.n_slabs) * ((M + nt - 1) / nt);
      return (tiles + h->num_sms - 1) / h->num_sms * nt;
    };
    if (h->tune.persist_nt96 && share(96) * 100 <= share(pnt) * 85) pnt = 96;
    const int kblocks = g.K / 64;
    // Long-K few-slab projections (down: K = 8960, 12 slabs) read every weight slab once per token
    // tile and every token tile once per slab through L2.  With persist_splitk = 2 they take
    // 256-token tiles with K split 2-4 ways so that the (tile, split) units still fill the SMs:
    // a third less L2 traffic for down at 1024 rows.
    // Split K (<= 4 ways, >= 8 k blocks each) when the tiles cover at most half the SMs (the
    // projections of a short prefill).
    int splits = 1;
    const int tiles0 = g.n_slabs * ((M + pnt - 1) / pnt);
    if ((h->tune.persist_splitk & 1) && tiles0 * 2 <= h->num_sms)
      while (splits < 4 && tiles0 * splits < h->num_sms && kblocks / (2 * splits) >= 8) splits *= 2;
    // The long-K plan wins when it covers at least as many SMs (down at 1024 rows: 48 tiles x 3
    // splits against 132 unsplit 96-token tiles; at 224 rows 12 x 4 loses to 36 x 4).
    if ((h->tune.persist_splitk & 2) && kblocks >= 64) {
      const int t256 = g.n_slabs * ((M + 255) / 256);
      const int sp = std::min(4, h->num_sms / std::max(t256, 1));
      if (sp >= 2 && kblocks / sp >= 32 && t256 * sp >= tiles0 * splits) {
        pnt = 256;
        splits = sp;
      }
    }
    g.n_tok_tiles = (M + pnt - 1) / pnt;
    g.tile_n = pnt;
    const int tiles = g.n_slabs * g.n_tok_tiles;
    g.splits = splits;
    g.kb_per_split = (kblocks + splits - 1) / splits;
    const int grid = std::min(h->num_sms, tiles * splits);
    if (splits > 1) {
      FDLLM_TRY(h->persist_part.ensure(static_cast<size_t>(tiles) * splits * pnt * 128));
      FDLLM_TRY(h->persist_ctr.ensure(2 * static_cast<size_t>(tiles), true));
      g.ppart = h->persist_part.p;
      g.pctr = h->persist_ctr.p;
      // all splits of a tile run at once only when no CTA holds two units (one wave)
      g.pmerge_all = h->tune.persist_merge_all && tiles * splits <= grid ? 1 : 0;
    }
    CUtensorMap tmB;
    FDLLM_TRY(cached_map(h, &tmB, X, M, g.K, pnt));
    return timed_launch(h, g, s, launch_persist_thunk, &w.map, &tmB, grid);
  }
  CUtensorMap tmB;
  FDLLM_TRY(cached_map(h, &tmB, X, M, g.K, nt));
  return timed_launch(h, g, s, launch_tc_thunk, &w.map, &tmB, nt);
}

// Key-split plan of the attention: enough CTAs to cover the SMs at small batch.  `max_l` is the
// longest key range the launch may see (the cache capacity for a replayable graph).
static void plan_attention(const fdllm_handle* h, int max_q, int max_l, int nreq, bool dense, int* n_splits,
                           int* split_len) {
  const fdllm_config& c = h->cfg;
  const int qtiles = (max_q + 15) / 16;
  const int base_ctas = qtiles * c.num_key_value_heads * nreq;
  *n_splits = 1;
  *split_len = std::max(64, static_cast<int>(round_up(std::max(max_l, 1), 64)));
  if (h->dtype == FDLLM_BFLOAT16 && !dense && base_ctas < h->num_sms) {
    // as many splits as keep the grid within one CTA per SM: a second wave, or two CTAs per SM
    // merging through distributed shared memory, costs more than the longer key loop (measured
    // per layer: 32 requests x 768 keys 32 µs unsplit vs 47 µs with 3 splits; 8 x 4096 keys 44 µs
    // with 4 splits vs 59 µs with 8)
    int want = std::min({h->num_sms / base_ctas, (max_l + 63) / 64, kMaxAttnSplits});
    if (h->tune.attn_splits > 0) want = std::min(h->tune.attn_splits, kMaxAttnSplits);
    if (want > 1) {
      *n_splits = want;
      *split_len = 64;  // the kernel divides each request's own key range evenly
    }
  }
}

// ---- workspace ----------------------------------------------------------------------------
static int ensure_ws(fdllm_handle* h, int M, int nreq) {
  const fdllm_config& c = h->cfg;
  const size_t m = round_up(static_cast<size_t>(std::max(M, 1)), 64);
  const size_t qd = static_cast<size_t>(c.num_attention_heads) * c.head_dim;
  FDLLM_TRY(h->h.ensure(m * c.hidden_size * h->esz));
  FDLLM_TRY(h->xn.ensure(m * std::max<size_t>(c.hidden_size, c.intermediate_size) * h->esz));
  FDLLM_TRY(h->q.ensure(m * qd * h->esz));
  FDLLM_TRY(h->attn.ensure(m * qd * h->esz));
  FDLLM_TRY(h->act.ensure(m * c.intermediate_size * h->esz));
  FDLLM_TRY(h->tok_req.ensure(m));
  FDLLM_TRY(h->tok_pos.ensure(m));
  FDLLM_TRY(h->tok_row.ensure(m));
  FDLLM_TRY(h->tmp_ids.ensure(m));
  FDLLM_TRY(h->tmp_maxp.ensure(m));
  FDLLM_TRY(h->targets.ensure(m));
  FDLLM_TRY(h->reqs.ensure(static_cast<size_t>(std::max(nreq, 1))));
  FDLLM_TRY(h->ss.ensure(m * (c.hidden_size / 128 + 1)));
  return FDLLM_OK;
}

static TokenMaps token_maps(fdllm_handle* h) { return TokenMaps{h->tok_req.p, h->tok_pos.p, h->tok_row.p}; }

// ---- the layer stack ----------------------------------------------------------------------

int fdllm::reserve_workspace(fdllm_handle* h, int M, int nreq, int max_l) {
  FDLLM_TRY(ensure_ws(h, M, nreq));
  const fdllm_config& c = h->cfg;
  int n_splits, split_len;
  plan_attention(h, M, max_l, nreq, false, &n_splits, &split_len);
  FDLLM_TRY(h->conf_part.ensure(static_cast<size_t>(M) * ((c.vocab_size + 127) / 128) * 4));
  return FDLLM_OK;
}

// ---- the layer stack ----------------------------------------------------------------------
// x: [M, hidden] input embeddings; reqs: host descriptors (q_tok0 / n_q filled); bias: dense fp32
// bias of request 0 (or null), causal_block: implicit block-causal mask when bias is null.
int fdllm::forward_core(fdllm_handle* h, const void* x, int M, std::vector<ReqDesc>& reqs, const float* bias,
                        int ld_bias, int causal_block, void* out, cudaStream_t s, int max_l_hint) {
  const fdllm_config& c = h->cfg;
  const int nreq = static_cast<int>(reqs.size());
  FDLLM_TRY(ensure_ws(h, M, nreq));
  for (int first = 0; first < nreq; first += kMaxReqsPerLaunch) {
    ReqBatch b{};
    b.n = std::min(kMaxReqsPerLaunch, nreq - first);
    b.first = first;
    for (int i = 0; i < b.n; ++i) b.r[i] = reqs[first + i];
    CUDA_TRY(launch_prepare(b, h->reqs.p, token_maps(h), c.max_positions, h->err.p, s));
  }

  int max_q = 0, max_l = 0;
  for (const ReqDesc& r : reqs) {
    max_q = std::max(max_q, r.n_q);
    max_l = std::max(max_l, r.plen_dev ? r.cap : r.attend_len);
  }
  if (max_l_hint > 0) max_l = max_l_hint;
  int n_splits, split_len;
  plan_attention(h, max_q, max_l, nreq, bias != nullptr || causal_block != 0, &n_splits, &split_len);

  // tcgen05 attention for calls with many query tokens per request (prefill, batched steps): its
  // per-request K/V tensor maps are encoded here and uploaded once for all layers.  Not inside a
  // stream capture, and not for device-side prefix lengths (the maps carry the attended length).
  // It runs one CTA per (request, KV head, query tile) without key splits, so it takes the call when
  // a request has attn_tc_min_q query tokens or the tiles alone cover attn_tc_min_ctas CTAs (a
  // batched step); a lone decode-sized request keeps the key-split mma.sync kernel (32 rows at
  // prefix 384: 1.41 ms per step against 1.55; 32 requests x 32 rows: 4.68 ms against 4.96).
  const int gqa = c.num_attention_heads / c.num_key_value_heads;
  const int tc_ctas = nreq * c.num_key_value_heads * ((max_q + 128 / gqa - 1) / (128 / gqa));
  // Long cached key ranges with few (request, KV head, query tile) CTAs: the tcgen05 kernel with the
  // keys split (up to 8 ways, >= 256 keys each) so that the grid covers the SMs, and a merge launch
  // (8 requests x 32 rows over 4096 keys: 27 against 43.5 us a layer on the mma.sync kernel).
  int tc_splits = 1;
  if (bias == nullptr && causal_block == 0 && h->tune.attn_tc_split_min_keys > 0 &&
      max_l >= h->tune.attn_tc_split_min_keys && tc_ctas > 0)
    tc_splits = std::max(1, std::min({kMaxAttnSplits,
                                      h->tune.attn_tc_split_target == 2 ? (2 * h->num_sms + tc_ctas - 1) / tc_ctas
                                                                        : h->num_sms / tc_ctas,
                                      max_l / 256}));
  bool attn_tc = h->dtype == FDLLM_BFLOAT16 && c.head_dim == 128 && bias == nullptr && !h->capturing && gqa <= 16 &&
                 h->tune.attn_tc_min_q > 0 &&
                 (max_q >= h->tune.attn_tc_min_q || tc_ctas >= h->tune.attn_tc_min_ctas || tc_splits > 1);
  for (const ReqDesc& r : reqs) attn_tc = attn_tc && r.plen_dev == nullptr && r.attend_len > 0;
  if (attn_tc) {
    // The maps depend on each request's caches and attended length only: a call with the same
    // requests as the previous one (the steps of one block) reuses the uploaded maps.
    std::vector<long long> key;
    key.reserve(4 * static_cast<size_t>(nreq));
    for (const ReqDesc& r : reqs) {
      key.push_back(reinterpret_cast<long long>(r.k));
      key.push_back(reinterpret_cast<long long>(r.v));
      key.push_back((static_cast<long long>(r.cap) << 32) | static_cast<unsigned>(r.attend_len));
      key.push_back(r.layer_stride);
    }
    const bool reuse = key == h->attn_maps_key && h->attn_maps.n >= 2 * static_cast<size_t>(nreq);
    std::vector<CUtensorMap> maps(reuse ? 0 : 2 * static_cast<size_t>(nreq));
    const size_t row_bytes = static_cast<size_t>(c.num_key_value_heads) * c.head_dim * h->esz;
    for (int i = 0; i < nreq && !reuse; ++i) {
      const ReqDesc& r = reqs[i];
      const int layers = r.layer_stride != 0 ? c.num_hidden_layers : 1;
      const size_t layer_bytes = static_cast<size_t>(r.cap) * row_bytes;
      FDLLM_TRY(make_kv_map(&maps[2 * i], r.k, c.num_key_value_heads * c.head_dim, r.attend_len, layers, row_bytes,
                            layer_bytes));
      FDLLM_TRY(make_kv_map(&maps[2 * i + 1], r.v, c.num_key_value_heads * c.head_dim, r.attend_len, layers, row_bytes,
                            layer_bytes));
    }
    if (!reuse) h->attn_maps_key.clear();  // set again below once the upload is queued
    FDLLM_TRY(h->attn_maps.ensure(2 * static_cast<size_t>(nreq)));
    if (tc_splits > 1) {
      const size_t rows = static_cast<size_t>(tc_splits) * M * c.num_attention_heads;
      FDLLM_TRY(h->attn_part.ensure(rows * c.head_dim));
      FDLLM_TRY(h->attn_part_lse.ensure(rows));
    }
    if (!reuse) {
      CUDA_TRY(cudaMemcpyAsync(h->attn_maps.p, maps.data(), maps.size() * sizeof(CUtensorMap), cudaMemcpyHostToDevice, s));
      h->attn_maps_key = std::move(key);
    }
  }

  Epilogue base{};
  base.hq = c.num_attention_heads;
  base.hkv = c.num_key_value_heads;
  base.hd = c.head_dim;
  base.reqs = h->reqs.p;
  base.tok = token_maps(h);
  base.rope_cos = h->rope_cos.p;
  base.rope_sin = h->rope_sin.p;
  base.max_pos = c.max_positions;

  // Decode-sized calls fold each layer's input RMSNorm into the qkv projection (its CTAs normalize
  // their B tiles in place, with row statistics left by the previous down projection); large calls
  // normalize once in a separate kernel.  The post-attention RMSNorm is folded into gate_up the
  // same way up to tune.gu_fused_rows token rows (a stage's normalisation is short there); above,
  // a separate vectorized rmsnorm kernel is faster (32 rows: 1.41 ms per step against 1.52).
  const bool fuse_norm = h->dtype == FDLLM_BFLOAT16 && M <= 64 && c.hidden_size <= 2560;
  const bool fuse_norm_gu = fuse_norm && M <= h->tune.gu_fused_rows;

  for (int l = 0; l < c.num_hidden_layers; ++l) {
    const LayerW& L = h->layers[l];
    const void* layer_in = l == 0 ? x : h->h.p;
    Epilogue e = base;
    e.kind = kEpiQkvRope;
    e.layer = l;
    e.bias = L.qkv_b;
    e.qout = h->q.p;
    if (fuse_norm && l > 0) {  // layer 0's input has no producer epilogue
      FDLLM_TRY(run_gemm(h, L.qkv, layer_in, M, e, s, L.ln1));
    } else {
      // layer 0 reads the input embeddings and starts the residual stream h as their copy
      CUDA_TRY(launch_rmsnorm(layer_in, L.ln1, h->xn.p, M, c.hidden_size, c.rms_norm_eps, h->dtype, s,
                              l == 0 ? h->h.p : nullptr));
      FDLLM_TRY(run_gemm(h, L.qkv, h->xn.p, M, e, s));
    }

    AttnArgs a{};
    a.q = h->q.p;
    a.out = h->attn.p;
    a.reqs = h->reqs.p;
    a.n_reqs = nreq;
    a.layer = l;
    a.hq = c.num_attention_heads;
    a.hkv = c.num_key_value_heads;
    a.hd = c.head_dim;
    a.scale = 1.0f / std::sqrt(static_cast<float>(c.head_dim));
    a.bias = bias;
    a.ld_bias = ld_bias;
    a.causal_block = causal_block;
    a.n_splits = n_splits;
    a.split_len = split_len;
    a.m_total = M;
    a.err = h->err.p;
    a.ktrace = h->dtype == FDLLM_BFLOAT16 ? ktrace_slot(h, attn_tc ? 2 : 1) : nullptr;
    if (attn_tc) {
      a.lazy_log2 = static_cast<float>(h->tune.attn_lazy_log2);
      a.n_splits = tc_splits;
      a.part = h->attn_part.p;
      a.part_lse = h->attn_part_lse.p;
      CUDA_TRY(launch_attention_tc(a, h->attn_maps.p, max_q, h->num_sms, s));
    } else {
      CUDA_TRY(launch_attention(a, max_q, h->dtype, s));
    }

    e = base;
    e.kind = kEpiResidual;
    e.resid = h->h.p;
    e.ld_resid = c.hidden_size;
    if (fuse_norm_gu) {  // leave the statistics of the post-attention RMSNorm
      e.ss_out = h->ss.p;
      e.ss_ld = c.hidden_size / 128;
    }
    FDLLM_TRY(run_gemm(h, L.o, h->attn.p, M, e, s));

    e = base;
    e.kind = kEpiSiluMul;
    e.out = h->act.p;
    e.ld_out = c.intermediate_size;
    if (fuse_norm_gu) {
      FDLLM_TRY(run_gemm(h, L.gu, h->h.p, M, e, s, L.ln2));
    } else {
      CUDA_TRY(launch_rmsnorm(h->h.p, L.ln2, h->xn.p, M, c.hidden_size, c.rms_norm_eps, h->dtype, s));
      FDLLM_TRY(run_gemm(h, L.gu, h->xn.p, M, e, s));
    }

    e = base;
    e.kind = kEpiResidual;
    e.resid = h->h.p;
    e.ld_resid = c.hidden_size;
    if (fuse_norm) {  // leave the statistics of the next layer's input RMSNorm
      e.ss_out = h->ss.p;
      e.ss_ld = c.hidden_size / 128;
    }
    FDLLM_TRY(run_gemm(h, L.down, h->act.p, M, e, s));
  }
  // out == null (build_prefix_cache): the final hidden states are not needed; xn is free by now.
  CUDA_TRY(launch_rmsnorm(h->h.p, h->final_norm, out ? out : h->xn.p, M, c.hidden_size, c.rms_norm_eps, h->dtype, s));
  return FDLLM_OK;
}

long long fdllm::layer_stride(const fdllm_handle* h, int cap) {
  return static_cast<long long>(cap) * h->cfg.num_key_value_heads * h->cfg.head_dim;
}

int fdllm::check_handle(fdllm_handle* h) {
  if (h == nullptr) return fail(FDLLM_ERR_INVALID, "null handle");
  if (!h->bound) return fail(FDLLM_ERR_UNBOUND, "parameters are not bound (call fdllm_bind_params)");
  cudaError_t e = cudaSetDevice(h->device);
  if (e != cudaSuccess) return fail(FDLLM_ERR_CUDA, std::string("cudaSetDevice: ") + cudaGetErrorString(e));
  return FDLLM_OK;
}

// Validate one cached request (runtime.py:56-57, 69-70, 258-263) and fill its descriptor.
int fdllm::cached_desc(fdllm_handle* h, const fdllm_request& r, int q_tok0, ReqDesc* d) {
  if (r.rows <= 0) return fail(FDLLM_ERR_INVALID, "rows must be positive");
  if (r.k_cache == nullptr || r.v_cache == nullptr) return fail(FDLLM_ERR_INVALID, "null KV cache");
  const long long write_start = static_cast<long long>(r.prefix_len) + r.write_rel;
  const long long attend_len = static_cast<long long>(r.prefix_len) + r.attend_rel;
  if (r.prefix_len < 0 || write_start < 0 || write_start + r.rows > r.cap)
    return fail(FDLLM_ERR_INVALID, "KV write [" + std::to_string(write_start) + ", " +
                                       std::to_string(write_start + r.rows) + ") outside cache capacity " +
                                       std::to_string(r.cap));
  if (write_start + r.rows > attend_len)
    return fail(FDLLM_ERR_INVALID, "KV write [" + std::to_string(write_start) + ", " +
                                       std::to_string(write_start + r.rows) + ") past the attended rows [0, " +
                                       std::to_string(attend_len) + ")");
  if (attend_len > r.cap)
    return fail(FDLLM_ERR_INVALID, "cached call needs " + std::to_string(attend_len) +
                                       " rows; cache capacity is " + std::to_string(r.cap));
  if (r.cache_offset_dev == nullptr &&
      (r.cache_offset_host < 0 || r.cache_offset_host + r.rows > h->cfg.max_positions))
    return fail(FDLLM_ERR_INVALID, "RoPE positions exceed max_positions");
  ReqDesc x{};
  x.k = r.k_cache;
  x.v = r.v_cache;
  x.layer_stride = layer_stride(h, r.cap);
  x.cap = r.cap;
  x.q_tok0 = q_tok0;
  x.n_q = r.rows;
  x.write_start = static_cast<int>(write_start);
  x.attend_len = static_cast<int>(attend_len);
  x.rope_base = r.cache_offset_host;
  x.rope_off = r.cache_offset_dev;
  *d = x;
  return FDLLM_OK;
}

// ---- the C ABI ---------------------------------------------------------------------------
extern "C" {

int fdllm_abi_version(void) { return FDLLM_ABI_VERSION; }

const char* fdllm_last_error(void) { return g_last_error.c_str(); }

int fdllm_create(const fdllm_config* cfg, int device, fdllm_handle** out) {
  if (cfg == nullptr || out == nullptr) return fail(FDLLM_ERR_INVALID, "null argument");
  *out = nullptr;
  const fdllm_config& c = *cfg;
  if (c.dtype != FDLLM_FLOAT32 && c.dtype != FDLLM_BFLOAT16) return fail(FDLLM_ERR_UNSUPPORTED, "dtype must be fp32 or bf16");
  if (c.hidden_size <= 0 || c.num_hidden_layers <= 0 || c.num_attention_heads <= 0 || c.num_key_value_heads <= 0 ||
      c.num_attention_heads % c.num_key_value_heads != 0 || c.head_dim % 32 != 0 || c.head_dim > 128)
    return fail(FDLLM_ERR_UNSUPPORTED, "unsupported head layout (head_dim must be 32/64/96/128, heads % kv_heads == 0)");
  if (c.max_positions <= 0 || c.bd_size <= 0 || c.bd_size > 32) return fail(FDLLM_ERR_INVALID, "bad max_positions / bd_size");
  const int qkv = (c.num_attention_heads + 2 * c.num_key_value_heads) * c.head_dim;
  if (c.dtype == FDLLM_BFLOAT16) {
    if (c.hidden_size % 128 || qkv % 128 || c.intermediate_size % 128 || c.vocab_size % 128 ||
        (c.num_attention_heads * c.head_dim) % 128 || 128 % c.head_dim)
      return fail(FDLLM_ERR_UNSUPPORTED, "bf16 tcgen05 path needs hidden, qkv, intermediate and vocab sizes "
                                         "divisible by 128 and head_dim dividing 128");
  } else if (c.hidden_size % 32 || c.intermediate_size % 32 || (c.num_attention_heads * c.head_dim) % 32 ||
             qkv % 128 || 128 % c.head_dim) {
    return fail(FDLLM_ERR_UNSUPPORTED, "fp32 path needs sizes divisible by 32, qkv by 128, head_dim dividing 128");
  }
  Tuning tune;
  FDLLM_TRY(parse_tuning(std::getenv("FDLLM_TUNING"), &tune));
  CUDA_TRY(cudaSetDevice(device));
  CUDA_TRY(init_kernel_attributes());
  fdllm_handle* h = new fdllm_handle();
  h->tune = tune;
  h->cfg = c;
  h->device = device;
  h->dtype = c.dtype;
  h->esz = c.dtype == FDLLM_BFLOAT16 ? 2 : 4;
  cudaDeviceGetAttribute(&h->num_sms, cudaDevAttrMultiProcessorCount, device);
  const size_t tab = static_cast<size_t>(c.max_positions) * (c.head_dim / 2) * h->esz;
  int r = h->rope_cos.ensure(tab);
  if (r == FDLLM_OK) r = h->rope_sin.ensure(tab);
  if (r == FDLLM_OK) r = h->err.ensure(4, true);
  if (r != FDLLM_OK) {
    fdllm_destroy(h);
    return r;
  }
  cudaError_t e = static_cast<cudaError_t>(
      launch_rope_tables(h->rope_cos.p, h->rope_sin.p, c.max_positions, c.head_dim, c.rope_theta, h->dtype, 0));
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    fdllm_destroy(h);
    return fail(FDLLM_ERR_CUDA, std::string("rope tables: ") + cudaGetErrorString(e));
  }
  *out = h;
  return FDLLM_OK;
}

int fdllm_destroy(fdllm_handle* h) {
  if (h == nullptr) return FDLLM_OK;
  cudaSetDevice(h->device);
  cudaDeviceSynchronize();
  for (auto* b : {&h->rope_cos, &h->rope_sin, &h->h, &h->xn, &h->q, &h->attn, &h->act, &h->scratch_k, &h->scratch_v,
                  &h->dec.k, &h->dec.v, &h->dec.x, &h->dec.hid})
    b->release();
  for (auto* b : {&h->err, &h->tok_req, &h->tok_pos, &h->tok_row, &h->tmp_ids, &h->targets, &h->dec.ids,
                  &h->dec.block, &h->dec.cids, &h->dec.out})
    b->release();
  for (auto* b : {&h->conf_part, &h->tmp_maxp, &h->ss, &h->dec.cmax}) b->release();
  h->persist_part.release();
  h->persist_ctr.release();
  h->ktrace.release();
  h->attn_maps.release();
  h->reqs.release();
  if (h->dec.host) cudaFreeHost(h->dec.host);
  if (h->dec.host_params) cudaFreeHost(h->dec.host_params);
  for (cudaEvent_t e : h->prof_ev) cudaEventDestroy(e);
  release_step_graphs(h);
  h->dec.plen.release();
  h->dec.loop.release();
  if (h->dec.stream) cudaStreamDestroy(h->dec.stream);
  delete h;
  return FDLLM_OK;
}

int fdllm_bind_params(fdllm_handle* h, const void* const* ptrs, int n) {
  if (h == nullptr || ptrs == nullptr) return fail(FDLLM_ERR_INVALID, "null argument");
  std::lock_guard<std::mutex> lock(h->mu);
  const fdllm_config& c = h->cfg;
  const int expect = 1 + 7 * c.num_hidden_layers + 1 + (c.tie_word_embeddings ? 0 : 1);
  if (n != expect)
    return fail(FDLLM_ERR_INVALID, "expected " + std::to_string(expect) + " params, got " + std::to_string(n));
  for (int i = 0; i < n; ++i)
    if (ptrs[i] == nullptr || (reinterpret_cast<uintptr_t>(ptrs[i]) & 15) != 0)
      return fail(FDLLM_ERR_INVALID, "param " + std::to_string(i) + " is null or not 16-byte aligned");
  CUDA_TRY(cudaSetDevice(h->device));
  const int qkv = (c.num_attention_heads + 2 * c.num_key_value_heads) * c.head_dim;
  const int qd = c.num_attention_heads * c.head_dim;
  h->embed = ptrs[0];
  h->layers.assign(c.num_hidden_layers, LayerW{});
  for (int l = 0; l < c.num_hidden_layers; ++l) {
    const void* const* p = ptrs + 1 + 7 * l;
    LayerW& L = h->layers[l];
    L.qkv = Weight{p[0], qkv, c.hidden_size, false, {}};
    L.qkv_b = p[1];
    L.o = Weight{p[2], c.hidden_size, qd, false, {}};
    L.gu = Weight{p[3], 2 * c.intermediate_size, c.hidden_size, true, {}};
    L.down = Weight{p[4], c.hidden_size, c.intermediate_size, false, {}};
    L.ln1 = p[5];
    L.ln2 = p[6];
  }
  h->final_norm = ptrs[1 + 7 * c.num_hidden_layers];
  h->lm = Weight{c.tie_word_embeddings ? ptrs[0] : ptrs[n - 1], c.vocab_size, c.hidden_size, false, {}};
  if (h->dtype == FDLLM_BFLOAT16) {
    for (LayerW& L : h->layers) {
      FDLLM_TRY(make_map(&L.qkv.map, L.qkv.ptr, L.qkv.rows, L.qkv.cols, 128));
      FDLLM_TRY(make_map(&L.o.map, L.o.ptr, L.o.rows, L.o.cols, 128));
      FDLLM_TRY(make_map(&L.gu.map, L.gu.ptr, L.gu.rows, L.gu.cols, 64));
      FDLLM_TRY(make_map(&L.down.map, L.down.ptr, L.down.rows, L.down.cols, 128));
    }
    FDLLM_TRY(make_map(&h->lm.map, h->lm.ptr, h->lm.rows, h->lm.cols, 128));
  }
  h->bound = true;
  return FDLLM_OK;
}

int fdllm_embed(fdllm_handle* h, const int32_t* ids, int n, void* out, void* stream) {
  FDLLM_TRY(check_handle(h));
  if (n < 0 || (n > 0 && (ids == nullptr || out == nullptr))) return fail(FDLLM_ERR_INVALID, "bad embed arguments");
  std::lock_guard<std::mutex> lock(h->mu);
  CUDA_TRY(launch_embed(ids, n, h->embed, h->cfg.vocab_size, h->cfg.hidden_size, out, h->dtype, h->err.p,
                        static_cast<cudaStream_t>(stream)));
  return FDLLM_OK;
}

}  // extern "C"

int fdllm::dense_forward(fdllm_handle* h, const void* x, const float* bias, int T, void* k, void* v, int cap,
                         bool scratch, void* out, cudaStream_t s) {
  const fdllm_config& c = h->cfg;
  ReqDesc d{};
  if (scratch) {
    const size_t bytes = static_cast<size_t>(T) * c.num_key_value_heads * c.head_dim * h->esz;
    FDLLM_TRY(h->scratch_k.ensure(bytes));
    FDLLM_TRY(h->scratch_v.ensure(bytes));
    d.k = h->scratch_k.p;
    d.v = h->scratch_v.p;
    d.layer_stride = 0;
    d.cap = T;
  } else {
    d.k = k;
    d.v = v;
    d.layer_stride = layer_stride(h, cap);
    d.cap = cap;
  }
  d.q_tok0 = 0;
  d.n_q = T;
  d.write_start = 0;
  d.attend_len = T;
  d.rope_base = 0;
  d.rope_off = nullptr;
  std::vector<ReqDesc> reqs{d};
  return forward_core(h, x, T, reqs, bias, T, bias == nullptr ? c.bd_size : 0, out, s);
}

extern "C" {


int fdllm_forward_hidden(fdllm_handle* h, const void* x, const float* bias, int T, void* out, void* stream) {
  FDLLM_TRY(check_handle(h));
  if (T <= 0 || x == nullptr || out == nullptr) return fail(FDLLM_ERR_INVALID, "bad forward_hidden arguments");
  if (T > h->cfg.max_positions) return fail(FDLLM_ERR_INVALID, "sequence longer than max_positions");
  std::lock_guard<std::mutex> lock(h->mu);
  return dense_forward(h, x, bias, T, nullptr, nullptr, 0, true, out, static_cast<cudaStream_t>(stream));
}

int fdllm_build_prefix_cache(fdllm_handle* h, const void* x, const float* bias, int P, void* k, void* v, int cap,
                             void* stream) {
  FDLLM_TRY(check_handle(h));
  if (P <= 0 || x == nullptr || k == nullptr || v == nullptr) return fail(FDLLM_ERR_INVALID, "bad build_prefix_cache arguments");
  if (P > cap) return fail(FDLLM_ERR_INVALID, "KV write [0, " + std::to_string(P) + ") outside cache capacity " + std::to_string(cap));
  if (P > h->cfg.max_positions) return fail(FDLLM_ERR_INVALID, "prefix longer than max_positions");
  std::lock_guard<std::mutex> lock(h->mu);
  return dense_forward(h, x, bias, P, k, v, cap, false, nullptr, static_cast<cudaStream_t>(stream));
}

int fdllm_build_prefix_cache_batch(fdllm_handle* h, const fdllm_request* reqs_host, int n, const void* x,
                                   void* stream) {
  FDLLM_TRY(check_handle(h));
  if (n <= 0 || reqs_host == nullptr || x == nullptr) return fail(FDLLM_ERR_INVALID, "bad prefix batch arguments");
  std::vector<ReqDesc> reqs(n);
  int tok = 0;
  for (int i = 0; i < n; ++i) {
    const fdllm_request& q = reqs_host[i];
    if (q.rows <= 0 || q.k_cache == nullptr || q.v_cache == nullptr)
      return fail(FDLLM_ERR_INVALID, "prefix request " + std::to_string(i) + ": bad rows or cache");
    if (q.rows > q.cap)
      return fail(FDLLM_ERR_INVALID, "prefix request " + std::to_string(i) + ": KV write [0, " + std::to_string(q.rows) +
                                         ") outside cache capacity " + std::to_string(q.cap));
    if (q.rows > h->cfg.max_positions) return fail(FDLLM_ERR_INVALID, "prefix longer than max_positions");
    ReqDesc d{};
    d.k = q.k_cache;
    d.v = q.v_cache;
    d.layer_stride = layer_stride(h, q.cap);
    d.cap = q.cap;
    d.q_tok0 = tok;
    d.n_q = q.rows;
    d.write_start = 0;
    d.attend_len = q.rows;
    d.rope_base = 0;
    d.rope_off = nullptr;
    reqs[i] = d;
    tok += q.rows;
  }
  std::lock_guard<std::mutex> lock(h->mu);
  return forward_core(h, x, tok, reqs, nullptr, 0, h->cfg.bd_size, nullptr, static_cast<cudaStream_t>(stream));
}

int fdllm_forward_cached(fdllm_handle* h, const void* x, int rows, void* k, void* v, int cap,
                         const int32_t* cache_offset_dev, int prefix_len, int write_rel, int attend_rel, void* out,
                         void* stream) {
  FDLLM_TRY(check_handle(h));
  if (x == nullptr || out == nullptr) return fail(FDLLM_ERR_INVALID, "null activation pointer");
  fdllm_request r{k, v, cap, rows, prefix_len, write_rel, attend_rel, prefix_len + write_rel, cache_offset_dev};
  std::vector<ReqDesc> reqs(1);
  FDLLM_TRY(cached_desc(h, r, 0, &reqs[0]));
  std::lock_guard<std::mutex> lock(h->mu);
  return forward_core(h, x, rows, reqs, nullptr, 0, 0, out, static_cast<cudaStream_t>(stream));
}

int fdllm_forward_cached_batch(fdllm_handle* h, const fdllm_request* reqs_host, int n, const void* x, void* out,
                               void* stream) {
  FDLLM_TRY(check_handle(h));
  if (n <= 0 || reqs_host == nullptr || x == nullptr || out == nullptr) return fail(FDLLM_ERR_INVALID, "bad batch arguments");
  std::vector<ReqDesc> reqs(n);
  int tok = 0;
  for (int i = 0; i < n; ++i) {
    FDLLM_TRY(cached_desc(h, reqs_host[i], tok, &reqs[i]));
    tok += reqs_host[i].rows;
  }
  std::lock_guard<std::mutex> lock(h->mu);
  return forward_core(h, x, tok, reqs, nullptr, 0, 0, out, static_cast<cudaStream_t>(stream));
}

int fdllm_get_logits(fdllm_handle* h, const void* hidden, int rows, float* logits, void* stream) {
  FDLLM_TRY(check_handle(h));
  if (rows <= 0 || hidden == nullptr || logits == nullptr) return fail(FDLLM_ERR_INVALID, "bad get_logits arguments");
  std::lock_guard<std::mutex> lock(h->mu);
  Epilogue e{};
  e.kind = kEpiLogitsF32;
  e.out = logits;
  e.ld_out = h->cfg.vocab_size;
  return run_gemm(h, h->lm, hidden, rows, e, static_cast<cudaStream_t>(stream));
}

}  // extern "C"

int fdllm::confidence_locked(fdllm_handle* h, const void* hidden, int rows, int32_t* ids, float* maxp,
                             const int32_t* targets, float* logprob, cudaStream_t s) {
  const int n_slabs = (h->cfg.vocab_size + 127) / 128;
  FDLLM_TRY(h->conf_part.ensure(static_cast<size_t>(rows) * n_slabs * 4));
  Epilogue e{};
  e.kind = targets ? kEpiLseGather : kEpiConf;
  e.part = h->conf_part.p;
  e.target = targets;
  FDLLM_TRY(run_gemm(h, h->lm, hidden, rows, e, s));
  if (targets) {
    CUDA_TRY(launch_lse_combine(h->conf_part.p, rows, n_slabs, logprob, s));
  } else {
    CUDA_TRY(launch_conf_combine(h->conf_part.p, rows, n_slabs, ids, maxp, s));
  }
  return FDLLM_OK;
}

extern "C" {


int fdllm_confidence(fdllm_handle* h, const void* hidden, int rows, int32_t* ids, float* maxp, void* stream) {
  FDLLM_TRY(check_handle(h));
  if (rows <= 0 || hidden == nullptr || ids == nullptr || maxp == nullptr) return fail(FDLLM_ERR_INVALID, "bad confidence arguments");
  std::lock_guard<std::mutex> lock(h->mu);
  return confidence_locked(h, hidden, rows, ids, maxp, nullptr, nullptr, static_cast<cudaStream_t>(stream));
}

int fdllm_confidence_from_logits(fdllm_handle* h, const float* logits, int rows, int32_t* ids, float* maxp,
                                 void* stream) {
  FDLLM_TRY(check_handle(h));
  if (rows <= 0 || logits == nullptr || ids == nullptr || maxp == nullptr) return fail(FDLLM_ERR_INVALID, "bad arguments");
  std::lock_guard<std::mutex> lock(h->mu);
  CUDA_TRY(launch_conf_from_logits(logits, rows, h->cfg.vocab_size, ids, maxp, static_cast<cudaStream_t>(stream)));
  return FDLLM_OK;
}

int fdllm_token_logprob(fdllm_handle* h, const void* hidden, int rows, const int32_t* targets, float* logprob,
                        void* stream) {
  FDLLM_TRY(check_handle(h));
  if (rows <= 0 || hidden == nullptr || targets == nullptr || logprob == nullptr) return fail(FDLLM_ERR_INVALID, "bad arguments");
  std::lock_guard<std::mutex> lock(h->mu);
  return confidence_locked(h, hidden, rows, nullptr, nullptr, targets, logprob, static_cast<cudaStream_t>(stream));
}

int fdllm_unmask(fdllm_handle* h, const int32_t* ids, const float* maxp, int rows, int32_t* block_tokens, int sub_start,
                 int sub_len, int partial, int mask_id, double threshold, int32_t* out_tokens, float* out_conf,
                 int32_t* out_unmask, int32_t* status, void* stream) {
  FDLLM_TRY(check_handle(h));
  if (ids == nullptr || maxp == nullptr || block_tokens == nullptr) return fail(FDLLM_ERR_INVALID, "null argument");
  if (sub_len <= 0 || sub_len > 32 || sub_start < 0 || sub_start + sub_len > h->cfg.bd_size)
    return fail(FDLLM_ERR_INVALID, "bad unmask window");
  if (partial ? rows != sub_len : rows < sub_start + sub_len) return fail(FDLLM_ERR_INVALID, "rows do not cover the window");
  CUDA_TRY(launch_unmask(ids, maxp, rows, block_tokens, sub_start, sub_len, partial, mask_id, threshold, out_tokens,
                         out_conf, out_unmask, status, static_cast<cudaStream_t>(stream)));
  return FDLLM_OK;
}

int fdllm_unmask_batch(fdllm_handle* h, const int32_t* ids, const float* maxp, const int32_t* desc, int n,
                       double threshold, int32_t* out, void* stream) {
  FDLLM_TRY(check_handle(h));
  if (n < 0 || (n > 0 && (ids == nullptr || maxp == nullptr || desc == nullptr || out == nullptr)))
    return fail(FDLLM_ERR_INVALID, "bad unmask batch arguments");
  CUDA_TRY(launch_unmask_batch(ids, maxp, desc, n, threshold, out, static_cast<cudaStream_t>(stream)));
  return FDLLM_OK;
}

int fdllm_device_error(fdllm_handle* h, int* code) {
  if (h == nullptr || code == nullptr) return fail(FDLLM_ERR_INVALID, "null argument");
  int w[4] = {0, 0, 0, 0};
  FDLLM_TRY(fdllm_device_error_detail(h, w));
  *code = w[0];
  return FDLLM_OK;
}

int fdllm_device_error_detail(fdllm_handle* h, int32_t* out4) {
  if (h == nullptr || out4 == nullptr) return fail(FDLLM_ERR_INVALID, "null argument");
  CUDA_TRY(cudaSetDevice(h->device));
  CUDA_TRY(cudaDeviceSynchronize());
  CUDA_TRY(cudaMemcpy(out4, h->err.p, 4 * sizeof(int), cudaMemcpyDeviceToHost));
  CUDA_TRY(cudaMemset(h->err.p, 0, 4 * sizeof(int)));
  return FDLLM_OK;
}

int fdllm_wait_selftest(fdllm_handle* h, unsigned long long limit_ns, int* code) {
  if (h == nullptr || code == nullptr) return fail(FDLLM_ERR_INVALID, "null argument");
  CUDA_TRY(cudaSetDevice(h->device));
  int* flag = nullptr;
  CUDA_TRY(cudaMalloc(&flag, sizeof(int)));
  cudaMemset(flag, 0, sizeof(int));
  cudaError_t e = static_cast<cudaError_t>(launch_wait_test(flag, h->err.p, limit_ns, 0));
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  cudaFree(flag);
  if (e != cudaSuccess) return fail(FDLLM_ERR_CUDA, std::string("wait self test: ") + cudaGetErrorString(e));
  return fdllm_device_error(h, code);
}

long long fdllm_kernel_launches(void) { return launch_count(); }

int fdllm_profile_enable(fdllm_handle* h, int enable) {
  if (h == nullptr) return fail(FDLLM_ERR_INVALID, "null handle");
  std::lock_guard<std::mutex> lock(h->mu);
  h->prof = enable != 0;
  return FDLLM_OK;
}

int fdllm_profile_read(fdllm_handle* h, double* out4) {
  if (h == nullptr || out4 == nullptr) return fail(FDLLM_ERR_INVALID, "null argument");
  std::lock_guard<std::mutex> lock(h->mu);
  CUDA_TRY(cudaSetDevice(h->device));
  double ms = 0.0;
  for (size_t i = 0; i + 1 < h->prof_used; i += 2) {
    CUDA_TRY(cudaEventSynchronize(h->prof_ev[i + 1]));
    float t = 0.f;
    CUDA_TRY(cudaEventElapsedTime(&t, h->prof_ev[i], h->prof_ev[i + 1]));
    ms += t;
  }
  out4[0] = ms + h->prof_ms_extra;
  out4[1] = h->prof_bytes;
  out4[2] = static_cast<double>(h->prof_used / 2 + h->prof_launch_extra);
  out4[3] = h->prof_flops;
  h->prof_used = 0;
  h->prof_bytes = h->prof_flops = h->prof_ms_extra = 0.0;
  h->prof_launch_extra = 0;
  return FDLLM_OK;
}

int fdllm_kernel_trace_enable(fdllm_handle* h, int enable) {
  if (h == nullptr) return fail(FDLLM_ERR_INVALID, "null handle");
  std::lock_guard<std::mutex> lock(h->mu);
  CUDA_TRY(cudaSetDevice(h->device));
  CUDA_TRY(cudaDeviceSynchronize());
  if (enable != 0) FDLLM_TRY(ktrace_reset(h));
  h->ktrace_on = enable != 0;
  return FDLLM_OK;
}

int fdllm_kernel_trace_read(fdllm_handle* h, uint64_t* out, int32_t* kinds, int cap, int32_t* n) {
  if (h == nullptr || n == nullptr) return fail(FDLLM_ERR_INVALID, "null argument");
  std::lock_guard<std::mutex> lock(h->mu);
  const int cnt = static_cast<int>(h->ktrace_kind.size());
  *n = cnt;
  if (out == nullptr || cnt == 0) return FDLLM_OK;
  if (cap < cnt || kinds == nullptr) return fail(FDLLM_ERR_INVALID, "trace buffer too small");
  CUDA_TRY(cudaSetDevice(h->device));
  CUDA_TRY(cudaDeviceSynchronize());
  std::vector<unsigned long long> rec(kKtraceRec * static_cast<size_t>(cnt));
  CUDA_TRY(cudaMemcpy(rec.data(), h->ktrace.p, rec.size() * sizeof(unsigned long long), cudaMemcpyDeviceToHost));
  for (int i = 0; i < cnt; ++i) {  // earliest and latest stamp of each phase over the launch's CTAs
    for (int p = 0; p < kKtracePhases; ++p) {
      unsigned long long lo = ~0ull, hi = 0;
      for (int c = 0; c < kKtraceMaxCta; ++c) {
        const unsigned long long t = rec[kKtraceRec * i + static_cast<size_t>(c) * kKtracePhases + p];
        if (t == 0) continue;
        lo = std::min(lo, t);
        hi = std::max(hi, t);
      }
      out[(static_cast<size_t>(i) * kKtracePhases + p) * 2] = lo;
      out[(static_cast<size_t>(i) * kKtracePhases + p) * 2 + 1] = hi;
    }
  }
  std::copy(h->ktrace_kind.begin(), h->ktrace_kind.end(), kinds);
  return ktrace_reset(h);
}

long long fdllm_workspace_bytes(fdllm_handle* h) {
  if (h == nullptr) return 0;
  long long t = 0;
  for (auto* b : {&h->h, &h->xn, &h->q, &h->attn, &h->act, &h->scratch_k, &h->scratch_v, &h->rope_cos, &h->rope_sin,
                  &h->dec.k, &h->dec.v, &h->dec.x, &h->dec.hid})
    t += static_cast<long long>(b->bytes());
  for (auto* b : {&h->conf_part, &h->tmp_maxp, &h->ss, &h->dec.cmax})
    t += static_cast<long long>(b->bytes());
  for (auto* b : {&h->err, &h->tok_req, &h->tok_pos, &h->tok_row, &h->tmp_ids, &h->targets, &h->dec.ids,
                  &h->dec.block, &h->dec.cids, &h->dec.out})
    t += static_cast<long long>(b->bytes());
  return t + static_cast<long long>(h->reqs.bytes());
}

}  // extern "C"

// ---- allocation-free confidence -------------------------------------------------------------
// The partials of the fused lm_head confidence live in a fixed module-scope device array instead
// of the handle's grown workspace, so the call allocates nothing.  Every (row, slab) entry the
// combine kernel reads is written earlier in the same call, so nothing in the array has to start
// at zero; it keeps the last call's contents.  One array per device, shared by every handle on it.
namespace {
constexpr size_t kStaticConfFloats = size_t(1) << 20;  // 4 MiB
__device__ __align__(256) float g_static_conf_part[kStaticConfFloats];
constexpr int kMaxStaticDevices = 64;
std::mutex g_static_mu;
// The array's device address per device, and the CUDA context it was looked up in: after a
// cudaDeviceReset (or any teardown of the primary context) the module is loaded again at another
// address, so a changed context triggers a fresh lookup instead of reusing a stale pointer.
float* g_static_conf_addr[kMaxStaticDevices] = {};
CUcontext g_static_conf_ctx[kMaxStaticDevices] = {};

typedef CUresult (*CtxGetCurrentFn)(CUcontext*);
CUcontext current_context() {
  static CtxGetCurrentFn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return static_cast<CtxGetCurrentFn>(nullptr);
    return reinterpret_cast<CtxGetCurrentFn>(p);
  }();
  CUcontext c = nullptr;
  if (fn != nullptr && fn(&c) != CUDA_SUCCESS) c = nullptr;
  return c;
}
}  // namespace

extern "C" int fdllm_confidence_static(fdllm_handle* h, const void* hidden, int rows, int32_t* ids, float* maxp,
                                       void* stream) {
  FDLLM_TRY(check_handle(h));
  if (rows <= 0 || hidden == nullptr || ids == nullptr || maxp == nullptr) return fail(FDLLM_ERR_INVALID, "bad confidence arguments");
  const int n_slabs = (h->cfg.vocab_size + 127) / 128;
  const size_t max_rows = kStaticConfFloats / (static_cast<size_t>(n_slabs) * 4);
  if (static_cast<size_t>(rows) > max_rows)
    return fail(FDLLM_ERR_INVALID, "fdllm_confidence_static: rows = " + std::to_string(rows) + " exceeds " +
                                       std::to_string(max_rows) + ", the most the fixed 4 MiB scratch holds at vocab " +
                                       std::to_string(h->cfg.vocab_size) + " (use fdllm_confidence)");
  if (h->device < 0 || h->device >= kMaxStaticDevices) return fail(FDLLM_ERR_UNSUPPORTED, "device ordinal out of range");
  float* part = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_static_mu);
    // check_handle made h->device current; the runtime call below initialises its context if needed
    void* p = nullptr;
    const CUcontext ctx = current_context();
    if (g_static_conf_addr[h->device] == nullptr || ctx == nullptr || ctx != g_static_conf_ctx[h->device]) {
      cudaError_t e = cudaGetSymbolAddress(&p, g_static_conf_part);  // first call on this device / context
      if (e != cudaSuccess || p == nullptr)
        return fail(FDLLM_ERR_CUDA, std::string("cudaGetSymbolAddress(static confidence scratch): ") + cudaGetErrorString(e));
      g_static_conf_addr[h->device] = static_cast<float*>(p);
      g_static_conf_ctx[h->device] = current_context();
    }
    part = g_static_conf_addr[h->device];
  }
  std::lock_guard<std::mutex> lock(h->mu);
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  Epilogue e{};
  e.kind = kEpiConf;
  e.part = part;
  GemmArgs g{};
  const int nt = plan_gemm(h, h->lm, rows, &g);
  g.err = h->err.p;
  g.epi = e;
  // The same launch path as fdllm_confidence (profiling counters, kernel trace, tuning bits).
  if (h->dtype == FDLLM_FLOAT32) {
    FDLLM_TRY(timed_launch(h, g, s, launch_simt_thunk, h->lm.ptr, hidden, 0));
  } else {
    g.ktrace = ktrace_slot(h, 100 + e.kind);
    g.tune = h->tune.gemm_tune;
    CUtensorMap tmB;
    FDLLM_TRY(make_map(&tmB, hidden, rows, g.K, nt));
    FDLLM_TRY(timed_launch(h, g, s, launch_tc_thunk, &h->lm.map, &tmB, nt));
  }
  CUDA_TRY(launch_conf_combine(part, rows, n_slabs, ids, maxp, s));
  return FDLLM_OK;
}
