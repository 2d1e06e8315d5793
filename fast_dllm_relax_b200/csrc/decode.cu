// Device-resident block-diffusion decode driver (greedy, threshold-parallel unmasking).
//
// Follows fast_dllm_relax/runtime.py:591-880 (relax_greedy_generate) for prompts of at least one
// block: the block-aligned prompt fast path (:679-708), the prefix-cache rebuild rule (:718-739),
// the sub-block refinement loop with the full / partial step choice (:748-805), the length and stop
// checks (:655-669, :839-849) and block-append (:851-878).  What differs is where the work runs:
// the token ids of the active block live on the device, each step is embed -> 28-layer cached
// forward -> fused lm_head + confidence -> unmask kernel (the unmask kernel writes the chosen
// tokens into the device block), and the host reads back only the step's window (status, tokens,
// unmask flags: ~70 bytes) to drive the loop.  The reference instead copies the fp32 logits'
// reductions back and decides in Python (runtime.py:176-181, 796-805).
#include <algorithm>
#include <cstring>

#include "handle.h"

using namespace fdllm;

namespace {

constexpr int kWin = 32;                  // max sub-block width read back per step
constexpr int kHostInts = 2 + 2 * kWin;   // pinned read-back: status[2], window tokens, unmask flags

// ---- device-side block loop (CUDA graph WHILE and IF/ELSE nodes) -----------------------------
// Loop state in device memory, read back once per block.
enum LoopSlot : int {
  kLKvValid = 0,    // the block's K/V rows hold a full step's values (partial steps allowed)
  kLPartial = 1,    // the current step is a partial one
  kLIter = 2,       // refinement steps in the current sub-block
  kLUnmask = 3,     // statistics: positions unmasked, refinement forwards, partial forwards
  kLRecompute = 4,
  kLPartialCnt = 5,
  kLToken = 6,      // the block-append forward's next token
  kLSlots = 8,
};
constexpr int kLoopLimit = 64;  // refinement steps per sub-block before the loop gives up (>= width)

// Before a sub-block's WHILE node: loop while the window still holds masks.
__global__ void loop_init_kernel(const int* block, int s0, int len, int mask_id, int* st,
                                 cudaGraphConditionalHandle hw) {
  int any = 0;
  for (int j = 0; j < len; ++j) any |= block[s0 + j] == mask_id;
  st[kLIter] = 0;
  cudaGraphSetConditional(hw, any ? 1u : 0u);
}

// Body head: the step is partial when the block cache is on, a full step of this block has run
// and the window's first position is decided (runtime.py:760-764).
__global__ void loop_choose_kernel(const int* block, int s0, int mask_id, int use_block_cache, int* st,
                                   cudaGraphConditionalHandle hi) {
  const int partial = (use_block_cache && st[kLKvValid] && block[s0] != mask_id) ? 1 : 0;
  st[kLPartial] = partial;
  cudaGraphSetConditional(hi, static_cast<unsigned>(partial));
}

// Body tail: statistics, the block-cache state, and whether the window still holds masks.
__global__ void loop_end_kernel(const int* status, int use_block_cache, int* st, int* err,
                                cudaGraphConditionalHandle hw) {
  st[kLUnmask] += status[1];
  st[kLRecompute] += 1;
  if (st[kLPartial]) {
    st[kLPartialCnt] += 1;
  } else {
    st[kLKvValid] = use_block_cache;
  }
  const int it = ++st[kLIter];
  unsigned more = status[0] > 0 ? 1u : 0u;
  if (it >= kLoopLimit && more) {  // every step unmasks at least one position: never reached
    report_error(err, kErrLoopLimit);
    more = 0u;
  }
  cudaGraphSetConditional(hw, more);
}

__global__ void loop_reset_kernel(int* st) {
  for (int i = 0; i < kLSlots; ++i) st[i] = 0;
}

__global__ void loop_token_kernel(const int* cids, int row, int* st) { st[kLToken] = cids[row]; }

struct Driver {
  fdllm_handle* h;
  cudaStream_t s;  // the handle's own non-blocking decode stream (capturable)
  int bs, sbs, mask_id, stop;
  double thr;
  bool block_cache;
  int cap = 0;
  int prefix_len = 0;
  int32_t st[4] = {0, 0, 0, 0};  // unmask_updates, block_recomputes, partial_recomputes, block_appends

  int* host() { return h->dec.host; }

  int setup(int n0, int max_new) {
    const fdllm_config& c = h->cfg;
    const long long need = (static_cast<long long>(n0) + max_new + bs - 1) / bs * bs + bs;
    // Capacity rounded up to 512 rows so that repeated calls reuse the captured step graphs.
    cap = static_cast<int>((need + 511) / 512 * 512);
    if (need > c.max_positions) return fail(FDLLM_ERR_INVALID, "prompt + max_new_tokens exceeds max_positions");
    cap = std::min(cap, std::max(static_cast<int>(need), c.max_positions));
    const size_t cache_bytes = static_cast<size_t>(c.num_hidden_layers) * cap * c.num_key_value_heads * c.head_dim * h->esz;
    FDLLM_TRY(h->dec.k.ensure(cache_bytes));
    FDLLM_TRY(h->dec.v.ensure(cache_bytes));
    FDLLM_TRY(h->dec.ids.ensure(static_cast<size_t>(cap)));
    FDLLM_TRY(h->dec.block.ensure(static_cast<size_t>(bs)));
    FDLLM_TRY(h->dec.x.ensure(static_cast<size_t>(cap) * c.hidden_size * h->esz));
    FDLLM_TRY(h->dec.hid.ensure(static_cast<size_t>(bs) * c.hidden_size * h->esz));
    FDLLM_TRY(h->dec.cids.ensure(static_cast<size_t>(bs)));
    FDLLM_TRY(h->dec.cmax.ensure(static_cast<size_t>(bs)));
    FDLLM_TRY(h->dec.out.ensure(kHostInts));
    FDLLM_TRY(h->dec.plen.ensure(1));
    FDLLM_TRY(h->dec.loop.ensure(kLSlots));
    if (h->dec.host == nullptr) CUDA_TRY(cudaMallocHost(&h->dec.host, kHostInts * sizeof(int)));
    if (h->dec.host_params == nullptr) CUDA_TRY(cudaMallocHost(&h->dec.host_params, 16 * sizeof(int)));
    if (h->dec.stream == nullptr) CUDA_TRY(cudaStreamCreateWithFlags(&h->dec.stream, cudaStreamNonBlocking));
    s = h->dec.stream;
    if (h->dec.graph_cache_ptr != h->dec.k.p || h->dec.graph_cap != cap) {
      release_step_graphs(h);
      h->dec.graph_cache_ptr = h->dec.k.p;
      h->dec.graph_cap = cap;
    }
    return FDLLM_OK;
  }

  // build_prefix_cache_from_ids (runtime.py:266-323): rows [0, n) of a fresh cache.
  int prefill(const int* ids, int n) {
    prefix_len = 0;
    if (n == 0) return FDLLM_OK;
    CUDA_TRY(cudaMemcpyAsync(h->dec.ids.p, ids, n * sizeof(int), cudaMemcpyHostToDevice, s));
    CUDA_TRY(launch_embed(h->dec.ids.p, n, h->embed, h->cfg.vocab_size, h->cfg.hidden_size, h->dec.x.p, h->dtype,
                          h->err.p, s));
    FDLLM_TRY(dense_forward(h, h->dec.x.p, nullptr, n, h->dec.k.p, h->dec.v.p, cap, false, nullptr, s));
    prefix_len = n;
    return FDLLM_OK;
  }

  int upload_block(const int* ids) {
    CUDA_TRY(cudaMemcpyAsync(h->dec.block.p, ids, bs * sizeof(int), cudaMemcpyHostToDevice, s));
    return FDLLM_OK;
  }

  // The device work of one step: embed the block rows, the cached forward (write_rel = s0 for a
  // partial step; the prefix length is read from h->dec.plen), the fused lm_head + confidence, then
  // either the unmask of window [s0, s0+len) or (append) the last row's token; results are copied
  // to the pinned host buffer.  Recorded once per step shape into a CUDA graph.
  int record(int kind, int s0, int len, bool host_copy = true) {
    const bool partial = kind == 1;
    const int rows = partial ? len : bs;
    CUDA_TRY(launch_embed(h->dec.block.p + (partial ? s0 : 0), rows, h->embed, h->cfg.vocab_size, h->cfg.hidden_size,
                          h->dec.x.p, h->dtype, h->err.p, s));
    ReqDesc d{};
    d.k = h->dec.k.p;
    d.v = h->dec.v.p;
    d.layer_stride = layer_stride(h, cap);
    d.cap = cap;
    d.q_tok0 = 0;
    d.n_q = rows;
    d.plen_dev = h->dec.plen.p;
    d.write_rel = partial ? s0 : 0;
    d.attend_rel = bs;
    std::vector<ReqDesc> reqs{d};
    FDLLM_TRY(forward_core(h, h->dec.x.p, rows, reqs, nullptr, 0, 0, h->dec.hid.p, s, cap));
    FDLLM_TRY(confidence_locked(h, h->dec.hid.p, rows, h->dec.cids.p, h->dec.cmax.p, nullptr, nullptr, s));
    int* out = h->dec.out.p;
    if (kind == 2) {
      if (host_copy) {
        CUDA_TRY(cudaMemcpyAsync(host(), h->dec.cids.p + bs - 1, sizeof(int), cudaMemcpyDeviceToHost, s));
      } else {
        loop_token_kernel<<<1, 1, 0, s>>>(h->dec.cids.p, bs - 1, h->dec.loop.p);
        count_launch();
        CUDA_TRY(cudaGetLastError());
      }
    } else {
      CUDA_TRY(launch_unmask(h->dec.cids.p, h->dec.cmax.p, rows, h->dec.block.p, s0, len, partial ? 1 : 0, mask_id,
                             thr, out + 2, nullptr, out + 2 + kWin, out, s));
      if (host_copy) CUDA_TRY(cudaMemcpyAsync(host(), out, kHostInts * sizeof(int), cudaMemcpyDeviceToHost, s));
    }
    return FDLLM_OK;
  }

  // Append the work captured on stream `s` to `graph` after `deps`; *leaf receives the captured
  // work's last node.
  template <typename F>
  int capture_into(cudaGraph_t graph, const cudaGraphNode_t* deps, size_t ndeps, cudaGraphNode_t* leaf, F&& body) {
    CUDA_TRY(cudaStreamBeginCaptureToGraph(s, graph, deps, nullptr, ndeps, cudaStreamCaptureModeRelaxed));
    const int rc = body();
    cudaStreamCaptureStatus cs;
    const cudaGraphNode_t* leaves = nullptr;
    size_t nleaves = 0;
    cudaGraph_t g2 = nullptr;
    const cudaError_t ei = cudaStreamGetCaptureInfo(s, &cs, nullptr, &g2, &leaves, &nleaves);
    *leaf = (ei == cudaSuccess && nleaves > 0) ? leaves[nleaves - 1] : nullptr;
    cudaGraph_t out = nullptr;
    const cudaError_t ee = cudaStreamEndCapture(s, &out);
    if (rc != FDLLM_OK) return rc;
    if (ei != cudaSuccess) return fail(FDLLM_ERR_CUDA, std::string("cudaStreamGetCaptureInfo: ") + cudaGetErrorString(ei));
    if (ee != cudaSuccess) return fail(FDLLM_ERR_CUDA, std::string("capture into graph: ") + cudaGetErrorString(ee));
    if (nleaves != 1) return fail(FDLLM_ERR_CUDA, "captured block work does not end in a single node");
    return FDLLM_OK;
  }

  // Build the graph of one whole block: for each sub-block, WHILE (masks in its window)
  // { IF (partial) partial step ELSE full step }, then the block-append forward; the block's
  // tokens and the loop state are copied to the host at the end.
  int build_block_graph(BlockGraph* bg) {
    FDLLM_TRY(reserve_workspace(h, bs, 1, cap));
    const unsigned long long gen = g_ws_generation.load();
    cudaGraph_t g = nullptr;
    CUDA_TRY(cudaGraphCreate(&g, 0));
    struct GraphGuard {
      cudaGraph_t g;
      ~GraphGuard() { if (g) cudaGraphDestroy(g); }
    } guard{g};
    const long long launches_before = launch_count();
    int* st = h->dec.loop.p;
    int* out = h->dec.out.p;
    int n_full = 0, n_partial = 0;
    cudaGraphNode_t prev = nullptr;
    FDLLM_TRY(capture_into(g, nullptr, 0, &prev, [&]() -> int {
      loop_reset_kernel<<<1, 1, 0, s>>>(st);
      count_launch();
      CUDA_TRY(cudaGetLastError());
      return FDLLM_OK;
    }));
    for (int s0 = 0; s0 < bs; s0 += sbs) {
      const int len = std::min(bs, s0 + sbs) - s0;
      cudaGraphConditionalHandle hw;
      CUDA_TRY(cudaGraphConditionalHandleCreate(&hw, g, 0, 0));
      cudaGraphNode_t init = nullptr;
      FDLLM_TRY(capture_into(g, &prev, 1, &init, [&]() -> int {
        loop_init_kernel<<<1, 1, 0, s>>>(h->dec.block.p, s0, len, mask_id, st, hw);
        count_launch();
        CUDA_TRY(cudaGetLastError());
        return FDLLM_OK;
      }));
      cudaGraphNodeParams wp{};
      wp.type = cudaGraphNodeTypeConditional;
      wp.conditional.handle = hw;
      wp.conditional.type = cudaGraphCondTypeWhile;
      wp.conditional.size = 1;
      cudaGraphNode_t wnode = nullptr;
      CUDA_TRY(cudaGraphAddNode(&wnode, g, &init, 1, &wp));
      cudaGraph_t body = wp.conditional.phGraph_out[0];
      // body: choose -> IF (partial) / ELSE (full) -> end
      cudaGraphConditionalHandle hi;
      CUDA_TRY(cudaGraphConditionalHandleCreate(&hi, body, 0, 0));
      cudaGraphNode_t choose = nullptr;
      FDLLM_TRY(capture_into(body, nullptr, 0, &choose, [&]() -> int {
        loop_choose_kernel<<<1, 1, 0, s>>>(h->dec.block.p, s0, mask_id, block_cache ? 1 : 0, st, hi);
        count_launch();
        CUDA_TRY(cudaGetLastError());
        return FDLLM_OK;
      }));
      cudaGraphNodeParams ip{};
      ip.type = cudaGraphNodeTypeConditional;
      ip.conditional.handle = hi;
      ip.conditional.type = cudaGraphCondTypeIf;
      ip.conditional.size = 2;  // body 0: condition true (partial), body 1: else (full)
      cudaGraphNode_t inode = nullptr;
      CUDA_TRY(cudaGraphAddNode(&inode, body, &choose, 1, &ip));
      cudaGraphNode_t leaf = nullptr;
      long long c0 = launch_count();
      FDLLM_TRY(capture_into(ip.conditional.phGraph_out[0], nullptr, 0, &leaf, [&]() { return record(1, s0, len, false); }));
      n_partial = static_cast<int>(launch_count() - c0);
      c0 = launch_count();
      FDLLM_TRY(capture_into(ip.conditional.phGraph_out[1], nullptr, 0, &leaf, [&]() { return record(0, s0, len, false); }));
      n_full = static_cast<int>(launch_count() - c0);
      cudaGraphNode_t endn = nullptr;
      FDLLM_TRY(capture_into(body, &inode, 1, &endn, [&]() -> int {
        loop_end_kernel<<<1, 1, 0, s>>>(out, block_cache ? 1 : 0, st, h->err.p, hw);
        count_launch();
        CUDA_TRY(cudaGetLastError());
        return FDLLM_OK;
      }));
      prev = wnode;
    }
    cudaGraphNode_t last = nullptr;
    const long long c_app = launch_count();
    FDLLM_TRY(capture_into(g, &prev, 1, &last, [&]() -> int {
      FDLLM_TRY(record(2, 0, bs, false));
      CUDA_TRY(cudaMemcpyAsync(host(), h->dec.block.p, bs * sizeof(int), cudaMemcpyDeviceToHost, s));
      CUDA_TRY(cudaMemcpyAsync(host() + kWin, st, kLSlots * sizeof(int), cudaMemcpyDeviceToHost, s));
      return FDLLM_OK;
    }));
    const int n_append = static_cast<int>(launch_count() - c_app);
    // recorded launches did not run; the block's launches are counted when it replays
    count_launch(-static_cast<int>(launch_count() - launches_before));
    if (g_ws_generation.load() != gen) return fail(FDLLM_ERR_CUDA, "workspace reallocated while building the block graph");
    if (bg->exec) cudaGraphExecDestroy(bg->exec);
    bg->exec = nullptr;
    CUDA_TRY(cudaGraphInstantiate(&bg->exec, g, 0));
    bg->gen = gen;
    bg->mask_id = mask_id;
    bg->thr = thr;
    bg->use_block_cache = block_cache ? 1 : 0;
    bg->sbs = sbs;
    bg->n_full = n_full;
    bg->n_partial = n_partial;
    bg->n_append = n_append;
    return FDLLM_OK;
  }

  // Run one whole block on the device; x_block receives its tokens, *tok the appended token.
  int run_block(int* x_block, int* tok) {
    BlockGraph& bg = h->dec.block_graph;
    const bool stale = bg.exec == nullptr || bg.gen != g_ws_generation.load() || bg.mask_id != mask_id ||
                       bg.thr != thr || bg.use_block_cache != (block_cache ? 1 : 0) || bg.sbs != sbs;
    if (stale) FDLLM_TRY(build_block_graph(&bg));
    h->dec.host_params[0] = prefix_len;
    CUDA_TRY(cudaMemcpyAsync(h->dec.plen.p, h->dec.host_params, sizeof(int), cudaMemcpyHostToDevice, s));
    CUDA_TRY(cudaGraphLaunch(bg.exec, s));
    CUDA_TRY(cudaStreamSynchronize(s));
    const int* hb = host();
    std::memcpy(x_block, hb, bs * sizeof(int));
    const int* ls = hb + kWin;
    const int full_steps = ls[kLRecompute] - ls[kLPartialCnt];
    count_launch(1 + (bs + sbs - 1) / sbs + 2 * ls[kLRecompute] + full_steps * bg.n_full +
                 ls[kLPartialCnt] * bg.n_partial + bg.n_append);  // kernels this replay ran
    st[0] += ls[kLUnmask];
    st[1] += ls[kLRecompute] + 1;  // + the block-append forward
    st[2] += ls[kLPartialCnt];
    st[3] += 1;
    *tok = ls[kLToken];
    return FDLLM_OK;
  }

  // Replay (capturing on first use) the graph of one step shape, then wait for its results.
  int run_step(int kind, int s0, int len) {
    h->dec.host_params[0] = prefix_len;
    CUDA_TRY(cudaMemcpyAsync(h->dec.plen.p, h->dec.host_params, sizeof(int), cudaMemcpyHostToDevice, s));
    const long long key = ((static_cast<long long>(kind) * 64 + s0) * 64 + len) * 2 + (h->prof ? 1 : 0);
    StepGraph* g = nullptr;
    for (auto& kv : h->dec.graphs)
      if (kv.first == key) g = &kv.second;
    if (g != nullptr && g->gen != g_ws_generation.load()) {  // a workspace buffer moved since capture
      release_step_graphs(h);
      g = nullptr;
    }
    if (g != nullptr && (g->mask_id != mask_id || g->thr != thr)) {  // other unmask parameters
      release_step_graphs(h);
      g = nullptr;
    }
    if (g == nullptr) {
      FDLLM_TRY(reserve_workspace(h, bs, 1, cap));  // nothing may allocate while capturing
      const unsigned long long gen = g_ws_generation.load();
      h->cap_prof.clear();
      h->capturing = true;
      const long long launches_before = launch_count();
      CUDA_TRY(cudaStreamBeginCapture(s, cudaStreamCaptureModeRelaxed));
      const int rc = record(kind, s0, len);
      cudaGraph_t graph = nullptr;
      const cudaError_t ec = cudaStreamEndCapture(s, &graph);
      h->capturing = false;
      if (rc != FDLLM_OK || ec != cudaSuccess) {
        if (graph) cudaGraphDestroy(graph);
        for (auto& pp : h->cap_prof) {
          cudaEventDestroy(pp.e0);
          cudaEventDestroy(pp.e1);
        }
        h->cap_prof.clear();
        return rc != FDLLM_OK ? rc : fail(FDLLM_ERR_CUDA, std::string("stream capture: ") + cudaGetErrorString(ec));
      }
      if (g_ws_generation.load() != gen) {  // something allocated while recording: refuse the graph
        cudaGraphDestroy(graph);
        return fail(FDLLM_ERR_CUDA, "workspace reallocated during stream capture");
      }
      StepGraph sg;
      sg.gen = gen;
      sg.mask_id = mask_id;
      sg.thr = thr;
      // recorded launches did not run; they are counted when the graph replays
      sg.n_kernels = static_cast<int>(launch_count() - launches_before);
      count_launch(-sg.n_kernels);
      const cudaError_t ei = cudaGraphInstantiate(&sg.exec, graph, 0);
      cudaGraphDestroy(graph);
      sg.prof.swap(h->cap_prof);
      if (ei != cudaSuccess) return fail(FDLLM_ERR_CUDA, std::string("cudaGraphInstantiate: ") + cudaGetErrorString(ei));
      h->dec.graphs.emplace_back(key, std::move(sg));
      g = &h->dec.graphs.back().second;
    }
    CUDA_TRY(cudaGraphLaunch(g->exec, s));
    count_launch(g->n_kernels);
    CUDA_TRY(cudaStreamSynchronize(s));
    if (h->prof) {
      for (const ProfPair& pp : g->prof) {
        float t = 0.f;
        CUDA_TRY(cudaEventElapsedTime(&t, pp.e0, pp.e1));
        h->prof_ms_extra += t;
        h->prof_bytes += pp.bytes;
        h->prof_flops += pp.flops;
        h->prof_launch_extra += 1;
      }
    }
    return FDLLM_OK;
  }

  // One refinement step; copies the unmasked tokens of the window into the host sequence.
  int refine(bool partial, int s0, int len, int* x_window) {
    FDLLM_TRY(run_step(partial ? 1 : 0, s0, len));
    const int* hb = host();
    for (int j = 0; j < len; ++j)
      if (hb[2 + kWin + j]) x_window[j] = hb[2 + j];
    st[0] += hb[1];
    return FDLLM_OK;
  }

  // Block-append: the committing forward; returns the last row's unshifted argmax (runtime.py:181).
  int append(int* tok) {
    FDLLM_TRY(run_step(2, 0, bs));
    *tok = host()[0];
    return FDLLM_OK;
  }
};

bool has_completed_stop(const std::vector<int>& seq, size_t plen, int stop, int mask_id) {
  if (stop < 0) return false;
  for (size_t i = plen; i < seq.size(); ++i) {
    if (seq[i] == stop) {
      for (size_t j = plen; j < i; ++j)
        if (seq[j] == mask_id) return false;
      return true;
    }
  }
  return false;
}

}  // namespace

extern "C" int fdllm_generate(fdllm_handle* h, const int32_t* prompt, int prompt_len, int max_new_tokens,
                              int block_size, int small_block_size, double threshold, int use_block_cache, int mask_id,
                              int stop_token, int32_t* out_tokens, int* n_out, int32_t* stats, float* timing_ms,
                              void* stream) {
  FDLLM_TRY(check_handle(h));
  if (prompt == nullptr || out_tokens == nullptr || n_out == nullptr) return fail(FDLLM_ERR_INVALID, "null argument");
  if (max_new_tokens < 0) return fail(FDLLM_ERR_INVALID, "max_new_tokens must be non-negative.");
  if (block_size != h->cfg.bd_size) return fail(FDLLM_ERR_INVALID, "block_size must equal the model's bd_size");
  if (small_block_size <= 0 || small_block_size > kWin || block_size % small_block_size != 0)
    return fail(FDLLM_ERR_INVALID, "small_block_size must divide block_size and be at most 32");
  if (prompt_len < block_size)
    return fail(FDLLM_ERR_UNSUPPORTED, "prompts shorter than one block take the stateless path (forward_hidden); "
                                       "use the Python runtime for them");
  std::lock_guard<std::mutex> lock(h->mu);
  CUDA_TRY(cudaStreamSynchronize(static_cast<cudaStream_t>(stream)));  // the caller's prior work is done
  Driver d{h, nullptr, block_size, small_block_size, mask_id, stop_token, threshold, use_block_cache != 0};
  // device-side block loops: without a stop token (checked on the host between steps) and without
  // per-launch profiling events; tuning block_graph=0 turns them off
  const bool use_block_graph = stop_token < 0 && !h->prof && h->tune.block_graph != 0;
  const int bs = block_size, sbs = small_block_size;
  std::vector<int> gen(prompt, prompt + prompt_len);
  const size_t n0 = gen.size();
  FDLLM_TRY(d.setup(prompt_len, max_new_tokens));
  bool kv_valid = false;
  cudaEvent_t ev[3] = {nullptr, nullptr, nullptr};
  bool prefill_marked = false;
  if (timing_ms) {
    for (auto& e : ev) CUDA_TRY(cudaEventCreate(&e));
    CUDA_TRY(cudaEventRecord(ev[0], d.s));
  }
  auto mark_prefill = [&]() -> int {
    if (timing_ms && !prefill_marked) CUDA_TRY(cudaEventRecord(ev[1], d.s));
    prefill_marked = true;
    return FDLLM_OK;
  };

  auto finish = [&](const std::vector<int>& toks) -> int {
    size_t end = std::min(toks.size(), n0 + static_cast<size_t>(max_new_tokens));
    int n = 0;
    for (size_t i = n0; i < end; ++i) {
      if (toks[i] == mask_id) break;
      out_tokens[n++] = toks[i];
    }
    *n_out = n;
    if (stats) std::memcpy(stats, d.st, sizeof(d.st));
    if (timing_ms) {
      FDLLM_TRY(mark_prefill());
      CUDA_TRY(cudaEventRecord(ev[2], d.s));
      CUDA_TRY(cudaEventSynchronize(ev[2]));
      CUDA_TRY(cudaEventElapsedTime(&timing_ms[0], ev[0], ev[1]));
      CUDA_TRY(cudaEventElapsedTime(&timing_ms[1], ev[0], ev[2]));
      for (auto& e : ev) cudaEventDestroy(e);
    }
    return FDLLM_OK;
  };

  if (n0 % bs == 0 && max_new_tokens > 0) {
    const int lb = static_cast<int>(n0) - bs;
    FDLLM_TRY(d.prefill(gen.data(), lb));
    FDLLM_TRY(d.upload_block(gen.data() + lb));
    int nxt = 0;
    FDLLM_TRY(d.append(&nxt));
    d.prefix_len += bs;  // commit
    d.st[1] += 1;
    d.st[3] += 1;
    gen.push_back(nxt);
    if (stop_token >= 0 && nxt == stop_token) return finish(gen);
  }

  while (gen.size() - n0 < static_cast<size_t>(max_new_tokens)) {
    const size_t plen = gen.size();
    std::vector<int> x(gen);
    x.resize(plen + (bs - plen % bs), mask_id);
    const int a0 = static_cast<int>(x.size()) - bs;
    if (a0 != d.prefix_len) {
      FDLLM_TRY(d.prefill(x.data(), a0));
      kv_valid = false;
    }
    FDLLM_TRY(mark_prefill());  // the reference's prefill boundary (runtime.py:741-746)
    FDLLM_TRY(d.upload_block(x.data() + a0));
    // A block that ends before max_new_tokens, with no stop token to watch, runs as one device-side
    // graph: the refinement loops of all its sub-blocks and the block-append, one host sync.
    if (use_block_graph && x.size() - n0 < static_cast<size_t>(max_new_tokens)) {
      int nxt = 0;
      FDLLM_TRY(d.run_block(x.data() + a0, &nxt));
      gen = x;
      d.prefix_len += bs;
      kv_valid = false;
      gen.push_back(nxt);
      continue;
    }
    bool length_done = false;
    for (int s0 = 0; s0 < bs && !length_done; s0 += sbs) {
      const int s1 = std::min(bs, s0 + sbs);
      while (true) {
        bool any_mask = false;
        for (int j = s0; j < s1; ++j) any_mask |= (x[a0 + j] == mask_id);
        if (!any_mask) break;
        if (has_completed_stop(x, plen, stop_token, mask_id)) return finish(x);
        const bool partial = d.block_cache && kv_valid && x[a0 + s0] != mask_id;
        FDLLM_TRY(d.refine(partial, s0, s1 - s0, x.data() + a0 + s0));
        if (partial) {
          d.st[2] += 1;
        } else {
          kv_valid = d.block_cache;
        }
        d.st[1] += 1;
        if (x.size() - n0 >= static_cast<size_t>(max_new_tokens)) {
          length_done = true;
          break;
        }
      }
      if (x.size() - n0 >= static_cast<size_t>(max_new_tokens)) length_done = true;
    }
    gen = x;
    if (gen.size() - n0 >= static_cast<size_t>(max_new_tokens)) break;
    if (has_completed_stop(gen, n0, stop_token, mask_id)) break;
    // block-append: the completed block is already on the device (the unmask kernel kept it)
    int nxt = 0;
    FDLLM_TRY(d.append(&nxt));
    d.prefix_len += bs;
    kv_valid = false;
    d.st[1] += 1;
    gen.push_back(nxt);
    d.st[3] += 1;
    if (stop_token >= 0 && nxt == stop_token) break;
  }
  return finish(gen);
}

void fdllm::release_step_graphs(fdllm_handle* h) {
  if (h->dec.block_graph.exec) cudaGraphExecDestroy(h->dec.block_graph.exec);
  h->dec.block_graph = BlockGraph{};
  for (auto& kv : h->dec.graphs) {
    if (kv.second.exec) cudaGraphExecDestroy(kv.second.exec);
    for (auto& pp : kv.second.prof) {
      cudaEventDestroy(pp.e0);
      cudaEventDestroy(pp.e1);
    }
  }
  h->dec.graphs.clear();
}
