// Persistent layer-stack kernel: the whole cached forward of a decode step in one launch.
//
// A decode step of the 1.5B model is 28 x (qkv, attention, o, gate_up, down) over <= 32 token rows
// plus the final norm (fast_dllm_relax/model/cuda.py:545-579, 639-666; the cached attention of
// runtime.py:63-73).  Run as separate kernels, every layer pays six kernel-boundary latencies
// (drain, flush, launch, pipeline fill) that dwarf its 94 MB of weight streaming.  Here one CTA
// per SM stays resident for all layers (cooperative launch: every CTA is co-resident, so the grid
// barriers below cannot deadlock), and each CTA runs three roles:
//
//   warp 0, lane 0  TMA producer: streams this CTA's weight tiles (128 rows x 64 k, 16 KB) for every
//                   projection of every layer, in order, through a 6-stage ring.  Weights depend on
//                   nothing, so the ring fills with the next projection's tiles while the current
//                   phase's epilogue, the attention and the grid barriers run.
//   warp 1, lane 0  MMA issuer: tcgen05.mma kind::f16, M = 128 weight rows x N = 32 token rows, fp32
//                   accumulator in TMEM; frees ring slots with tcgen05.commit.
//   warps 2-7       compute: stage the B operand (activations, TMA + fused RMSNorm in shared memory),
//                   drain TMEM, split-K reduction, the fused epilogues (epilogue.cuh), attention
//                   (mma.sync flash attention, key splits), grid barriers.
//
// Work split per phase (each CTA owns at most one unit of each projection):
//   qkv / o / down: slab x k-split units; every unit writes its fp32 partial tile to global memory,
//     and the CTA that arrives last for a slab sums the partials in split order (deterministic)
//     and runs the epilogue (bias + RoPE + KV append / residual + row sums of squares).
//   gate_up: one paired slab (64 gate + 64 up rows) per CTA, full K, SiLU(gate)*up epilogue.
//   attention: (request, 16-token q tile, kv head, key split) units; the last split of a group to
//     finish merges the partials by log-sum-exp.
// Phases are separated by grid barriers.  Cross-CTA data is read with L2-only loads (ld.global.cg,
// cp.async.cg) or TMA, never through L1.
//
// Every wait is bounded (kWaitLimitNs) and also gives up as soon as another CTA has raised the
// launch's abort flag; on expiry the CTA records an error code, raises the flag, drains its own
// TMA copies (bounded), frees its TMEM and returns.
#include <algorithm>

#include "common.cuh"
#include "epilogue.cuh"
#include "kernels.h"

namespace fdllm {

namespace {

constexpr int kThreads = 256;
constexpr int kCompute = 192;           // warps 2-7
constexpr int kComputeBar = 1;          // named barrier id of the compute warps
constexpr int kAStage = 128 * 64 * 2;   // weight tile
constexpr int kBChunk = kStackRows * 64 * 2;  // one 64-wide k block of the B operand (4 KB)
constexpr int kRingBytes = kStackStages * kAStage;
constexpr int kBarOff = kRingBytes + kStackBBytes;
constexpr int kSmemBytes = 1024 + kBarOff + 2048;  // alignment slack + tiles + barriers / row scales
constexpr int kTmemCols = 32;
constexpr int kBGroups = 4;  // the B operand lands and is released to the MMA in up to 4 groups
constexpr int kQT = 16;
constexpr int kKT = 64;
constexpr float kLog2e = 1.4426950408889634f;
// arrival counter bases inside a layer's block of kStackCtrPerLayer
constexpr int kCtrQkv = 0, kCtrAttn = 64, kCtrO = 128, kCtrDown = 192;

static_assert(kSmemBytes <= 227 * 1024, "shared memory budget");

__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

__device__ __forceinline__ bool aborted(const unsigned* sync) {
  return *reinterpret_cast<const volatile unsigned*>(sync + 1) != 0u;
}

__device__ __forceinline__ void raise_abort(const StackArgs& a, int code) {
  report_error(a.err, code);
  atomicExch(a.sync + 1, 1u);
}

// mbarrier wait bounded in time and by the launch's abort flag.
__device__ __forceinline__ bool wait_bar(const StackArgs& a, uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 8; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (aborted(a.sync) || global_timer_ns() - t0 > kWaitLimitNs) return false;
    __nanosleep(64);  // leave the issue slots to the compute warps
  }
}

// Grid barrier over the compute warps of all CTAs (the producer and MMA warps never join).
// Writes before it by any compute thread are visible to every compute thread after it, to
// generic loads and (fence.proxy.async) to TMA reads.
__device__ bool grid_barrier(const StackArgs& a, unsigned& epoch, int tid, volatile int* s_flag) {
  fence_proxy_async_smem();  // this phase's generic shared-memory accesses before the next TMA writes
  named_sync(kComputeBar, kCompute);
  ++epoch;
  if (tid == 0) {
    int ok = 1;
    fence_proxy_async_global();
    __threadfence();
    atomicAdd(a.sync, 1u);
    const unsigned target = epoch * gridDim.x;
    if (ld_acquire(a.sync) < target) {
      const uint64_t t0 = global_timer_ns();
      while (ld_acquire(a.sync) < target) {
        if (aborted(a.sync) || global_timer_ns() - t0 > kWaitLimitNs) {
          ok = 0;
          break;
        }
        __nanosleep(20);
      }
    }
    __threadfence();
    fence_proxy_async_global();
    if (!ok) raise_abort(a, kErrTimeoutBarrier);
    *s_flag = ok;
  }
  named_sync(kComputeBar, kCompute);
  const int ok = *s_flag;
  named_sync(kComputeBar, kCompute);  // s_flag is reused by the next barrier
  return ok != 0;
}

// Arrive on `ctr`, then wait until all `count` participants have arrived.  The participants of
// one counter are distinct CTAs working in the same phase (one unit per CTA per phase), so they
// all run concurrently.  Their global writes before arriving are visible afterwards.
__device__ bool arrive_and_wait(const StackArgs& a, unsigned* ctr, unsigned count, int tid, volatile int* s_flag) {
  named_sync(kComputeBar, kCompute);
  if (tid == 0) {
    int ok = 1;
    __threadfence();
    atomicAdd(ctr, 1u);
    if (ld_acquire(ctr) < count) {
      const uint64_t t0 = global_timer_ns();
      while (ld_acquire(ctr) < count) {
        if (aborted(a.sync) || global_timer_ns() - t0 > kWaitLimitNs) {
          ok = 0;
          break;
        }
        __nanosleep(20);
      }
    }
    __threadfence();
    if (!ok) raise_abort(a, kErrTimeoutBarrier);
    *s_flag = ok;
  }
  named_sync(kComputeBar, kCompute);
  const int ok = *s_flag;
  named_sync(kComputeBar, kCompute);
  return ok != 0;
}

struct Unit {
  int valid, slab, split, splits, kb0, kb1;
};

// The unit of projection `proj` (0 qkv, 1 o, 2 gate_up, 3 down) owned by CTA `cta`.
__device__ __forceinline__ Unit gemm_unit(const StackArgs& a, int proj, int cta) {
  int slabs, splits, kbt;
  switch (proj) {
    case 0: slabs = (a.hq + 2 * a.hkv) * a.hd / 128; splits = a.qkv_splits; kbt = a.H / 64; break;
    case 1: slabs = a.H / 128; splits = a.o_splits; kbt = a.hq * a.hd / 64; break;
    case 2: slabs = a.I / 64; splits = 1; kbt = a.H / 64; break;
    default: slabs = a.H / 128; splits = a.down_splits; kbt = a.I / 64; break;
  }
  Unit u{0, 0, 0, splits, 0, 0};
  if (cta < slabs * splits) {
    u.valid = 1;
    u.slab = cta / splits;
    u.split = cta % splits;
    u.kb0 = u.split * kbt / splits;
    u.kb1 = (u.split + 1) * kbt / splits;
  }
  return u;
}

// Byte offset of 16-byte chunk `cc` of row `t` inside one 128-byte-swizzled k block.
__device__ __forceinline__ int sw128_off(int t, int cc) { return (t >> 3) * 1024 + (t & 7) * 128 + ((cc ^ (t & 7)) << 4); }

// ---- attention (one unit: request, 16-token q tile, kv head, key split) ---------------------
__device__ __forceinline__ void mma_16816(float (&c)[4], const uint32_t (&x)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(x[0]), "r"(x[1]), "r"(x[2]), "r"(x[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

template <int HD>
__device__ __forceinline__ uint32_t tile_off(int key, int c) {
  return static_cast<uint32_t>(key * (HD * 2) + ((c ^ (key & 7)) << 4));
}

struct Group {
  int req, qtile, kvh;
};

__device__ __forceinline__ Group attn_group(const StackArgs& a, int g) {
  Group r{0, 0, 0};
  for (int i = 0; i < a.n_reqs; ++i) {
    const int nqt = (a.reqs[i].n_q + kQT - 1) / kQT;
    if (g < nqt * a.hkv) {
      r.req = i;
      r.qtile = g / a.hkv;
      r.kvh = g % a.hkv;
      return r;
    }
    g -= nqt * a.hkv;
  }
  return r;
}

// Partial attention of one unit: normalised O rows (fp32) and their log-sum-exp, to apart / alse.
// Cached semantics: no mask, keys [0, attend_len) split evenly over attn_splits.
template <int HD>
__device__ void attn_unit(const StackArgs& a, int layer, int group, int split, uint8_t* smem, int tid,
                          unsigned long long* t_kv) {
  constexpr int kChunks = HD / 8;
  constexpr int kTileBytes = kKT * HD * 2;
  uint8_t* Ks = smem;
  uint8_t* Vs = smem + 2 * kTileBytes;
  const int G = a.hq / a.hkv;
  const int rows = kQT * G;
  const int warp = tid >> 5, lane = tid & 31;
  const int g8 = lane >> 2, t4 = lane & 3;
  const Group gr = attn_group(a, group);
  const ReqDesc r = a.reqs[gr.req];
  const int tq0 = gr.qtile * kQT;
  const int L = r.attend_len;
  const int S = a.attn_splits;
  const int split_len = max(kKT, ((L + S - 1) / S + kKT - 1) / kKT * kKT);
  const int key0 = split * split_len;
  const int key1 = min(L, key0 + split_len);
  const bool active = warp < G;
  const size_t kv_row = static_cast<size_t>(a.hkv) * HD;
  const bf16* kg = static_cast<const bf16*>(r.k) + static_cast<size_t>(layer) * r.layer_stride + gr.kvh * HD;
  const bf16* vg = static_cast<const bf16*>(r.v) + static_cast<size_t>(layer) * r.layer_stride + gr.kvh * HD;
  const bf16* qg = static_cast<const bf16*>(a.q);

  int tok_row[2], qh_row[2];
  bool valid_row[2];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int rr = warp * 16 + g8 + h * 8;
    const int tq = tq0 + rr / G;
    valid_row[h] = active && (tq < r.n_q);
    tok_row[h] = r.q_tok0 + (valid_row[h] ? tq : 0);
    qh_row[h] = gr.kvh * G + rr % G;
  }
  uint32_t qf[HD / 16][4];
#pragma unroll
  for (int kk = 0; kk < HD / 16; ++kk) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const bf16* qp = qg + static_cast<size_t>(tok_row[h]) * (a.hq * HD) + qh_row[h] * HD + kk * 16 + 2 * t4;
      qf[kk][h] = valid_row[h] ? __ldcg(reinterpret_cast<const unsigned int*>(qp)) : 0u;
      qf[kk][h + 2] = valid_row[h] ? __ldcg(reinterpret_cast<const unsigned int*>(qp + 8)) : 0u;
    }
  }
  float o[HD / 8][4];
#pragma unroll
  for (int n = 0; n < HD / 8; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
  float m_run[2] = {-INFINITY, -INFINITY};
  float l_run[2] = {0.f, 0.f};

  const int n_tiles = (key1 > key0) ? (key1 - key0 + kKT - 1) / kKT : 0;
  auto load_tile = [&](int it, int buf) {
    const int kt0 = key0 + it * kKT;
    for (int idx = tid; idx < kKT * kChunks; idx += kCompute) {
      const int key = idx / kChunks, c = idx % kChunks;
      const bool ok = kt0 + key < key1;
      const size_t src = static_cast<size_t>(ok ? kt0 + key : 0) * kv_row + c * 8;
      cp_async_16(Ks + buf * kTileBytes + tile_off<HD>(key, c), kg + src, ok);
      cp_async_16(Vs + buf * kTileBytes + tile_off<HD>(key, c), vg + src, ok);
    }
    cp_async_commit();
  };
  if (n_tiles > 0) load_tile(0, 0);
  for (int it = 0; it < n_tiles; ++it) {
    const int buf = it & 1;
    if (it + 1 < n_tiles) {
      load_tile(it + 1, buf ^ 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    named_sync(kComputeBar, kCompute);
    if (it == 0 && t_kv != nullptr && tid == 0) *t_kv = global_timer_ns();
    if (active) {
      const uint32_t kb = smem_addr(Ks + buf * kTileBytes);
      const uint32_t vb = smem_addr(Vs + buf * kTileBytes);
      const int kt0 = key0 + it * kKT;
      float s[8][4];
#pragma unroll
      for (int j = 0; j < 8; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
#pragma unroll
      for (int kk = 0; kk < HD / 16; ++kk) {
#pragma unroll
        for (int jp = 0; jp < 4; ++jp) {
          const int m = lane >> 3, i = lane & 7;
          const int key = (2 * jp + (m >> 1)) * 8 + i;
          uint32_t b[4];
          ldsm_x4(b, kb + tile_off<HD>(key, kk * 2 + (m & 1)));
          mma_16816(s[2 * jp], qf[kk], b[0], b[1]);
          mma_16816(s[2 * jp + 1], qf[kk], b[2], b[3]);
        }
      }
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        float mx = -INFINITY;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int key = kt0 + j * 8 + 2 * t4 + e;
            float v = s[j][2 * h + e] * a.scale;
            if (key >= key1) v = -INFINITY;
            s[j][2 * h + e] = v;
            mx = fmaxf(mx, v);
          }
        }
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
        const float m_new = fmaxf(m_run[h], mx);
        const float m_use = (m_new == -INFINITY) ? 0.f : m_new;
        const float alpha = exp2f((m_run[h] - m_use) * kLog2e);
        float psum = 0.f;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const float p = exp2f((s[j][2 * h + e] - m_use) * kLog2e);
            s[j][2 * h + e] = p;
            psum += p;
          }
        }
        l_run[h] = l_run[h] * alpha + psum;
        m_run[h] = m_new;
#pragma unroll
        for (int n = 0; n < HD / 8; ++n) {
          o[n][2 * h] *= alpha;
          o[n][2 * h + 1] *= alpha;
        }
      }
#pragma unroll
      for (int kc = 0; kc < 4; ++kc) {
        uint32_t pa[4];
        pa[0] = pack_bf16(s[2 * kc][0], s[2 * kc][1]);
        pa[1] = pack_bf16(s[2 * kc][2], s[2 * kc][3]);
        pa[2] = pack_bf16(s[2 * kc + 1][0], s[2 * kc + 1][1]);
        pa[3] = pack_bf16(s[2 * kc + 1][2], s[2 * kc + 1][3]);
#pragma unroll
        for (int np = 0; np < HD / 16; ++np) {
          const int m = lane >> 3, i = lane & 7;
          const int key = kc * 16 + (m & 1) * 8 + i;
          uint32_t b[4];
          ldsm_x4_t(b, vb + tile_off<HD>(key, 2 * np + (m >> 1)));
          mma_16816(o[2 * np], pa, b[0], b[1]);
          mma_16816(o[2 * np + 1], pa, b[2], b[3]);
        }
      }
    }
    named_sync(kComputeBar, kCompute);
  }
  if (!active) return;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    l_run[h] += __shfl_xor_sync(0xffffffffu, l_run[h], 1);
    l_run[h] += __shfl_xor_sync(0xffffffffu, l_run[h], 2);
  }
  if (S == 1) {  // the whole key range in this unit: normalised bf16 output directly
    bf16* out = static_cast<bf16*>(a.attn);
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      if (!valid_row[h]) continue;
      const float inv = l_run[h] > 0.f ? 1.f / l_run[h] : 0.f;
      bf16* orow = out + static_cast<size_t>(tok_row[h]) * (a.hq * HD) + qh_row[h] * HD;
#pragma unroll
      for (int n = 0; n < HD / 8; ++n)
        *reinterpret_cast<__nv_bfloat162*>(orow + n * 8 + 2 * t4) =
            __floats2bfloat162_rn(o[n][2 * h] * inv, o[n][2 * h + 1] * inv);
    }
    return;
  }
  const int unit = group * S + split;
  float* op = a.apart + static_cast<size_t>(unit) * rows * HD;
  float* lp = a.alse + static_cast<size_t>(unit) * rows;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int rr = warp * 16 + g8 + h * 8;
    const float inv = l_run[h] > 0.f ? 1.f / l_run[h] : 0.f;
#pragma unroll
    for (int n = 0; n < HD / 8; ++n)
      __stcg(reinterpret_cast<float2*>(op + rr * HD + n * 8 + 2 * t4), make_float2(o[n][2 * h] * inv, o[n][2 * h + 1] * inv));
    if (t4 == 0) lp[rr] = (valid_row[h] && l_run[h] > 0.f) ? m_run[h] + logf(l_run[h]) : -INFINITY;
  }
}

// Rows [r0, r1) of a group: out = sum_s w_s o_s / sum_s w_s, w_s = exp(lse_s - max lse), in split
// order; bf16 to a.attn.  s_w: (r1 - r0) * (S + 1) floats of shared scratch.
template <int HD>
__device__ void attn_merge(const StackArgs& a, int group, int r0, int r1, int tid, float* s_w) {
  const int G = a.hq / a.hkv;
  const int rows = kQT * G;
  const int S = a.attn_splits;
  const Group gr = attn_group(a, group);
  const ReqDesc r = a.reqs[gr.req];
  const int tq0 = gr.qtile * kQT;
  for (int rr = r0 + tid; rr < r1; rr += kCompute) {  // per-row split weights, once
    float l[kStackMaxSplits];
    float mx = -INFINITY;
#pragma unroll
    for (int m = 0; m < kStackMaxSplits; ++m) {
      l[m] = m < S ? __ldcg(a.alse + static_cast<size_t>(group * S + m) * rows + rr) : -INFINITY;
      mx = fmaxf(mx, l[m]);
    }
    float den = 0.f;
    float* w = s_w + (rr - r0) * (S + 1);
#pragma unroll
    for (int m = 0; m < kStackMaxSplits; ++m) {
      if (m < S) {
        const float wm = l[m] == -INFINITY ? 0.f : expf(l[m] - mx);
        w[m] = wm;
        den += wm;
      }
    }
    w[S] = den > 0.f ? 1.f / den : 0.f;
  }
  named_sync(kComputeBar, kCompute);
  bf16* out = static_cast<bf16*>(a.attn);
  for (int idx = tid; idx < (r1 - r0) * (HD / 4); idx += kCompute) {
    const int rr = r0 + idx / (HD / 4), c4 = idx % (HD / 4);
    const int tq = tq0 + rr / G;
    if (tq >= r.n_q) continue;
    const float* w = s_w + (rr - r0) * (S + 1);
    float4 v[kStackMaxSplits];
#pragma unroll
    for (int m = 0; m < kStackMaxSplits; ++m)
      v[m] = (m < S && w[m] != 0.f)
                 ? __ldcg(reinterpret_cast<const float4*>(a.apart + (static_cast<size_t>(group * S + m) * rows + rr) * HD + c4 * 4))
                 : make_float4(0.f, 0.f, 0.f, 0.f);
    float4 num = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int m = 0; m < kStackMaxSplits; ++m) {
      if (m < S) {
        num.x += w[m] * v[m].x;
        num.y += w[m] * v[m].y;
        num.z += w[m] * v[m].z;
        num.w += w[m] * v[m].w;
      }
    }
    const float inv = w[S];
    bf16* op = out + static_cast<size_t>(r.q_tok0 + tq) * (a.hq * HD) + (gr.kvh * G + rr % G) * HD + c4 * 4;
    *reinterpret_cast<__nv_bfloat162*>(op) = __floats2bfloat162_rn(num.x * inv, num.y * inv);
    *reinterpret_cast<__nv_bfloat162*>(op + 2) = __floats2bfloat162_rn(num.z * inv, num.w * inv);
  }
}

// Sum of squares per 128-feature slab of row `row` of x (written to ss), copying x to h: the
// residual stream and the statistics of layer 0's input RMSNorm.  Same summation order as the
// residual epilogue (8-element chunks, then chunks in order).
__device__ void start_row(const StackArgs& a, int row, int tid, float* s_part) {
  const int H = a.H, cpr = H / 8;
  const bf16* x = static_cast<const bf16*>(a.x) + static_cast<size_t>(row) * H;
  bf16* hrow = static_cast<bf16*>(a.h) + static_cast<size_t>(row) * H;
  for (int c = tid; c < cpr; c += kCompute) {
    Chunk<bf16> v = ld_chunk(x + c * 8);
    st_chunk(hrow + c * 8, v);
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float f = __bfloat162float(v.e[j]);
      ss = fmaf(f, f, ss);
    }
    s_part[c] = ss;
  }
  named_sync(kComputeBar, kCompute);
  for (int sl = tid; sl < H / 128; sl += kCompute) {
    float ss = 0.f;
    for (int j = 0; j < 16; ++j) ss += s_part[sl * 16 + j];
    a.ss[static_cast<size_t>(row) * (H / 128) + sl] = ss;
  }
  named_sync(kComputeBar, kCompute);
}

__device__ __forceinline__ float row_rs(const StackArgs& a, int row) {
  constexpr int kMaxSlabs = 24;  // H <= 3072
  const int n = a.H / 128;
  const float* ssr = a.ss + static_cast<size_t>(row) * n;
  float v[kMaxSlabs];
#pragma unroll
  for (int j = 0; j < kMaxSlabs; ++j) v[j] = j < n ? __ldcg(ssr + j) : 0.f;  // all loads in flight at once
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < kMaxSlabs; ++j)
    if (j < n) ss += v[j];
  return rsqrtf(ss / static_cast<float>(a.H) + a.eps);
}

// Final RMSNorm of row `row`: out = T(w * T(h * rs)).
__device__ void final_row(const StackArgs& a, int row, int tid) {
  const int H = a.H;
  const float rs = row_rs(a, row);
  const bf16* hrow = static_cast<const bf16*>(a.h) + static_cast<size_t>(row) * H;
  const bf16* w = static_cast<const bf16*>(a.final_norm);
  bf16* out = static_cast<bf16*>(a.out) + static_cast<size_t>(row) * H;
  for (int c = tid; c < H / 8; c += kCompute) {
    Chunk<bf16> x = ld_chunk(hrow + c * 8);
    Chunk<bf16> wv;
    wv.u = *reinterpret_cast<const uint4*>(w + c * 8);
    Chunk<bf16> o;
    const __nv_bfloat162* x2 = reinterpret_cast<const __nv_bfloat162*>(&x.u);
    const __nv_bfloat162* w2 = reinterpret_cast<const __nv_bfloat162*>(&wv.u);
    __nv_bfloat162* o2 = reinterpret_cast<__nv_bfloat162*>(&o.u);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 xf = __bfloat1622float2(x2[j]);
      const float2 wf = __bfloat1622float2(w2[j]);
      const float2 xn = round2_bf16(xf.x * rs, xf.y * rs);
      o2[j] = __floats2bfloat162_rn(wf.x * xn.x, wf.y * xn.y);
    }
    st_chunk(out + c * 8, o);
  }
}

template <int HD>
__global__ void __launch_bounds__(kThreads, 1)
    stack_kernel(const __grid_constant__ StackArgs a, const __grid_constant__ CUtensorMap tm_h,
                 const __grid_constant__ CUtensorMap tm_attn, const __grid_constant__ CUtensorMap tm_act) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* ring = base;
  uint8_t* breg = base + kRingBytes;  // B operand k blocks / attention tiles / fp32 accumulator tile
  float* acc = reinterpret_cast<float*>(breg);
  uint64_t* full = reinterpret_cast<uint64_t*>(base + kBarOff);
  uint64_t* empty = full + kStackStages;
  uint64_t* b_tma = empty + kStackStages;  // [kBGroups] B operand group landed
  uint64_t* b_full = b_tma + kBGroups;     // [kBGroups] B operand group ready (normalised) for the MMA
  uint64_t* accf = b_full + kBGroups;      // accumulator complete
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accf + 1);
  volatile int* s_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* s_rs = reinterpret_cast<float*>(base + kBarOff + 256);    // [32] row scales
  float* s_part = reinterpret_cast<float*>(base + kBarOff + 512);  // start_row chunk sums (H / 8 <= 384)
  __shared__ __align__(16) unsigned char s_epi[5120];

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int cta = blockIdx.x;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStackStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int g = 0; g < kBGroups; ++g) {
      mbar_init(&b_tma[g], 1);
      mbar_init(&b_full[g], 1);
    }
    mbar_init(accf, 1);
    mbar_fence_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before_sync();
  __syncthreads();
  tc_fence_after_sync();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer: every weight tile of this CTA, all layers ----------------
      const uint64_t pol_w = l2_policy_evict_first();
      uint32_t it = 0;
      bool ok = true;
      for (int l = 0; l < a.L && ok; ++l) {
        for (int p = 0; p < 4 && ok; ++p) {
          const Unit u = gemm_unit(a, p, cta);
          if (!u.valid) continue;
          const CUtensorMap* m = a.wmaps + l * 4 + p;
          const int nk = u.kb1 - u.kb0;
          for (int gi = 0; gi < kBGroups && ok; ++gi) {
            const int g = (gi + cta) % kBGroups;
          for (int c = g * nk / kBGroups; c < (g + 1) * nk / kBGroups; ++c, ++it) {
            const int kb = u.kb0 + c;
            const int s = it % kStackStages;
            const uint32_t ph = (it / kStackStages) & 1u;
            if (!wait_bar(a, &empty[s], ph ^ 1u)) {
              if (!aborted(a.sync)) raise_abort(a, kErrTimeoutProducer);
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(&full[s], kAStage);
            uint8_t* dst = ring + s * kAStage;
            if (p == 2) {
              tma_load_2d(dst, m, &full[s], kb * 64, u.slab * 64, pol_w);
              tma_load_2d(dst + kAStage / 2, m, &full[s], kb * 64, a.I + u.slab * 64, pol_w);
            } else {
              tma_load_2d(dst, m, &full[s], kb * 64, u.slab * 128, pol_w);
            }
          }
          }
        }
      }
      // drain: the copies still in flight must land before shared memory goes away
      for (uint32_t i = it > static_cast<uint32_t>(kStackStages) ? it - kStackStages : 0u; i < it; ++i)
        if (!mbar_wait(&full[i % kStackStages], (i / kStackStages) & 1u)) break;
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer ----------------
      constexpr uint32_t idesc = umma_idesc_bf16(128, kStackRows);
      uint32_t it = 0, ucnt = 0;
      bool ok = true;
      for (int l = 0; l < a.L && ok; ++l) {
        for (int p = 0; p < 4 && ok; ++p) {
          const Unit u = gemm_unit(a, p, cta);
          if (!u.valid) continue;
          const int nk = u.kb1 - u.kb0;
          int kdone = 0;  // k blocks accumulated so far (the first one overwrites the accumulator)
          for (int gi = 0; gi < kBGroups && ok; ++gi) {
            const int g = (gi + cta) % kBGroups;  // rotated group order (spreads the B reads over L2)
            if (!wait_bar(a, &b_full[g], ucnt & 1u)) {
              if (!aborted(a.sync)) raise_abort(a, kErrTimeoutMma);
              ok = false;
              break;
            }
            tc_fence_after_sync();
            const int c0 = g * nk / kBGroups, c1 = (g + 1) * nk / kBGroups;
          for (int c = c0; c < c1; ++c, ++it, ++kdone) {
            const int kb = u.kb0 + c;
            const int s = it % kStackStages;
            const uint32_t ph = (it / kStackStages) & 1u;
            if (!wait_bar(a, &full[s], ph)) {
              if (!aborted(a.sync)) raise_abort(a, kErrTimeoutMma);
              ok = false;
              break;
            }
            tc_fence_after_sync();
            const uint64_t ad = umma_desc_sw128(ring + s * kAStage);
            const uint64_t bd = umma_desc_sw128(breg + c * kBChunk);
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
              tc_mma_bf16(tmem, ad + 2 * kk, bd + 2 * kk, idesc, (kdone > 0 || kk > 0) ? 1u : 0u);
            tc_commit(&empty[s]);
          }
          }
          if (!ok) break;
          tc_commit(accf);
          ++ucnt;
        }
      }
    }
  } else {
    // ---------------- compute warps ----------------
    const int tid = threadIdx.x - 64;
    const int cw = warp - 2;  // compute warp 0..5
    const uint64_t pol_x = l2_policy_evict_last();
    unsigned epoch = 0;
    uint32_t ucnt = 0, btcnt = 0;
    bool ok = true;
    const int G = a.hq / a.hkv;

    const size_t tstride = kStackTraceHead + static_cast<size_t>(a.L) * kStackTracePerLayer;
    auto mark = [&](int slot) {
      if (a.trace != nullptr && tid == 0) a.trace[static_cast<size_t>(cta) * tstride + slot] = global_timer_ns();
    };
    auto lmark = [&](int l, int ev) { mark(kStackTraceHead + l * kStackTracePerLayer + ev); };

    // Layer 0's input: residual stream h = x and its row statistics.
    mark(0);
    for (int row = cta; row < a.M; row += gridDim.x) start_row(a, row, tid, s_part);
    mark(1);
    ok = grid_barrier(a, epoch, tid, s_flag);
    mark(2);

    Epilogue base{};
    base.hq = a.hq;
    base.hkv = a.hkv;
    base.hd = a.hd;
    base.reqs = a.reqs;
    base.tok = a.tok;
    base.rope_cos = a.rope_cos;
    base.rope_sin = a.rope_sin;
    base.max_pos = a.max_pos;

    // One projection unit: B operand, MMA, TMEM drain, split-K merge, epilogue.
    auto gemm_phase = [&](int l, int p) -> bool {
      const Unit u = gemm_unit(a, p, cta);
      if (!u.valid) return true;
      const int ev = p == 0 ? 0 : (p == 1 ? 9 : (p == 2 ? 15 : 21));
      lmark(l, ev);
      const int nk = u.kb1 - u.kb0;
      const CUtensorMap* tmB = p == 1 ? &tm_attn : (p == 3 ? &tm_act : &tm_h);
      const StackLayer& Ly = a.layers[l];
      const void* norm_w = p == 0 ? Ly.ln1 : (p == 2 ? Ly.ln2 : nullptr);
      // B operand: TMA of the activation k blocks (rows >= M arrive as zeros) in ng groups; each
      // group is normalised in place (projections after an RMSNorm, model/cuda.py:269-275) and
      // released to the MMA issuer as soon as it is ready, so the MMAs start on the first group.
      // Always kBGroups groups (an empty group completes with 0 bytes), so every group barrier
      // completes exactly once per unit; CTAs visit the groups in rotated order.
      if (a.b_lsu) {
        // the same tiles through the load/store path (16-byte cp.async.cg), one commit group per
        // B group; rows >= M are zero-filled
        const bf16* src = static_cast<const bf16*>(p == 1 ? a.attn : (p == 3 ? a.act : a.h));
        const int ld = p == 1 ? a.hq * a.hd : (p == 3 ? a.I : a.H);
        for (int gi = 0; gi < kBGroups; ++gi) {
          const int g = (gi + cta) % kBGroups;
          const int c0 = g * nk / kBGroups, c1 = (g + 1) * nk / kBGroups;
          for (int idx = tid; idx < (c1 - c0) * kStackRows * 8; idx += kCompute) {
            const int c = c0 + idx / (kStackRows * 8), t = (idx >> 3) % kStackRows, cc = idx & 7;
            const bool valid = t < a.M;
            const bf16* sp = src + static_cast<size_t>(valid ? t : 0) * ld + (u.kb0 + c) * 64 + cc * 8;
            cp_async_16(breg + c * kBChunk + sw128_off(t, cc), sp, valid);
          }
          cp_async_commit();
        }
      } else if (tid == 0) {
        fence_proxy_async_global();
        for (int gi = 0; gi < kBGroups; ++gi) {
          const int g = (gi + cta) % kBGroups;
          const int c0 = g * nk / kBGroups, c1 = (g + 1) * nk / kBGroups;
          mbar_arrive_expect_tx(&b_tma[g], static_cast<uint32_t>((c1 - c0) * kBChunk));
          for (int c = c0; c < c1; ++c) tma_load_2d(breg + c * kBChunk, tmB, &b_tma[g], (u.kb0 + c) * 64, 0, pol_x);
        }
      }
      bf16* s_w = reinterpret_cast<bf16*>(s_epi);  // this unit's norm weights (nk * 64 <= 2560)
      if (norm_w != nullptr) {
        if (tid < kStackRows) s_rs[tid] = tid < a.M ? row_rs(a, tid) : 0.f;
        const uint4* wsrc = reinterpret_cast<const uint4*>(static_cast<const bf16*>(norm_w) + u.kb0 * 64);
        for (int c = tid; c < nk * 8; c += kCompute) reinterpret_cast<uint4*>(s_w)[c] = wsrc[c];
        named_sync(kComputeBar, kCompute);  // s_rs, s_w written
      }
      for (int gi = 0; gi < kBGroups; ++gi) {
        const int g = (gi + cta) % kBGroups;
        if (a.b_lsu) {
          switch (kBGroups - 1 - gi) {  // this thread's copies of groups 0..gi have landed
            case 3: cp_async_wait<3>(); break;
            case 2: cp_async_wait<2>(); break;
            case 1: cp_async_wait<1>(); break;
            default: cp_async_wait<0>(); break;
          }
          fence_proxy_async_smem();
          named_sync(kComputeBar, kCompute);  // everyone's copies of the group have landed
        } else if (!wait_bar(a, &b_tma[g], btcnt & 1u)) {
          if (tid == 0 && !aborted(a.sync)) raise_abort(a, kErrTimeoutEpilogue);
          return false;
        }
        if (gi == 0) lmark(l, ev + 1);
        const int c0 = g * nk / kBGroups, c1 = (g + 1) * nk / kBGroups;
        if (norm_w != nullptr && c1 > c0) {
          // thread -> one 8-column chunk of the group (8 weights in registers) x a stride of rows
          const int ncol = (c1 - c0) * 8;
          const int rgroups = max(1, kCompute / ncol);
          if (tid < ncol * rgroups) {
            const int col = c0 * 8 + tid % ncol, c = col >> 3, cc = col & 7;
            Chunk<bf16> wc;
            wc.u = reinterpret_cast<const uint4*>(s_w)[col];
            float wf[8];
#pragma unroll
            for (int v = 0; v < 8; ++v) wf[v] = __bfloat162float(wc.e[v]);
            uint8_t* cbase = breg + c * kBChunk;
#pragma unroll 4
            for (int t = tid / ncol; t < a.M; t += rgroups) {
              uint4* ptr = reinterpret_cast<uint4*>(cbase + sw128_off(t, cc));
              Chunk<bf16> x;
              x.u = *ptr;
              const float r = s_rs[t];
              __nv_bfloat162* x2 = reinterpret_cast<__nv_bfloat162*>(&x.u);
#pragma unroll
              for (int v = 0; v < 4; ++v) {
                const float2 xf = __bfloat1622float2(x2[v]);
                const float2 xn = round2_bf16(xf.x * r, xf.y * r);
                x2[v] = __floats2bfloat162_rn(wf[2 * v] * xn.x, wf[2 * v + 1] * xn.y);
              }
              *ptr = x.u;
            }
          }
          fence_proxy_async_smem();
          named_sync(kComputeBar, kCompute);
        }
        if (tid == 0) mbar_arrive(&b_full[g]);
      }
      ++btcnt;
      lmark(l, ev + 2);
      // accumulator -> shared fp32 tile acc[t][f] (over the B operand, which the MMAs are done with)
      if (!wait_bar(a, accf, ucnt & 1u)) {
        if (tid == 0 && !aborted(a.sync)) raise_abort(a, kErrTimeoutEpilogue);
        return false;
      }
      ++ucnt;
      lmark(l, ev + 3);
      tc_fence_after_sync();
      if (cw < 4) {
        const int q = warp & 3;  // TMEM lane quarter this warp may access
        uint32_t r[32];
        tmem_ld_32x32b_x32(tmem + (static_cast<uint32_t>(q * 32) << 16), r);
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 32; ++j) acc[j * 128 + q * 32 + lane] = __uint_as_float(r[j]);
      }
      tc_fence_before_sync();
      named_sync(kComputeBar, kCompute);

      GemmArgs g{};
      g.M = a.M;
      g.err = a.err;
      Epilogue e = base;
      e.layer = l;
      int ctr_base = kCtrQkv;
      switch (p) {
        case 0:
          g.N = (a.hq + 2 * a.hkv) * a.hd;
          e.kind = kEpiQkvRope;
          e.bias = Ly.qkv_b;
          e.qout = a.q;
          ctr_base = kCtrQkv;
          break;
        case 1:
          g.N = a.H;
          e.kind = kEpiResidual;
          e.resid = a.h;
          e.ld_resid = a.H;
          e.ss_out = a.ss;
          e.ss_ld = a.H / 128;
          ctr_base = kCtrO;
          break;
        case 2:
          g.N = 2 * a.I;
          g.paired = 1;
          e.kind = kEpiSiluMul;
          e.out = a.act;
          e.ld_out = a.I;
          break;
        default:
          g.N = a.H;
          e.kind = kEpiResidual;
          e.resid = a.h;
          e.ld_resid = a.H;
          e.ss_out = a.ss;
          e.ss_ld = a.H / 128;
          ctr_base = kCtrDown;
          break;
      }
      g.epi = e;
      int row0 = 0, row1 = kStackRows;
      if (u.splits > 1) {
        // split-K: publish this partial; once every split of the slab has, each split CTA sums its
        // own share of the token rows over all partials, in split order (deterministic), and runs
        // the epilogue for those rows.
        float4* mine = reinterpret_cast<float4*>(a.gpart + static_cast<size_t>(cta) * (kStackRows * 128));
        const float4* acc4 = reinterpret_cast<const float4*>(acc);
        for (int i = tid; i < a.M * 32; i += kCompute) __stcg(mine + i, acc4[i]);
        unsigned* ctr = a.sync + 64 + l * kStackCtrPerLayer + ctr_base + u.slab;
        if (p == 0) lmark(l, 30);
        if (!arrive_and_wait(a, ctr, static_cast<unsigned>(u.splits), tid, s_flag)) return false;
        if (p == 0) lmark(l, 31);
        row0 = u.split * a.M / u.splits;
        row1 = (u.split + 1) * a.M / u.splits;
        float4* accw = reinterpret_cast<float4*>(acc);
        const float4* part0 = reinterpret_cast<const float4*>(a.gpart) +
                              static_cast<size_t>(u.slab * u.splits) * (kStackRows * 32);
        for (int i = row0 * 32 + tid; i < row1 * 32; i += kCompute) {
          float4 v[kStackMaxSplits];
#pragma unroll
          for (int j = 0; j < kStackMaxSplits; ++j)
            v[j] = j < u.splits ? __ldcg(part0 + static_cast<size_t>(j) * (kStackRows * 32) + i)
                                : make_float4(0.f, 0.f, 0.f, 0.f);
          float4 sum = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
          for (int j = 0; j < kStackMaxSplits; ++j) {
            if (j < u.splits) {
              sum.x += v[j].x;
              sum.y += v[j].y;
              sum.z += v[j].z;
              sum.w += v[j].w;
            }
          }
          accw[i] = sum;
        }
        named_sync(kComputeBar, kCompute);
      }
      if (row1 > row0)
        gemm_epilogue<bf16>(g, acc, kStackRows, 0, u.slab, row0, row1, s_epi, tid, kCompute, kComputeBar);
      lmark(l, ev + 4);
      return true;
    };

    for (int l = 0; l < a.L && ok; ++l) {
      // qkv projection (+ input RMSNorm, bias, RoPE, KV append)
      ok = gemm_phase(l, 0);
      ok = grid_barrier(a, epoch, tid, s_flag) && ok;
      lmark(l, 5);
      if (!ok) break;
      // attention over the cache window
      lmark(l, 6);
      if (cta < a.attn_groups * a.attn_splits) {  // at most one unit per CTA (host-checked)
        const int group = cta / a.attn_splits, split = cta % a.attn_splits;
        attn_unit<HD>(a, l, group, split, breg, tid,
                      a.trace ? a.trace + static_cast<size_t>(cta) * tstride + kStackTraceHead + l * kStackTracePerLayer + 27
                              : nullptr);
        lmark(l, 28);
        unsigned* ctr = a.sync + 64 + l * kStackCtrPerLayer + kCtrAttn + group;
        if (a.attn_splits > 1) ok = arrive_and_wait(a, ctr, static_cast<unsigned>(a.attn_splits), tid, s_flag);
        lmark(l, 29);
        if (ok && a.attn_splits > 1) {  // every split of the group merges its share of the query rows
          const int rows = 16 * G;
          attn_merge<HD>(a, group, split * rows / a.attn_splits, (split + 1) * rows / a.attn_splits, tid,
                         reinterpret_cast<float*>(s_epi));
        }
      }
      lmark(l, 7);
      ok = grid_barrier(a, epoch, tid, s_flag) && ok;
      lmark(l, 8);
      if (!ok) break;
      // o projection + residual
      ok = gemm_phase(l, 1);
      ok = grid_barrier(a, epoch, tid, s_flag) && ok;
      lmark(l, 14);
      if (!ok) break;
      // gate_up (+ post-attention RMSNorm) -> SiLU(gate) * up
      ok = gemm_phase(l, 2);
      ok = grid_barrier(a, epoch, tid, s_flag) && ok;
      lmark(l, 20);
      if (!ok) break;
      // down projection + residual
      ok = gemm_phase(l, 3);
      ok = grid_barrier(a, epoch, tid, s_flag) && ok;
      lmark(l, 26);
    }
    if (ok && a.out != nullptr)
      for (int row = cta; row < a.M; row += gridDim.x) final_row(a, row, tid);
    mark(3);
  }
  __syncwarp();
  tc_fence_before_sync();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after_sync();
    tmem_dealloc(tmem, kTmemCols);
  }
}

}  // namespace

int stack_smem_bytes() { return kSmemBytes; }

int launch_stack(const StackArgs& a, const CUtensorMap& tm_h, const CUtensorMap& tm_attn, const CUtensorMap& tm_act,
                 int grid, cudaStream_t s) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = kSmemBytes;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;  // all CTAs co-resident: the grid barriers are safe
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  count_launch();
  if (a.hd == 128) return cudaLaunchKernelEx(&cfg, stack_kernel<128>, a, tm_h, tm_attn, tm_act);
  if (a.hd == 64) return cudaLaunchKernelEx(&cfg, stack_kernel<64>, a, tm_h, tm_attn, tm_act);
  return cudaErrorInvalidValue;
}

int init_stack_attributes() {
  cudaError_t e = cudaFuncSetAttribute(stack_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
  if (e == cudaSuccess) e = cudaFuncSetAttribute(stack_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
  return e;
}

}  // namespace fdllm
