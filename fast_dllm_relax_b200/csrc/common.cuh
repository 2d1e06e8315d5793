// Shared device helpers for the sm_100a Fast-dLLM v2 library: element types, the device error
// word, bounded mbarrier waits, TMA loads and the tcgen05 (5th-gen tensor core / TMEM) wrappers.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace fdllm {

using bf16 = __nv_bfloat16;

// ---- device error word ----------------------------------------------------------------------
// Kernels never trap: a failed check or an expired wait records the first error code here and the
// kernel returns.  The host reads it with fdllm_device_error().
enum DeviceError : int {
  kErrNone = 0,
  kErrTimeoutProducer = 1,   // TMA producer waited too long for a free pipeline slot
  kErrTimeoutMma = 2,        // MMA issuer waited too long for a filled slot
  kErrTimeoutEpilogue = 3,   // epilogue waited too long for the accumulator
  kErrTokenRange = 4,        // an input id outside [0, vocab)
  kErrPositionRange = 5,     // a RoPE position outside the precomputed table
  kErrCacheRange = 6,        // a KV write outside the cache capacity
  kErrTimeoutTest = 7,       // the bounded-wait self test expired (expected in that test)
  kErrReserved8 = 8,         // no longer raised (kept so that codes keep their meaning)
  kErrLoopLimit = 9,         // a device-side refinement loop exceeded its iteration limit
};

__device__ __forceinline__ void report_error(int* err, int code) {
  if (err != nullptr) atomicCAS(err, 0, code);
}

// report_error for an expired wait, with where it gave up: the first error also leaves err[1] =
// the wait site, err[2] = the call's token rows, err[3] = block index | split count << 16.
__device__ __forceinline__ void report_wait(int* err, int code, int site, int rows, int splits) {
  if (err == nullptr) return;
  if (atomicCAS(err, 0, code) == 0) {
    err[1] = site;
    err[2] = rows;
    err[3] = static_cast<int>(blockIdx.x) | (splits << 16);
  }
}

// ---- element conversions ------------------------------------------------------------------
template <typename T> __device__ __forceinline__ float to_f(T v);
template <> __device__ __forceinline__ float to_f<float>(float v) { return v; }
template <> __device__ __forceinline__ float to_f<bf16>(bf16 v) { return __bfloat162float(v); }

template <typename T> __device__ __forceinline__ T from_f(float v);
template <> __device__ __forceinline__ float from_f<float>(float v) { return v; }
template <> __device__ __forceinline__ bf16 from_f<bf16>(float v) { return __float2bfloat16_rn(v); }

// Round an fp32 value to the model dtype and widen it back (one op's result, in fp32 registers).
template <typename T> __device__ __forceinline__ float round_t(float v) { return to_f<T>(from_f<T>(v)); }

// Two values rounded to bf16 with one packed conversion (cvt.rn.bf16x2.f32; the scalar conversion
// runs at a fraction of the ALU rate) and widened back: identical to two round_t<bf16> calls.
__device__ __forceinline__ float2 round2_bf16(float a, float b) {
  return __bfloat1622float2(__floats2bfloat162_rn(a, b));
}

// Two fp32 values rounded to bf16 and packed (lo in the low half).
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// ---- time / addresses ---------------------------------------------------------------------
__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Kernel trace: tr[cta * kKtracePhases + p] = the %globaltimer value (ns) at which CTA `cta` (linear
// block index) of one launch reached phase p (0 entry, 1 dependency wait passed, 2 main loop done,
// 7 exit, the others kernel-specific); 0 = not reached.  Plain stores to distinct words: atomics
// on one per-launch word serialise in L2 and delay the stamping thread.  Phases 1 and 7 are always
// compiled in (a null check when tracing is off): the span from the first CTA passing its
// dependency wait to the last CTA leaving is the launch's share of the critical path.  The other
// phases only with FDLLM_KTRACE (compiled in, they slow every traced launch).
// Kernels that stamp come in two instantiations (kOn): the launch takes the stamping one only when
// a trace slot is attached, so an untraced launch carries no stamp code at all.
constexpr int kKtracePhases = 12;
constexpr int kKtraceMaxCta = 1280;  // CTAs of one launch recorded
template <bool kOn>
__device__ __forceinline__ void ktrace_stamp(unsigned long long* tr, int phase) {
  if constexpr (!kOn) return;
#ifndef FDLLM_KTRACE
  if (phase != 1 && phase != 7) return;
#endif
  if (tr == nullptr) return;
  const unsigned cta = blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z);
  if (cta < static_cast<unsigned>(kKtraceMaxCta)) tr[cta * kKtracePhases + phase] = global_timer_ns();
}

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// Every wait in this library gives up after this long and reports an error instead of hanging.
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s (a legitimate wait is microseconds)

// ---- mbarrier -----------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_fence_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(done)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

// Wait until the phase with parity `parity` has completed; false if kWaitLimitNs elapsed first.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 256; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (global_timer_ns() - t0 > kWaitLimitNs) return false;
  }
}

// Wait until the global counter *p reaches `target` (acquire at GPU scope: what the arriving
// CTAs wrote before their release is then visible); false if kWaitLimitNs elapsed first.
__device__ __forceinline__ bool wait_count_geq(const unsigned* p, unsigned target) {
  auto ld = [&]() {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
  };
  if (ld() >= target) return true;
  const uint64_t t0 = global_timer_ns();
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 64; ++i) {
      __nanosleep(32);
      if (ld() >= target) return true;
    }
    if (global_timer_ns() - t0 > kWaitLimitNs) return false;
  }
}

// Barrier `id` over the first `nthr` threads that reach it (a multiple of 32); id 0 with
// nthr == blockDim.x is __syncthreads().
__device__ __forceinline__ void named_sync(int id, int nthr) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthr) : "memory");
}

// ---- programmatic dependent launch ---------------------------------------------------------
// Kernels are launched with programmatic stream serialization: a kernel may start while its
// predecessor drains.  pdl_wait() blocks until the predecessor grid has completed and its memory is
// visible, so every read of a predecessor's output and every global write comes after it; work
// that touches only read-only data (weights) may come before.  pdl_trigger() lets the successor
// launch.  Both are no-ops for a kernel launched without the attribute.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ---- thread-block clusters: rank, barrier, distributed shared memory --------------------------
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// Every thread of every CTA in the cluster must reach this (no early exits before it).
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// cluster_sync in two halves (every thread calls arrive, then wait, alternately); the work between
// them overlaps the barrier.
__device__ __forceinline__ void cluster_arrive() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() {
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// The address of the same shared-memory location in cluster member `rank`.
__device__ __forceinline__ uint32_t map_shared_rank(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}

__device__ __forceinline__ float ld_dsmem_f32(uint32_t addr) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
  return v;
}

__device__ __forceinline__ float4 ld_dsmem_f4(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(addr)
               : "memory");
  return v;
}

// Make this thread's generic-proxy shared-memory writes visible to the async proxy (TMA / tcgen05).
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---- TMA (bulk tensor copies; plain CTA-local loads, no cluster forms) -----------------------
__device__ __forceinline__ void tma_prefetch_map(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

__device__ __forceinline__ uint64_t l2_policy_evict_last() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

// 2D tiled load of box (c0 = inner/contiguous coordinate, c1 = row) into shared memory; completion
// is signalled as transaction bytes on `bar`.
// L2 prefetch of one tile of a tensor map (no shared memory, no completion to wait for).
__device__ __forceinline__ void tma_prefetch_l2_2d(const CUtensorMap* map, int c0, int c1) {
  asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];" ::"l"(reinterpret_cast<uint64_t>(map)),
               "r"(c0), "r"(c1)
               : "memory");
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1,
                                            uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_addr(bar)), "r"(c0), "r"(c1), "l"(policy)
      : "memory");
}

// 3D tiled load of box (c0 inner, c1, c2) into shared memory, completion on `bar` (CTA-local).
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1, int c2,
                                            uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4, %5}], [%2], %6;" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_addr(bar)), "r"(c0), "r"(c1), "r"(c2), "l"(policy)
      : "memory");
}

// ---- tcgen05: TMEM allocation, MMA, commit, loads ------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t* slot, uint32_t ncols) {  // whole warp
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(slot)),
               "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tmem_relinquish() {  // whole warp
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {  // whole warp
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void tc_fence_before_sync() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after_sync() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T, bf16 inputs, fp32 accumulate (kind::f16), one CTA.
__device__ __forceinline__ void tc_mma_bf16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive once on `bar` when every tcgen05.mma issued so far by this thread has completed.
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_addr(bar))
               : "memory");
}

// 32 TMEM lanes (this warp's quarter) x 32 consecutive 32-bit columns -> 32 registers per thread.
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

// 32 TMEM lanes x 16 consecutive 32-bit columns -> 16 registers per thread.
__device__ __forceinline__ void tmem_ld_32x32b_x16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// 32 registers per thread -> 32 TMEM lanes x 32 consecutive 32-bit columns (the inverse of the load).
__device__ __forceinline__ void tmem_st_32x32b_x32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
      "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
      "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
      "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// UMMA shared-memory descriptor for a K-major bf16 tile written by TMA with 128-byte swizzling:
// rows of 64 elements (128 B), 8-row core groups 1024 B apart (stride byte offset), sm100 version
// bits = 1, layout type 2 = SWIZZLE_128B.  The tile base must be 1024-byte aligned; stepping K by 16
// elements inside the swizzle atom adds 32 bytes (2 in the >>4 address field).
__device__ __forceinline__ uint64_t umma_desc_sw128(const void* tile) {
  const uint32_t a = smem_addr(tile);
  uint64_t d = 0;
  d |= static_cast<uint64_t>((a >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>(1u) << 16;            // leading byte offset (unused for swizzled K-major)
  d |= static_cast<uint64_t>(1024u >> 4) << 32;    // stride byte offset: 8 rows x 128 B
  d |= static_cast<uint64_t>(1u) << 46;            // descriptor version (sm100)
  d |= static_cast<uint64_t>(2u) << 61;            // SWIZZLE_128B
  return d;
}

// UMMA shared-memory descriptor for an MN-major bf16 operand written by TMA with 128-byte swizzling:
// rows of 64 MN-consecutive elements (128 B) along K, 8-row (K) groups `sbo` bytes apart, and the
// next 64 MN elements `lbo` bytes further (the next 64-column TMA box).  Base 1024-byte aligned.
__device__ __forceinline__ uint64_t umma_desc_sw128_mn(const void* tile, uint32_t lbo, uint32_t sbo) {
  const uint32_t a = smem_addr(tile);
  uint64_t d = 0;
  d |= static_cast<uint64_t>((a >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1u) << 46;
  d |= static_cast<uint64_t>(2u) << 61;
  return d;
}

// Instruction descriptor, kind::f16: fp32 accumulator, bf16 A and B, both K-major, shape M x N.
__host__ __device__ constexpr uint32_t umma_idesc_bf16(int m, int n) {
  return (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(n >> 3) << 17) |
         (static_cast<uint32_t>(m >> 4) << 24);
}

// Instruction descriptor as umma_idesc_bf16 with the B operand MN-major (transposed).
__host__ __device__ constexpr uint32_t umma_idesc_bf16_bmn(int m, int n) { return umma_idesc_bf16(m, n) | (1u << 16); }

// ---- cp.async (Ampere-style 16-byte async copies, used by the attention kernel) -------------
__device__ __forceinline__ void cp_async_16(void* dst, const void* src, bool valid) {
  const int n = valid ? 16 : 0;  // n == 0 zero-fills the destination
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_addr(dst)), "l"(src), "r"(n)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N> __device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

}  // namespace fdllm
