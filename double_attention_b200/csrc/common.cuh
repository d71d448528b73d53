// Device-side building blocks for the sm_100a kernels of this library:
// mbarriers with bounded waits, TMA tile loads, tcgen05 (TMEM alloc, MMA,
// commit, loads) and the shared-memory / instruction descriptors the
// 5th-generation tensor cores consume.
//
// Every wait in this file is bounded by wall-clock time (the %globaltimer
// register).  A wait that runs out records DA_DEV_TIMEOUT in the kernel's
// status word and returns false; callers then leave their role loops and
// tear down normally, so a logic error ends the kernel with an error status
// instead of hanging the GPU.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <type_traits>

#define DA_DEV __device__ __forceinline__

namespace da {

// Status bits a kernel may OR into its device status word.
enum : int {
  DA_DEV_TIMEOUT = 1,        // a bounded wait ran out
  DA_DEV_ROW_OVERFLOW = 2,   // more low-mass rows than the repair list holds
  DA_DEV_LOW_MASS = 4,       // a softmax row's largest term fell below 2^-100
};

constexpr unsigned long long kWaitTimeoutNs = 2000000000ull;  // 2 s per wait

DA_DEV uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

DA_DEV unsigned long long globaltimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

DA_DEV uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// Address of the same shared variable in CTA `rank` of this cluster.
DA_DEV uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}

DA_DEV void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\t"
               "barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

DA_DEV void named_bar_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" :: "r"(id), "r"(threads) : "memory");
}

// ---------------------------------------------------------------- mbarrier
DA_DEV void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" :: "r"(smem_u32(bar)), "r"(count)
               : "memory");
}

DA_DEV void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

DA_DEV void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;"
               :: "r"(smem_u32(bar)), "r"(bytes) : "memory");
}

DA_DEV void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" :: "r"(smem_u32(bar)) : "memory");
}

// Arrive on a barrier that may live in another CTA of the cluster.
DA_DEV void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];"
               :: "r"(cluster_addr) : "memory");
}

// Arrive (release at CTA scope, the default) on a barrier that may live in another CTA of the cluster:
// the hand-off of shared-memory tiles written with generic stores and fenced to the async proxy.
DA_DEV void mbar_arrive_remote(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" :: "r"(cluster_addr) : "memory");
}

// Arrive with relaxed semantics (no memory ordering): for barriers that only count events, such as
// "this warp has read its TMEM columns" after tcgen05.fence::before_thread_sync.
DA_DEV void mbar_arrive_cluster_relaxed(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.relaxed.cluster.shared::cluster.b64 _, [%0];" :: "r"(cluster_addr) : "memory");
}

// Upper bound on how long one probe may suspend the thread (the hardware
// resumes it earlier when the phase completes).
#ifndef DA_SUSPEND_HINT_NS
#define DA_SUSPEND_HINT_NS 20000u
#endif
constexpr uint32_t kSuspendHintNs = DA_SUSPEND_HINT_NS;

// One bounded probe of a barrier phase.
DA_DEV bool mbar_test(uint32_t addr, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok) : "r"(addr), "r"(parity), "r"(kSuspendHintNs) : "memory");
  return ok != 0;
}

// Kernel-wide abort state: a shared flag plus the global status words
// (status[0]: OR of DA_DEV_* bits; status[1]: site code of the first wait
// that gave up, 0 if none).
struct Abort {
  int* smem_flag;   // shared: set once any wait in this CTA gives up
  int* status;      // global status words (may be null)
};

// Wait until the barrier phase with the given parity has completed.
// Returns false when the wait gave up (timeout, or another role of this CTA
// aborted).  `site` identifies the wait in status[1] when it times out.
// `timeout_ns` bounds the wait (kWaitTimeoutNs for every kernel wait; the
// failure-detection self-test passes a short limit).
DA_DEV bool mbar_wait(uint64_t* bar, uint32_t parity, const Abort& ab, int site = 0,
                      unsigned long long timeout_ns = kWaitTimeoutNs) {
  const uint32_t addr = smem_u32(bar);
  if (mbar_test(addr, parity)) return true;
  const unsigned long long t0 = globaltimer();
  while (true) {
    if (mbar_test(addr, parity)) return true;
    if (*reinterpret_cast<volatile int*>(ab.smem_flag)) return false;
    if (globaltimer() - t0 > timeout_ns) {
      *reinterpret_cast<volatile int*>(ab.smem_flag) = 1;
      if (ab.status) {
        atomicOr(ab.status, DA_DEV_TIMEOUT);
        atomicCAS(ab.status + 1, 0, site ? site : -1);
      }
      return false;
    }
  }
}

// Like mbar_wait but ignores the abort flag: used while draining in-flight
// asynchronous work before teardown.  Still bounded by the timeout.
DA_DEV bool mbar_wait_drain(uint64_t* bar, uint32_t parity) {
  const uint32_t addr = smem_u32(bar);
  const unsigned long long t0 = globaltimer();
  while (!mbar_test(addr, parity)) {
    if (globaltimer() - t0 > kWaitTimeoutNs) return false;
  }
  return true;
}

// Debug progress markers: when `trace` is non-null (pinned host memory that
// the host can read while a kernel runs), trace[cta * 8 + slot] = value with
// a system-scope store.  Used to locate a kernel that does not finish.
DA_DEV void trace_mark(int* trace, int slot, int value) {
  if (trace) {
    int* dst = trace + blockIdx.x * 8 + slot;
    asm volatile("st.volatile.global.s32 [%0], %1;" :: "l"(dst), "r"(value) : "memory");
    __threadfence_system();
  }
}

// Post-mortem timestamp (no fence; read after the kernel completed):
// trace[index] = low 31 bits of %globaltimer in ns.
DA_DEV void trace_at(int* trace, int index) {
  if (trace) {
    const int v = static_cast<int>(globaltimer() & 0x7fffffffull);
    asm volatile("st.global.s32 [%0], %1;" :: "l"(trace + index), "r"(v) : "memory");
  }
}

// Records the low 31 bits of %globaltimer (ns) in the trace slot (plain
// store, read after the kernel completed).
DA_DEV void trace_time(int* trace, int slot) {
  if (trace) trace_at(trace, blockIdx.x * 8 + slot);
}

// ---------------------------------------------------------------- programmatic dependent launch
// Kernels are launched with programmatic stream serialisation allowed: a
// kernel may start (and run its setup) while the previous kernel on the
// stream drains.  Every kernel calls grid_dependency_wait() after its setup
// and before touching global memory, which returns once the previous kernels
// have completed and their writes are visible; grid_launch_dependents() lets
// the next kernel be scheduled as soon as every CTA of this one has started.
DA_DEV void grid_dependency_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
DA_DEV void grid_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ---------------------------------------------------------------- TMA
DA_DEV void prefetch_tmap(const void* tmap) {
  asm volatile("prefetch.tensormap [%0];" :: "l"(tmap) : "memory");
}

// 2-D tiled load into this CTA's shared memory; completion is signalled on
// a barrier of this CTA.
DA_DEV void tma_load_2d(const void* tmap, uint64_t* bar, void* dst, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];"
      :: "r"(smem_u32(dst)), "l"(tmap), "r"(smem_u32(bar)), "r"(x), "r"(y) : "memory");
}

// Warms L2 with one 2-D tile of this GPU's global memory (no shared memory,
// no barrier): issued a few stages ahead of the real loads so that they hit
// L2 instead of waiting on HBM.
DA_DEV void tma_prefetch_2d(const void* tmap, int x, int y) {
  asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];"
               :: "l"(tmap), "r"(x), "r"(y) : "memory");
}

// 2-D tiled load for a CTA pair running paired (cta_group::2) MMAs: the data
// lands in this CTA's shared memory and the byte count is signalled on the
// barrier at `bar_cluster_addr`, which lives in the pair's leader CTA.
DA_DEV void tma_load_2d_pair(const void* tmap, uint32_t bar_cluster_addr, void* dst, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];"
      :: "r"(smem_u32(dst)), "l"(tmap), "r"(bar_cluster_addr), "r"(x), "r"(y) : "memory");
}

// 3-D / 4-D tiled loads for a CTA pair (see tma_load_2d_pair): one issue
// brings several 128-byte column blocks of the same rows (make_tmap_blocks).
DA_DEV void tma_load_3d_pair(const void* tmap, uint32_t bar_cluster_addr, void* dst, int x, int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];"
      :: "r"(smem_u32(dst)), "l"(tmap), "r"(bar_cluster_addr), "r"(x), "r"(y), "r"(z) : "memory");
}
DA_DEV void tma_load_4d_pair(const void* tmap, uint32_t bar_cluster_addr, void* dst, int x, int y, int z, int w) {
  asm volatile(
      "cp.async.bulk.tensor.4d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];"
      :: "r"(smem_u32(dst)), "l"(tmap), "r"(bar_cluster_addr), "r"(x), "r"(y), "r"(z), "r"(w) : "memory");
}

// 1-D bulk copy of `bytes` (a multiple of 16; both addresses 16-byte aligned) from global memory into
// this CTA's shared memory, completion signalled on a barrier of this CTA.
DA_DEV void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
               :: "r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar)) : "memory");
}

// 2-D tiled store from shared memory (bulk-group completion).
DA_DEV void tma_store_2d(const void* tmap, const void* src, int x, int y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.tile.bulk_group [%0, {%2, %3}], [%1];"
               :: "l"(tmap), "r"(smem_u32(src)), "r"(x), "r"(y) : "memory");
}
DA_DEV void tma_store_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
DA_DEV void tma_store_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// Make generic-proxy shared-memory writes visible to the async proxy
// (tensor cores, TMA).
DA_DEV void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// ---------------------------------------------------------------- tcgen05
template <int kCtaGroup>
DA_DEV void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  if constexpr (kCtaGroup == 1)
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                 :: "r"(smem_u32(dst_smem)), "r"(ncols) : "memory");
  else
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;"
                 :: "r"(smem_u32(dst_smem)), "r"(ncols) : "memory");
}

template <int kCtaGroup>
DA_DEV void tmem_relinquish() {
  if constexpr (kCtaGroup == 1)
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  else
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}

template <int kCtaGroup>
DA_DEV void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  if constexpr (kCtaGroup == 1)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" :: "r"(taddr), "r"(ncols)
                 : "memory");
  else
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" :: "r"(taddr), "r"(ncols)
                 : "memory");
}

DA_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
DA_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
DA_DEV void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// D[tmem] (+)= A[smem] * B[smem]^T, kind::f16 (fp16/bf16 operands, fp32 accum).
template <int kCtaGroup>
DA_DEV void mma_f16_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                       uint32_t accumulate) {
  if constexpr (kCtaGroup == 1)
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        :: "r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate) : "memory");
  else
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        :: "r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate) : "memory");
}

// Arrive once on the barrier (any CTA of the cluster) when all previously
// issued tcgen05 operations of this thread have completed.
template <int kCtaGroup>
DA_DEV void mma_commit(uint32_t bar_cluster_addr) {
  if constexpr (kCtaGroup == 1)
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                 :: "r"(bar_cluster_addr) : "memory");
  else
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                 :: "r"(bar_cluster_addr) : "memory");
}

// Paired-CTA form of mma_commit: one arrive on the barrier at this shared-memory offset in each CTA of
// the pair (a multicast commit instead of one per CTA).
DA_DEV void mma_commit_pair(uint32_t bar_smem_addr) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;"
               :: "r"(bar_smem_addr), "h"((uint16_t)0x3) : "memory");
}

// 32 lanes x 32 bit, 32 consecutive columns: thread i of the warp receives
// TMEM lane (base lane + i), columns [col, col+32).
DA_DEV void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// 32 lanes x 32 bit, 16 consecutive columns.
DA_DEV void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// ---------------------------------------------------------------- descriptors
// Shared-memory matrix descriptor for the 128-byte swizzled canonical
// layouts that a TMA load with CU_TENSOR_MAP_SWIZZLE_128B produces
// (rows of 128 bytes; 16-byte chunk c of row r stored at chunk c ^ (r & 7);
// tile bases 1024-byte aligned).
//   K-major : rows run along M/N, the 128 bytes run along K.  SBO = byte
//             distance between consecutive groups of 8 rows; LBO unused.
//   MN-major: rows run along K, the 128 bytes run along M/N (64 elements).
//             LBO = byte distance between consecutive 64-element M/N blocks,
//             SBO = byte distance between consecutive groups of 8 K rows.
// Bits: [0,14) start>>4, [16,30) LBO>>4, [32,46) SBO>>4, [46,48) version=1,
// [49,52) base offset=0, bit 52 LBO mode=0, [61,64) layout (2 = 128B swizzle).
DA_DEV uint64_t sdesc_sw128(uint32_t smem_addr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1) << 46;
  d |= static_cast<uint64_t>(2) << 61;
  return d;
}

// Instruction descriptor for kind::f16 with fp32 accumulation.
//   ab_bf16: operands are bf16 (else fp16); both operands share one type.
//   a_mn / b_mn: operand is MN-major (else K-major).
__host__ __device__ constexpr uint32_t idesc_f16(int M, int N, bool ab_bf16, bool a_mn, bool b_mn) {
  return (1u << 4)                                   // D format: f32
         | ((ab_bf16 ? 1u : 0u) << 7)                // A format
         | ((ab_bf16 ? 1u : 0u) << 10)               // B format
         | ((a_mn ? 1u : 0u) << 15)                  // A major
         | ((b_mn ? 1u : 0u) << 16)                  // B major
         | (static_cast<uint32_t>(N >> 3) << 17)     // N / 8
         | (static_cast<uint32_t>(M >> 4) << 24);    // M / 16
}

// Byte offset of the 16-byte chunk `chunk` (0..7) of row `row` inside a
// 128-byte-swizzled tile whose rows are 128 bytes long.
DA_DEV uint32_t sw128_offset(uint32_t row, uint32_t chunk) {
  return row * 128u + ((chunk ^ (row & 7u)) << 4);
}

// ---------------------------------------------------------------- numerics
// 2^x on the special-function unit (PTX ex2.approx, flush-to-zero).
DA_DEV float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

template <typename T> DA_DEV T from_f32(float x);
template <> DA_DEV __nv_bfloat16 from_f32<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }
template <> DA_DEV __half from_f32<__half>(float x) { return __float2half_rn(x); }

DA_DEV uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}
DA_DEV uint32_t pack_f16x2(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}
template <typename T> DA_DEV uint32_t pack2(float lo, float hi);
template <> DA_DEV uint32_t pack2<__nv_bfloat16>(float lo, float hi) { return pack_bf16x2(lo, hi); }
template <> DA_DEV uint32_t pack2<__half>(float lo, float hi) { return pack_f16x2(lo, hi); }

template <typename T> DA_DEV float2 unpack2(uint32_t v);
template <> DA_DEV float2 unpack2<__nv_bfloat16>(uint32_t v) {
  return __bfloat1622float2(*reinterpret_cast<__nv_bfloat162*>(&v));
}
template <> DA_DEV float2 unpack2<__half>(uint32_t v) {
  return __half22float2(*reinterpret_cast<__half2*>(&v));
}

DA_DEV void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" :: "r"(addr), "r"(a), "r"(b), "r"(c),
               "r"(d) : "memory");
}
DA_DEV uint4 ld_shared_v4(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr) : "memory");
  return v;
}

}  // namespace da
