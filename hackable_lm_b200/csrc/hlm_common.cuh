// Shared device/host helpers for the hackable-lm B200 operator library.
//
// Everything here is sm_100a-only: mbarrier / TMA / tcgen05 wrappers written as
// inline PTX, bounded waits that report a timeout through a device error word
// instead of hanging, and small vector/numeric helpers used by the
// memory-bound kernels.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>

#include "../../include/hlm_b200.h"

#define HLM_DEVICE __device__ __forceinline__

namespace hlm {

// ---------------------------------------------------------------------------
// Device error word.  Kernels never trap: a bounded wait that runs out, or an
// index check that fails, records a code here and the kernel returns.  The
// host reads it with hlm_device_error_get().  device_error_ptr() returns the
// device address of the word for the current device (defined in gemm.cu).
// ---------------------------------------------------------------------------
int* device_error_ptr();

// One non-blocking side stream per device with a start event and kSideEvents
// completion events, created on first use and kept for the process (runtime.cu).
// Operators that run a memory-bound pass beside a GEMM fork it from the
// caller's stream (record ev_start there, wait on the side stream) and join it
// back (record ev_done[i] on the side stream, wait on the caller's), so each
// call stays stream-ordered for the caller.  Hold `mu` for the whole
// record/wait sequence of one call.
constexpr int kSideEvents = 4;
struct SideStream {
  std::mutex mu;
  cudaStream_t stream = nullptr;
  cudaEvent_t ev_start = nullptr;
  cudaEvent_t ev_done[kSideEvents] = {};
};
SideStream* side_stream_of_current_device();

// RAII scope around one kernel launch: counts the launch (hlm_launch_count)
// and, while hlm_profile_begin is active for `kernel_id`, records the
// caller's CUDA events around it on the launching stream.
class LaunchScope {
 public:
  LaunchScope(int kernel_id, cudaStream_t stream);
  ~LaunchScope();
  LaunchScope(const LaunchScope&) = delete;
  LaunchScope& operator=(const LaunchScope&) = delete;

 private:
  int id_;
  cudaStream_t stream_;
  int slot_ = -1;
};

enum DeviceErrorCode : int {
  kDevErrNone = 0,
  kDevErrTimeoutFull = 1,      // MMA warp waited too long for a TMA stage
  kDevErrTimeoutEmpty = 2,     // producer waited too long for a free stage
  kDevErrTimeoutTmemFull = 3,  // epilogue waited too long for an accumulator
  kDevErrTimeoutTmemEmpty = 4, // MMA warp waited too long for the epilogue
  kDevErrTimeoutDrain = 5,     // teardown drain of in-flight TMA copies ran out
  kDevErrBadTmem = 6,          // tcgen05.alloc returned an unexpected address
  kDevErrSelftestTimeout = 7,  // hlm_selftest_bounded_wait: the wait ran out (expected)
  kDevErrTimeoutEpiLoad = 8,   // an epilogue waited too long for its own TMA input load
  kDevErrTimeoutPeer = 9,      // an epilogue waited too long for its cluster peers' row sums
};
static_assert(kDevErrTimeoutFull == HLM_DEVERR_TIMEOUT_FULL && kDevErrTimeoutEmpty == HLM_DEVERR_TIMEOUT_EMPTY &&
                  kDevErrTimeoutTmemFull == HLM_DEVERR_TIMEOUT_TMEM_FULL &&
                  kDevErrTimeoutTmemEmpty == HLM_DEVERR_TIMEOUT_TMEM_EMPTY &&
                  kDevErrTimeoutDrain == HLM_DEVERR_TIMEOUT_DRAIN && kDevErrBadTmem == HLM_DEVERR_BAD_TMEM &&
                  kDevErrSelftestTimeout == HLM_DEVERR_SELFTEST_TIMEOUT &&
                  kDevErrTimeoutEpiLoad == HLM_DEVERR_TIMEOUT_EPI_LOAD &&
                  kDevErrTimeoutPeer == HLM_DEVERR_TIMEOUT_PEER,
              "device error codes match the public header");

// Upper bound for any single mbarrier wait.  Legitimate waits in these kernels
// are microseconds; one second means something is broken.
constexpr unsigned long long kWaitTimeoutNs = 1000000000ull;

HLM_DEVICE unsigned long long globaltimer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

HLM_DEVICE void record_error(int* err, int code) { atomicCAS(err, 0, code); }

// ---------------------------------------------------------------------------
// Shared-memory address helpers
// ---------------------------------------------------------------------------
HLM_DEVICE uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------
HLM_DEVICE void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

HLM_DEVICE void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

HLM_DEVICE void mbar_arrive(uint32_t bar) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\t"
      "mbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(bar)
      : "memory");
}

HLM_DEVICE void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\t"
      "mbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(bar),
      "r"(bytes)
      : "memory");
}

HLM_DEVICE bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// try_wait that lets the hardware suspend the thread for up to `hint_ns`; it
// resumes as soon as the phase completes.  Waiting this way keeps idle roles
// (e.g. an epilogue warp waiting out a long K loop) from spinning and taking
// issue slots and shared-memory cycles from the warps that do work.
HLM_DEVICE bool mbar_try_wait_sleep(uint32_t bar, uint32_t parity, uint32_t hint_ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity), "r"(hint_ns)
      : "memory");
  return ok != 0;
}

constexpr uint32_t kWaitSliceNs = 20000;  // suspend slice between timeout checks

// Bounded wait on phase `parity` of an mbarrier.  Returns false (and records
// `code` in the error word) if the phase did not complete within the timeout.
// The error word is sticky across launches, so it is not used to cut waits
// short: every wait in a failing CTA ends by its own timeout.
HLM_DEVICE bool mbar_wait_bounded(uint32_t bar, uint32_t parity, unsigned long long limit_ns,
                                  int* err, int code) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = globaltimer_ns();
  while (!mbar_try_wait_sleep(bar, parity, kWaitSliceNs)) {
    if (globaltimer_ns() - t0 > limit_ns) {
      record_error(err, code);
      return false;
    }
  }
  return true;
}
HLM_DEVICE bool mbar_wait(uint32_t bar, uint32_t parity, int* err, int code) {
  return mbar_wait_bounded(bar, parity, kWaitTimeoutNs, err, code);
}

// try_wait with cluster-scope acquire (pairs with mbar_arrive_cluster).
HLM_DEVICE bool mbar_try_wait_cluster(uint32_t bar, uint32_t parity, uint32_t hint_ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity), "r"(hint_ns)
      : "memory");
  return ok != 0;
}
// Bounded wait with cluster-scope acquire, for barriers that the peer CTA of a
// pair arrives on.
HLM_DEVICE bool mbar_wait_cluster_bounded(uint32_t bar, uint32_t parity, unsigned long long limit_ns,
                                          int* err, int code) {
  const unsigned long long t0 = globaltimer_ns();
  while (!mbar_try_wait_cluster(bar, parity, kWaitSliceNs)) {
    if (globaltimer_ns() - t0 > limit_ns) {
      record_error(err, code);
      return false;
    }
  }
  return true;
}
HLM_DEVICE bool mbar_wait_cluster(uint32_t bar, uint32_t parity, int* err, int code) {
  return mbar_wait_cluster_bounded(bar, parity, kWaitTimeoutNs, err, code);
}

// Wait by lane 0, result broadcast to the warp (keeps .sync.aligned
// instructions that follow convergent even when a wait times out).
HLM_DEVICE bool warp_wait(uint32_t bar, uint32_t parity, int* err, int code, int lane) {
  int ok = 1;
  if (lane == 0) ok = mbar_wait(bar, parity, err, code) ? 1 : 0;
  ok = __shfl_sync(0xffffffffu, ok, 0);
  return ok != 0;
}

// ---------------------------------------------------------------------------
// TMA (cp.async.bulk.tensor), plain CTA-local loads only.
// ---------------------------------------------------------------------------
HLM_DEVICE void tma_load_2d(uint32_t dst_smem, const CUtensorMap* map, int c0, int c1, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(dst_smem),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(bar)
      : "memory");
}

// TMA load into this CTA's shared memory whose completion is counted on an
// mbarrier given by cluster address -- the even CTA's barrier of a CTA pair
// (.cta_group::2).  The source is global memory of this GPU.
HLM_DEVICE void tma_load_2d_pair(uint32_t dst_smem, const CUtensorMap* map, int c0, int c1,
                                 uint32_t bar_cluster) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(dst_smem),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(bar_cluster)
      : "memory");
}

// TMA store of a 2-D box from shared memory (bulk async group of the issuing thread).
// Bring one box of a tensor map into L2 (no shared memory, no completion).
HLM_DEVICE void tma_prefetch_l2_2d(const CUtensorMap* map, int c0, int c1) {
  asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global [%0, {%1, %2}];" ::"l"(reinterpret_cast<uint64_t>(map)),
               "r"(c0), "r"(c1)
               : "memory");
}
HLM_DEVICE void tma_store_2d(const CUtensorMap* map, int c0, int c1, uint32_t src_smem) {
  asm volatile(
      "cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(c0), "r"(c1), "r"(src_smem)
      : "memory");
}
// L2 policy that marks written lines first in line for eviction (streamed
// outputs that should not push reused operands out of L2).
HLM_DEVICE uint64_t l2_policy_evict_first() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}
HLM_DEVICE void tma_store_2d_hint(const CUtensorMap* map, int c0, int c1, uint32_t src_smem,
                                  uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.global.shared::cta.bulk_group.L2::cache_hint [%0, {%1, %2}], [%3], %4;" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(c0), "r"(c1), "r"(src_smem), "l"(policy)
      : "memory");
}
HLM_DEVICE void bulk_commit_group() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Wait until at most N committed bulk groups still read their shared-memory source.
template <int N>
HLM_DEVICE void bulk_wait_group_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
// Wait until every committed bulk group has fully completed.
HLM_DEVICE void bulk_wait_group_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// Plain (untiled) bulk copy global -> this CTA's shared memory, completing on
// mbarrier bar; addresses 16-byte aligned, bytes a multiple of 16.
HLM_DEVICE void bulk_load_1d(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
               "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(bar)
               : "memory");
}

HLM_DEVICE uint4 ld_shared_v4(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(addr)
               : "memory");
  return v;
}
HLM_DEVICE void st_shared_v4(uint32_t addr, uint4 v) {
  asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z),
               "r"(v.w)
               : "memory");
}

HLM_DEVICE void prefetch_tensormap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

HLM_DEVICE void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---------------------------------------------------------------------------
// tcgen05 (5th-generation tensor cores + tensor memory)
// ---------------------------------------------------------------------------
HLM_DEVICE void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
               "r"(ncols)
               : "memory");
}
HLM_DEVICE void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
HLM_DEVICE void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
HLM_DEVICE void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
HLM_DEVICE void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T, kind::f16 (bf16 inputs, fp32 accumulate).
HLM_DEVICE void tc_mma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                           uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive on an mbarrier once every tcgen05.mma issued so far by this thread
// has completed.
HLM_DEVICE void tc_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   bar)
               : "memory");
}

// ---------------------------------------------------------------------------
// CTA pairs (clusters of two CTAs on one TPC) for tcgen05 cta_group::2: one
// thread of the even CTA issues an MMA with M = 256 whose A rows 0..127 and
// 128..255 live in the two CTAs' shared memory at the same offset, B columns
// split likewise, and D rows in each CTA's own TMEM.  No TMA load here reads
// another CTA's memory or fans out to several CTAs: every load stays CTA-local.
// ---------------------------------------------------------------------------
HLM_DEVICE uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
HLM_DEVICE uint32_t cluster_id_x() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
  return r;
}
HLM_DEVICE uint32_t num_clusters_x() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%nclusterid.x;" : "=r"(r));
  return r;
}
// Address of the same shared-memory offset in CTA `rank` of the cluster.
HLM_DEVICE uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}
// Arrive on an mbarrier given by a cluster address (possibly the peer CTA's),
// releasing this thread's prior writes at cluster scope.
HLM_DEVICE void mbar_arrive_cluster(uint32_t bar_cluster) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar_cluster)
               : "memory");
}
HLM_DEVICE void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::
                   : "memory");
}
HLM_DEVICE void tmem_alloc_pair(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
               "r"(ncols)
               : "memory");
}
HLM_DEVICE void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
HLM_DEVICE void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
HLM_DEVICE void tc_mma_f16_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive on the mbarrier at cluster address `bar_cluster` (this CTA's or the
// peer's) once every pair MMA issued so far by this thread has completed.
HLM_DEVICE void tc_commit_pair(uint32_t bar_cluster) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   bar_cluster)
               : "memory");
}

// 32 lanes x 32 consecutive 32-bit columns: thread i of the warp receives lane
// (taddr.lane + i), columns [taddr.col, taddr.col + 32).
HLM_DEVICE void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32"
      " {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15,"
      " %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]),
        "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]),
        "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
HLM_DEVICE void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Shared-memory matrix descriptor (tcgen05 format, version 1), 128-byte swizzle.
//   K-major operand : LBO = 16 B (unused), SBO = 1024 B (8 rows x 128 B)
//   MN-major operand: LBO = byte stride between 64-element MN blocks,
//                     SBO = 1024 B (8 K-rows x 128 B)
HLM_DEVICE uint64_t make_sw128_desc(uint32_t smem_addr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= 1ull << 46;  // descriptor version for tcgen05
  d |= 2ull << 61;  // layout: 128-byte swizzle
  return d;
}

// Instruction descriptor for kind::f16 with bf16 A/B and fp32 D.
__host__ __device__ constexpr uint32_t make_idesc_bf16_f32(int M, int N, bool a_mn_major,
                                                          bool b_mn_major) {
  return (1u << 4)                                  // D format: f32
         | (1u << 7)                                // A format: bf16
         | (1u << 10)                               // B format: bf16
         | (static_cast<uint32_t>(a_mn_major) << 15)  // A major
         | (static_cast<uint32_t>(b_mn_major) << 16)  // B major
         | (static_cast<uint32_t>(N >> 3) << 17)      // N / 8
         | (static_cast<uint32_t>(M >> 4) << 24);     // M / 16
}

// ---------------------------------------------------------------------------
// Numeric helpers
// ---------------------------------------------------------------------------
template <typename T>
HLM_DEVICE float to_f32(T v);
template <>
HLM_DEVICE float to_f32<float>(float v) { return v; }
template <>
HLM_DEVICE float to_f32<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <>
HLM_DEVICE float to_f32<__half>(__half v) { return __half2float(v); }

template <typename T>
HLM_DEVICE T from_f32(float v);
template <>
HLM_DEVICE float from_f32<float>(float v) { return v; }
template <>
HLM_DEVICE __nv_bfloat16 from_f32<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }
template <>
HLM_DEVICE __half from_f32<__half>(float v) { return __float2half_rn(v); }

// 16-byte vector of T, converted to/from fp32 registers.
template <typename T>
struct Vec16 {
  static constexpr int N = 16 / sizeof(T);
  uint4 raw;
  HLM_DEVICE void to_float(float (&f)[N]) const {
    const T* p = reinterpret_cast<const T*>(&raw);
#pragma unroll
    for (int i = 0; i < N; ++i) f[i] = to_f32<T>(p[i]);
  }
  HLM_DEVICE void from_float(const float (&f)[N]) {
    T* p = reinterpret_cast<T*>(&raw);
#pragma unroll
    for (int i = 0; i < N; ++i) p[i] = from_f32<T>(f[i]);
  }
};

HLM_DEVICE uint4 ld_global_nc_v4(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}
HLM_DEVICE uint4 ld_global_v4(const void* p) {
  uint4 v;
  asm volatile("ld.global.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}
HLM_DEVICE void st_global_v4(void* p, uint4 v) {
  asm volatile("st.global.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z),
               "r"(v.w)
               : "memory");
}

// Element `idx` of a cos/sin table stored as fp32, bf16 or fp16.
HLM_DEVICE float load_cs(const void* p, int64_t idx, int cs_dtype) {
  switch (cs_dtype) {
    case HLM_BF16:
      return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[idx]);
    case HLM_F16:
      return __half2float(static_cast<const __half*>(p)[idx]);
    default:
      return static_cast<const float*>(p)[idx];
  }
}

// 2^x with the hardware approximation (PTX ex2.approx.ftz.f32): results below
// the smallest normal float flush to zero, which is harmless where the values
// are softmax terms.
HLM_DEVICE float ex2_ftz(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// bf16 pair (packed, low half first) -> two floats; exact.
HLM_DEVICE float bf16_lo(uint32_t w) { return __uint_as_float(w << 16); }
HLM_DEVICE float bf16_hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }
HLM_DEVICE uint32_t max_bf16x2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("max.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
HLM_DEVICE uint32_t pack_bf16x2(float lo, float hi) {
  const __nv_bfloat162 h2 = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h2);
}

HLM_DEVICE float sigmoidf_(float x) { return 1.0f / (1.0f + __expf(-x)); }
// 1 / (1 + 2^(-x log2 e)) with the hardware ex2 and an approximate divide
// (two MUFU ops, a few ulp of fp32): for kernels whose outputs are bf16.
HLM_DEVICE float sigmoid_fast(float x) {
  return __fdividef(1.0f, 1.0f + ex2_ftz(x * -1.4426950408889634f));
}

HLM_DEVICE float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Host helper: 16-byte alignment of a device pointer.
inline bool host_aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

inline int num_sms_of_current_device() {
  static int cached[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (dev < 0 || dev >= 64) return 148;
  if (cached[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
    cached[dev] = n;
  }
  return cached[dev];
}

inline int launch_status() {
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? HLM_OK : HLM_ERR_LAUNCH;
}

}  // namespace hlm
