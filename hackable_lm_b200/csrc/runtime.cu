// Library-wide runtime utilities behind the C ABI: version, error strings,
// the device error word, the launch counter and the per-kernel timing hooks.
#include <atomic>
#include <mutex>

#include "hlm_common.cuh"

namespace hlm {

__device__ int g_device_error = 0;

int* device_error_ptr() {
  static int* ptr[64] = {nullptr};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  if (ptr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_device_error) != cudaSuccess) return nullptr;
    ptr[dev] = static_cast<int*>(p);
  }
  return ptr[dev];
}

SideStream* side_stream_of_current_device() {
  static std::mutex init_mu;
  static SideStream side[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> lock(init_mu);
  SideStream& ss = side[dev];
  if (ss.stream == nullptr) {
    if (cudaStreamCreateWithFlags(&ss.stream, cudaStreamNonBlocking) != cudaSuccess) return nullptr;
    if (cudaEventCreateWithFlags(&ss.ev_start, cudaEventDisableTiming) != cudaSuccess) return nullptr;
    for (int i = 0; i < kSideEvents; ++i)
      if (cudaEventCreateWithFlags(&ss.ev_done[i], cudaEventDisableTiming) != cudaSuccess) return nullptr;
  }
  return &ss;
}

static std::atomic<uint64_t> g_launches{0};

struct ProfileSlot {
  void* const* starts = nullptr;
  void* const* stops = nullptr;
  int capacity = 0;
  int launches = 0;
};
static ProfileSlot g_profile[HLM_KERNEL_MAX];
static std::mutex g_profile_mu;
static std::atomic<int> g_profile_active{0};

LaunchScope::LaunchScope(int kernel_id, cudaStream_t stream) : id_(kernel_id), stream_(stream) {
  if (g_profile_active.load(std::memory_order_relaxed) == 0) return;
  std::lock_guard<std::mutex> lock(g_profile_mu);
  if (id_ <= 0 || id_ >= HLM_KERNEL_MAX) return;
  ProfileSlot& sl = g_profile[id_];
  if (sl.starts == nullptr) return;
  slot_ = sl.launches++;
  if (slot_ < sl.capacity)
    cudaEventRecord(static_cast<cudaEvent_t>(sl.starts[slot_]), stream_);
  else
    slot_ = -1;
}

LaunchScope::~LaunchScope() {
  g_launches.fetch_add(1, std::memory_order_relaxed);
  if (slot_ < 0) return;
  std::lock_guard<std::mutex> lock(g_profile_mu);
  ProfileSlot& sl = g_profile[id_];
  if (sl.stops != nullptr && slot_ < sl.capacity)
    cudaEventRecord(static_cast<cudaEvent_t>(sl.stops[slot_]), stream_);
}

}  // namespace hlm

using namespace hlm;

extern "C" int hlm_version(void) { return 100; }

extern "C" const char* hlm_strerror(int code) {
  switch (code) {
    case HLM_OK:
      return "ok";
    case HLM_ERR_INVALID_ARG:
      return "invalid argument (null pointer, negative size or bad rank)";
    case HLM_ERR_UNSUPPORTED:
      return "unsupported shape, dtype, stride or alignment";
    case HLM_ERR_LAUNCH:
      return "CUDA launch or runtime error";
    case HLM_ERR_WORKSPACE:
      return "workspace smaller than required";
    case HLM_ERR_DRIVER:
      return "CUDA driver entry point or tensor-map encoding failed";
    default:
      return "unknown error code";
  }
}

extern "C" int hlm_device_error_get(int* out, void* stream) {
  if (out == nullptr) return HLM_ERR_INVALID_ARG;
  int* p = device_error_ptr();
  if (p == nullptr) return HLM_ERR_LAUNCH;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (cudaMemcpyAsync(out, p, sizeof(int), cudaMemcpyDeviceToHost, s) != cudaSuccess)
    return HLM_ERR_LAUNCH;
  if (cudaStreamSynchronize(s) != cudaSuccess) return HLM_ERR_LAUNCH;
  return HLM_OK;
}

extern "C" int hlm_device_error_clear(void* stream) {
  int* p = device_error_ptr();
  if (p == nullptr) return HLM_ERR_LAUNCH;
  if (cudaMemsetAsync(p, 0, sizeof(int), static_cast<cudaStream_t>(stream)) != cudaSuccess)
    return HLM_ERR_LAUNCH;
  return HLM_OK;
}

// One warp: lane 0 waits on a fresh mbarrier (phase 0 never completes: no
// thread arrives) through the bounded wait helpers the GEMM kernels use.
__global__ void __launch_bounds__(32) selftest_bounded_wait_kernel(unsigned long long limit_ns,
                                                                   int scope, int* err) {
  __shared__ alignas(8) uint64_t bar;
  const uint32_t b = smem_u32(&bar);
  if (threadIdx.x == 0) {
    mbar_init(b, 1);
    fence_mbar_init();
  }
  __syncwarp();
  if (threadIdx.x == 0) {
    if (scope == 0)
      mbar_wait_bounded(b, 0, limit_ns, err, kDevErrSelftestTimeout);
    else
      mbar_wait_cluster_bounded(b, 0, limit_ns, err, kDevErrSelftestTimeout);
  }
  __syncwarp();
}

extern "C" int hlm_selftest_bounded_wait(int64_t limit_us, int scope, void* stream) {
  if (limit_us < 1 || limit_us > 1000000 || (scope != 0 && scope != 1)) return HLM_ERR_INVALID_ARG;
  int* err = device_error_ptr();
  if (err == nullptr) return HLM_ERR_LAUNCH;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  {
    LaunchScope ls(0, s);
    selftest_bounded_wait_kernel<<<1, 32, 0, s>>>(static_cast<unsigned long long>(limit_us) * 1000ull,
                                                  scope, err);
  }
  return launch_status();
}

extern "C" uint64_t hlm_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

extern "C" int hlm_profile_begin(int kernel_id, void* const* start_events, void* const* stop_events,
                                 int capacity) {
  if (kernel_id <= 0 || kernel_id >= HLM_KERNEL_MAX || capacity < 0) return HLM_ERR_INVALID_ARG;
  if (capacity > 0 && (start_events == nullptr || stop_events == nullptr)) return HLM_ERR_INVALID_ARG;
  std::lock_guard<std::mutex> lock(g_profile_mu);
  ProfileSlot& sl = g_profile[kernel_id];
  const bool was_active = sl.starts != nullptr;
  sl.starts = capacity > 0 ? start_events : reinterpret_cast<void* const*>(&sl);
  sl.stops = capacity > 0 ? stop_events : nullptr;
  sl.capacity = capacity;
  sl.launches = 0;
  if (!was_active) g_profile_active.fetch_add(1);
  return HLM_OK;
}

extern "C" int hlm_profile_end(int kernel_id, int* launches) {
  if (kernel_id <= 0 || kernel_id >= HLM_KERNEL_MAX) return HLM_ERR_INVALID_ARG;
  std::lock_guard<std::mutex> lock(g_profile_mu);
  ProfileSlot& sl = g_profile[kernel_id];
  if (launches != nullptr) *launches = sl.launches;
  if (sl.starts != nullptr) g_profile_active.fetch_sub(1);
  sl = ProfileSlot();
  return HLM_OK;
}
