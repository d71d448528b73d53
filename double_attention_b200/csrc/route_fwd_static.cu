// Dictionary-route forward without any caller-provided or allocated scratch.
//
// Who needs this: callers that cannot obtain device memory at the moment they
// run the route.  Two common cases are code that runs while a CUDA stream is
// being captured into a graph (a device allocation there is not allowed and
// would end the capture), and host engines that plan every device buffer
// before execution and hand a plugin only its inputs and outputs, with no
// workspace.  da_route_fwd needs a small global work area (a ticket counter
// for its last CTA, a counter and a list of rows to recompute exactly), which
// its normal callers allocate and pass in.  This entry point instead uses a
// work area compiled into the library as a file-scope __device__ array, so
// it takes only inputs and outputs and never allocates.
//
// Limits and sharing (also stated in include/da_b200.h):
//   * at most kStaticRouteRows route rows (groups * rows) per call; larger
//     calls are rejected with DA_ERR_WORKSPACE before any device work;
//   * every GPU that loads this library holds the array (about 256 KiB of
//     global memory) until the process exits;
//   * all calls on one device share the array; the kernel leaves its counters
//     at zero and this entry point clears them on the stream before each
//     launch, but calls that can overlap on the GPU (different streams, or
//     graphs replayed concurrently) race on it and must be serialised;
//   * the array's device address is looked up (cudaGetSymbolAddress) the first
//     time the entry point runs on a device, with that device made current;
//     that first call should therefore happen before any stream capture;
//   * the call makes q's device current while it runs and restores the
//     caller's current device before it returns.
#include <mutex>

#include "common.cuh"
#include "host_util.h"
#include "route_common.h"

namespace {

constexpr int kStaticRouteRows = 65536;

// [0] CTA ticket, [1] repair count, [2 ..] rows to recompute
static __device__ __align__(256) int g_route_scratch[2 + kStaticRouteRows];

std::mutex g_scratch_mutex;
int* g_scratch_addr[64] = {nullptr};

// Makes the device that owns `ptr` current for the lifetime of the guard and
// puts the caller's previous device back when it goes out of scope, so the
// entry point leaves the calling thread's current device as it found it.
class DeviceGuard {
 public:
  int enter(const void* ptr) {
    cudaPointerAttributes attr;
    if (cudaPointerGetAttributes(&attr, ptr) != cudaSuccess) return da::record_cuda_error();
    if (attr.type != cudaMemoryTypeDevice && attr.type != cudaMemoryTypeManaged) return DA_ERR_NULL;
    if (cudaGetDevice(&prev_) != cudaSuccess) {
      cudaGetLastError();
      prev_ = -1;
    }
    if (prev_ != attr.device) {
      if (cudaSetDevice(attr.device) != cudaSuccess) return da::record_cuda_error();
      switched_ = true;
    }
    device_ = attr.device;
    return DA_OK;
  }
  int device() const { return device_; }
  ~DeviceGuard() {
    if (switched_ && prev_ >= 0) cudaSetDevice(prev_);
  }

 private:
  int prev_ = -1, device_ = -1;
  bool switched_ = false;
};

// Device address of the static work area on device `dev` (looked up once).
int scratch_address(int dev, int** out) {
  if (dev < 0 || dev >= 64) return DA_ERR_UNSUPPORTED;
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  if (!g_scratch_addr[dev]) {
    void* p = nullptr;
    const cudaError_t err = cudaGetSymbolAddress(&p, g_route_scratch);
    if (err != cudaSuccess || !p) return da::record_cuda_error_code(static_cast<int>(err));
    g_scratch_addr[dev] = static_cast<int*>(p);
  }
  *out = g_scratch_addr[dev];
  return DA_OK;
}

}  // namespace

extern "C" int da_route_fwd_static(const void* q, int64_t rows, int64_t q_cols, int64_t q_row_stride, int groups,
                                   int64_t group_col_stride, int64_t R, int64_t M, int dtype, const void* dict_key_t,
                                   const void* dict_value, const float* beta, const float* dk_max, float eps,
                                   int normalize_input, int normalize_output, void* z, float* lse, float* out_norm,
                                   int* argmax, int* status, void* stream) {
  using namespace da;
  if (!q || !dict_key_t || !dict_value || !beta || !dk_max || !z || !lse || !out_norm || !status)
    return DA_ERR_NULL;
  if (dtype != DA_BF16 && dtype != DA_F16) return DA_ERR_DTYPE;
  if (rows <= 0 || groups <= 0 || M <= 0 || M % 64) return DA_ERR_SHAPE;
  if (R != 64 && R != 128 && R != 256 && R != 512) return DA_ERR_UNSUPPORTED;
  if ((int64_t)(groups - 1) * group_col_stride + R > q_cols || q_row_stride < q_cols) return DA_ERR_SHAPE;
  if (group_col_stride % 64 || (reinterpret_cast<uintptr_t>(z) & 15)) return DA_ERR_ALIGN;
  if ((int64_t)groups * rows > kStaticRouteRows) return DA_ERR_WORKSPACE;  // beyond the static work area
  DeviceGuard guard;  // q's device is current until this call returns
  if (int rc = guard.enter(q)) return rc;
  int* work = nullptr;
  if (int rc = scratch_address(guard.device(), &work)) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // The counters must start at zero; the row list needs no clearing.
  if (cudaMemsetAsync(work, 0, 2 * sizeof(int), st) != cudaSuccess) return record_cuda_error();
  route::RouteFwdArgs a{q, rows, q_cols, q_row_stride, groups, group_col_stride, R, M, dtype, dict_key_t,
                        dict_value, beta, dk_max, eps, normalize_input, normalize_output, z, lse, out_norm,
                        argmax, work, kStaticRouteRows, status};
  return route::route_fwd(a, st);
}
