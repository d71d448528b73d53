// Host helpers: error bookkeeping, tensor-map encoding, device attributes.
#include "host_util.h"

#include <atomic>
#include <mutex>

namespace da {

static thread_local int g_last_cuda_error = 0;

int record_cuda_error() {
  g_last_cuda_error = static_cast<int>(cudaGetLastError());
  return DA_ERR_CUDA;
}

int record_cuda_error_code(int code) {
  g_last_cuda_error = code;
  return DA_ERR_CUDA;
}

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*,
                                   CUtensorMapInterleave, CUtensorMapSwizzle, CUtensorMapL2promotion,
                                   CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
    else
      cudaGetLastError();
  });
  return fn;
}

int make_tmap_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, int elem_bytes, uint64_t inner,
                 uint64_t outer, uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer,
                 bool swizzle128) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return record_cuda_error_code(static_cast<int>(cudaErrorNotSupported));
  if ((reinterpret_cast<uintptr_t>(base) & 15) || (row_stride_bytes & 15)) return DA_ERR_ALIGN;
  if (swizzle128 && box_inner * static_cast<uint32_t>(elem_bytes) != 128) return DA_ERR_ALIGN;
  if (box_inner == 0 || box_outer == 0 || box_inner > 256 || box_outer > 256) return DA_ERR_SHAPE;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_stride_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return record_cuda_error_code(static_cast<int>(r));
  return DA_OK;
}

int make_tmap_blocks(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, int elem_bytes, int rank,
                     const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return record_cuda_error_code(static_cast<int>(cudaErrorNotSupported));
  if (rank < 3 || rank > 5) return DA_ERR_SHAPE;
  if (reinterpret_cast<uintptr_t>(base) & 15) return DA_ERR_ALIGN;
  if (box[0] * static_cast<uint32_t>(elem_bytes) != 128) return DA_ERR_ALIGN;
  cuuint64_t d[5], st[4];
  cuuint32_t b[5], e[5];
  for (int i = 0; i < rank; ++i) {
    if (dims[i] == 0 || box[i] == 0 || box[i] > 256 || box[i] > dims[i]) return DA_ERR_SHAPE;
    d[i] = dims[i];
    b[i] = box[i];
    e[i] = 1;
  }
  for (int i = 0; i < rank - 1; ++i) {
    if (strides_bytes[i] & 15) return DA_ERR_ALIGN;
    st[i] = strides_bytes[i];
  }
  CUresult r = fn(map, dtype, static_cast<cuuint32_t>(rank), const_cast<void*>(base), d, st, b, e,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return record_cuda_error_code(static_cast<int>(r));
  return DA_OK;
}

int bind_device(const void* ptr) {
  // One device per host thread (one process per GPU; autograd keeps one
  // worker thread per device), so the binding is done once per thread.
  static thread_local int bound = -1;
  if (bound >= 0) return DA_OK;
  cudaPointerAttributes attr;
  if (cudaPointerGetAttributes(&attr, ptr) != cudaSuccess) return record_cuda_error();
  if (attr.type != cudaMemoryTypeDevice && attr.type != cudaMemoryTypeManaged) return DA_OK;
  int cur = -1;
  if (cudaGetDevice(&cur) != cudaSuccess || cur != attr.device) {
    cudaGetLastError();
    if (cudaSetDevice(attr.device) != cudaSuccess) return record_cuda_error();
  }
  // cudaSetDevice is lazy about making the context current; touch it.
  if (cudaFree(nullptr) != cudaSuccess) return record_cuda_error();
  bound = attr.device;
  return DA_OK;
}

static int* g_debug_trace = nullptr;
int* debug_trace() { return g_debug_trace; }
void set_debug_trace(int* p) { g_debug_trace = p; }

int sm_count() {
  static int cached[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) { cudaGetLastError(); return 148; }
  if (dev < 0 || dev >= 64) return 148;
  if (!cached[dev]) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) {
      cudaGetLastError();
      n = 148;
    }
    cached[dev] = n;
  }
  return cached[dev];
}

}  // namespace da

extern "C" int da_last_cuda_error(void) { return da::g_last_cuda_error; }

namespace da {
namespace {
std::atomic<unsigned long long> g_kernel_launches{0};
}  // namespace
void note_launch() { g_kernel_launches.fetch_add(1, std::memory_order_relaxed); }
}  // namespace da

extern "C" uint64_t da_kernel_launches(void) { return da::g_kernel_launches.load(std::memory_order_relaxed); }

extern "C" int da_set_debug_trace(int* host_mapped) {
  da::set_debug_trace(host_mapped);
  return DA_OK;
}

extern "C" const char* da_status_string(int status) {
  switch (status) {
    case DA_OK: return "ok";
    case DA_ERR_NULL: return "null pointer argument";
    case DA_ERR_SHAPE: return "unsupported or inconsistent shape";
    case DA_ERR_DTYPE: return "unsupported dtype";
    case DA_ERR_ALIGN: return "pointer or stride not 16-byte aligned";
    case DA_ERR_UNSUPPORTED: return "unsupported variant";
    case DA_ERR_DEVICE_TIMEOUT: return "device-side wait timed out";
    case DA_ERR_CUDA: return "CUDA error (see da_last_cuda_error)";
    case DA_ERR_WORKSPACE: return "workspace too small";
    default: return "unknown status";
  }
}

extern "C" const char* da_version(void) { return "double-attention-b200 0.1.0 (sm_100a)"; }
