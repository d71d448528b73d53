// Outer routed attention, backward: the row deltas of one map,
//   delta[r] = <dY[r, :], Y[r, :]>,
// the preprocess step of _routed_attention_triton_backward
// (triton_kernels.py:2093-2160) for a single map, whose saved forward output
// is Y.  The backward products themselves are in attn_bwd_mixed.cu.
#include "common.cuh"
#include "host_util.h"

namespace da {
namespace attn {
namespace bwd {

// =============================================================================== delta
// delta[b, t] = <dY[b, t, :], Y[b, t, :]>  (one warp per row)
template <typename T>
__global__ void delta_kernel(const T* __restrict__ dy, const T* __restrict__ y, int64_t rows, int D,
                             float* __restrict__ delta) {
  grid_dependency_wait();
  grid_launch_dependents();
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (row >= rows) return;
  float acc = 0.f;
  for (int c = lane * 8; c < D; c += 256) {
    const uint4 a = *reinterpret_cast<const uint4*>(dy + row * D + c);
    const uint4 bq = *reinterpret_cast<const uint4*>(y + row * D + c);
    const uint32_t wa[4] = {a.x, a.y, a.z, a.w}, wb[4] = {bq.x, bq.y, bq.z, bq.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 fa = unpack2<T>(wa[e]), fb = unpack2<T>(wb[e]);
      acc = fmaf(fa.x, fb.x, fmaf(fa.y, fb.y, acc));
    }
  }
  for (int o = 16; o; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if (lane == 0) delta[row] = acc;
}

}  // namespace bwd
}  // namespace attn
}  // namespace da

extern "C" int da_attn_bwd_delta(const void* dy, const void* y, int64_t rows, int D, int dtype, float* delta,
                                 void* stream) {
  using namespace da;
  if (!dy || !y || !delta) return DA_ERR_NULL;
  if (dtype != DA_BF16 && dtype != DA_F16) return DA_ERR_DTYPE;
  if (int rc = bind_device(dy)) return rc;
  if (rows <= 0 || D <= 0 || D % 256) return DA_ERR_SHAPE;
  if ((reinterpret_cast<uintptr_t>(dy) | reinterpret_cast<uintptr_t>(y)) & 15) return DA_ERR_ALIGN;
  const int per_block = 8;
  const unsigned grid = (unsigned)((rows + per_block - 1) / per_block);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (dtype == DA_BF16)
    return launch_kernel(attn::bwd::delta_kernel<__nv_bfloat16>, dim3(grid), dim3(32 * per_block), 0, st, false,
                         static_cast<const __nv_bfloat16*>(dy), static_cast<const __nv_bfloat16*>(y), rows, D, delta);
  return launch_kernel(attn::bwd::delta_kernel<__half>, dim3(grid), dim3(32 * per_block), 0, st, false,
                       static_cast<const __half*>(dy), static_cast<const __half*>(y), rows, D, delta);
}
