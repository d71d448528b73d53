// Column sums of a [rows, cols] bf16 / fp16 matrix in fp32: the bias gradient of a Linear layer
// (d bias = sum over rows of dY) in the block layers around the routed attention (reference
// modules.py:272 output projection, :339-346 feed-forward, :212 value projection, all nn.Linear).
//
// An HBM-bound pass.  First kernel: CTAs tile the matrix by 256-column strips and row chunks; each of
// a CTA's 8 warps walks every 8th row of the chunk with a lane owning 8 consecutive columns (16-byte
// loads), and the 8 warp sums are added in warp order into one fp32 partial row per chunk.  Second
// kernel: each column's partials are added in a fixed order (below).  The partition depends only on the
// shape, so the result is bit-reproducible.
#include "common.cuh"
#include "host_util.h"

namespace da {
namespace colsum {

constexpr int kWarps = 8;
constexpr int kStrip = 256;  // columns per CTA: 32 lanes x 8

template <typename T>
__global__ void __launch_bounds__(kWarps * 32) colsum_partial_kernel(const T* __restrict__ d, int64_t rows,
                                                                     int64_t cols, int64_t ld, int64_t rows_per,
                                                                     float* __restrict__ partial) {
  __shared__ float red[kWarps][kStrip];
  grid_dependency_wait();
  grid_launch_dependents();
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int64_t col = (int64_t)blockIdx.x * kStrip + lane * 8;
  const int64_t r0 = (int64_t)blockIdx.y * rows_per;
  const int64_t r1 = r0 + rows_per < rows ? r0 + rows_per : rows;
  float acc[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) acc[e] = 0.f;
  if (col < cols) {
    for (int64_t r = r0 + w; r < r1; r += kWarps) {
      const uint4 v = *reinterpret_cast<const uint4*>(d + r * ld + col);
      const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = unpack2<T>(u[e]);
        acc[2 * e] += f.x;
        acc[2 * e + 1] += f.y;
      }
    }
  }
#pragma unroll
  for (int e = 0; e < 8; ++e) red[w][lane * 8 + e] = acc[e];
  __syncthreads();
  const int64_t c = (int64_t)blockIdx.x * kStrip + threadIdx.x;
  if (c < cols) {
    float t = 0.f;
#pragma unroll
    for (int k = 0; k < kWarps; ++k) t += red[k][threadIdx.x];
    partial[(int64_t)blockIdx.y * cols + c] = t;
  }
}

// Second kernel: a CTA takes 32 columns; warp w adds chunks w, w + 8, ... of its lane's column in chunk
// order and the 8 warp sums are added in warp order (coalesced 128-byte rows, 16 CTAs for 512 columns).
__global__ void __launch_bounds__(kWarps * 32) colsum_final_kernel(const float* __restrict__ partial, int chunks,
                                                                   int64_t cols, float* __restrict__ out) {
  __shared__ float red[kWarps][32];
  grid_dependency_wait();
  grid_launch_dependents();
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int64_t c = (int64_t)blockIdx.x * 32 + lane;
  float t = 0.f;
  if (c < cols)
    for (int k = w; k < chunks; k += kWarps) t += partial[(int64_t)k * cols + c];
  red[w][lane] = t;
  __syncthreads();
  if (w == 0 && c < cols) {
    float a = 0.f;
#pragma unroll
    for (int k = 0; k < kWarps; ++k) a += red[k][lane];
    out[c] = a;
  }
}

// Row chunks: enough CTAs for about two per SM, each chunk a multiple of the 8 warps' row stride.
inline void plan(int64_t rows, int64_t cols, int* chunks, int64_t* rows_per) {
  const int64_t strips = (cols + kStrip - 1) / kStrip;
  int64_t n = (2 * (int64_t)sm_count() + strips - 1) / strips;
  const int64_t max_chunks = (rows + kWarps - 1) / kWarps;
  if (n > max_chunks) n = max_chunks;
  if (n < 1) n = 1;
  int64_t per = (rows + n - 1) / n;
  per = (per + kWarps - 1) / kWarps * kWarps;
  *rows_per = per;
  *chunks = (int)((rows + per - 1) / per);
}

}  // namespace colsum
}  // namespace da

extern "C" int64_t da_col_sum_workspace_elems(int64_t rows, int64_t cols) {
  if (rows <= 0 || cols <= 0) return -1;
  int chunks;
  int64_t per;
  da::colsum::plan(rows, cols, &chunks, &per);
  return (int64_t)chunks * cols;
}

extern "C" int da_col_sum(const void* d, int64_t rows, int64_t cols, int64_t ld, int dtype, float* out,
                          float* workspace, int64_t workspace_elems, void* stream) {
  using namespace da;
  using namespace da::colsum;
  if (!d || !out || !workspace) return DA_ERR_NULL;
  if (dtype != DA_BF16 && dtype != DA_F16) return DA_ERR_DTYPE;
  if (rows <= 0 || cols <= 0 || ld < cols || cols % 8 || ld % 8) return DA_ERR_SHAPE;
  if ((reinterpret_cast<uintptr_t>(d) & 15) || (reinterpret_cast<uintptr_t>(out) & 3)) return DA_ERR_ALIGN;
  if (int rc = bind_device(d)) return rc;
  int chunks;
  int64_t per;
  plan(rows, cols, &chunks, &per);
  if (workspace_elems < (int64_t)chunks * cols) return DA_ERR_WORKSPACE;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const dim3 grid((unsigned)((cols + kStrip - 1) / kStrip), (unsigned)chunks);
  int rc = dtype == DA_BF16
               ? launch_kernel(colsum_partial_kernel<__nv_bfloat16>, grid, dim3(kWarps * 32), 0, st, false,
                               static_cast<const __nv_bfloat16*>(d), rows, cols, ld, per, workspace)
               : launch_kernel(colsum_partial_kernel<__half>, grid, dim3(kWarps * 32), 0, st, false,
                               static_cast<const __half*>(d), rows, cols, ld, per, workspace);
  if (rc) return rc;
  return launch_kernel(colsum_final_kernel, dim3((unsigned)((cols + 31) / 32)), dim3(kWarps * 32), 0, st, false,
                       (const float*)workspace, chunks, cols, out);
}
