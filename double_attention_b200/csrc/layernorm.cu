// Residual add + LayerNorm around the double-attention block, forward and backward.
//
// Reference: the pre-norm block of DoubleAttentionBlock (modules.py:294-356) and the final norm of
// DoubleAttentionLM (modules.py:415-460):
//   x_out = x + branch            (fp32 residual stream; the branch is the attention or FFN output)
//   y     = LayerNorm(x_out) * gamma + beta      (nn.LayerNorm, biased variance, eps)
// Under autocast the reference computes LayerNorm in fp32 and the next Linear casts y to bf16; here y
// is written directly in the dtype its consumer reads, from the same fp32 values.
//
// Backward, with x_hat = (x_out - mean) * rstd and g = dy * gamma:
//   dx_out = d_res + rstd * (g - mean(g) - x_hat * mean(g * x_hat))
//   d branch = dx_out (in the branch's dtype), d x = dx_out
//   d gamma = sum_rows dy * x_hat,  d beta = sum_rows dy
// Both directions are HBM-bound row passes: one warp per row, each lane owning 8-element column
// chunks (coalesced 16-/32-byte accesses), the row's values kept in registers between the two
// reductions.  Measured at 262144 rows x 512 (one B200, L2 flushed): the forward moves 1.61 GB in
// 256 us (97 % of the measured copy bandwidth); the backward 2.15 GB in 424 us (78 %) with all of a
// row's loads issued before its first store (501 us with the residual gradient loaded after the
// reductions; issuing the forward's loads that way cost it occupancy and 28 % more time).  The column sums of the backward are accumulated per block in registers and shared
// memory, written as [blocks, 2, D] partials, and summed by a second small kernel (deterministic).
#include "common.cuh"
#include "host_util.h"

namespace da {
namespace {

constexpr int kLnWarps = 8;  // rows in flight per block

DA_DEV void load8(const void* p, int dtype, size_t off, float* v) {
  if (dtype == DA_F32) {
    const float4* s = reinterpret_cast<const float4*>(static_cast<const float*>(p) + off);
    const float4 a = s[0], b = s[1];
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  } else {
    const uint4 w = *reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(p) + off);
    const uint32_t u[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = dtype == DA_BF16 ? unpack2<__nv_bfloat16>(u[e]) : unpack2<__half>(u[e]);
      v[2 * e] = f.x;
      v[2 * e + 1] = f.y;
    }
  }
}

DA_DEV void store8(void* p, int dtype, size_t off, const float* v) {
  if (dtype == DA_F32) {
    float4* d = reinterpret_cast<float4*>(static_cast<float*>(p) + off);
    d[0] = make_float4(v[0], v[1], v[2], v[3]);
    d[1] = make_float4(v[4], v[5], v[6], v[7]);
  } else {
    uint32_t u[4];
#pragma unroll
    for (int e = 0; e < 4; ++e)
      u[e] = dtype == DA_BF16 ? pack2<__nv_bfloat16>(v[2 * e], v[2 * e + 1]) : pack2<__half>(v[2 * e], v[2 * e + 1]);
    *reinterpret_cast<uint4*>(static_cast<uint16_t*>(p) + off) = make_uint4(u[0], u[1], u[2], u[3]);
  }
}

DA_DEV float warp_sum(float v) {
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// kNV: 256-column chunks per row (D = 256 * kNV); lane l owns columns c * 256 + 8 l .. + 8.
template <int kNV>
__global__ void __launch_bounds__(kLnWarps * 32) add_ln_fwd_kernel(const float* __restrict__ x, const void* branch,
                                                                   int branch_dtype, const float* __restrict__ gamma,
                                                                   const float* __restrict__ beta, int64_t rows,
                                                                   float eps, float* x_out, void* y, int y_dtype,
                                                                   float* __restrict__ mean_out,
                                                                   float* __restrict__ rstd_out) {
  constexpr int D = 256 * kNV;
  grid_dependency_wait();
  grid_launch_dependents();
  const int lane = threadIdx.x & 31;
  const int64_t stride = (int64_t)gridDim.x * kLnWarps;
  for (int64_t row = (int64_t)blockIdx.x * kLnWarps + threadIdx.x / 32; row < rows; row += stride) {
    float v[kNV][8];
    float s = 0.f;
#pragma unroll
    for (int c = 0; c < kNV; ++c) {
      const size_t off = (size_t)row * D + c * 256 + lane * 8;
      load8(x, DA_F32, off, v[c]);
      if (branch) {
        float b[8];
        load8(branch, branch_dtype, off, b);
#pragma unroll
        for (int e = 0; e < 8; ++e) v[c][e] += b[e];
        store8(x_out, DA_F32, off, v[c]);
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) s += v[c][e];
    }
    const float mean = warp_sum(s) * (1.f / D);
    float q = 0.f;
#pragma unroll
    for (int c = 0; c < kNV; ++c)
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float d = v[c][e] - mean;
        q = fmaf(d, d, q);
      }
    const float rstd = rsqrtf(warp_sum(q) * (1.f / D) + eps);
#pragma unroll
    for (int c = 0; c < kNV; ++c) {
      const int col = c * 256 + lane * 8;
      const float4 g0 = *reinterpret_cast<const float4*>(gamma + col), g1 = *reinterpret_cast<const float4*>(gamma + col + 4);
      const float4 b0 = *reinterpret_cast<const float4*>(beta + col), b1 = *reinterpret_cast<const float4*>(beta + col + 4);
      const float g[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
      const float bb[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
      float o[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) o[e] = fmaf((v[c][e] - mean) * rstd, g[e], bb[e]);
      store8(y, y_dtype, (size_t)row * D + col, o);
    }
    if (lane == 0) {
      mean_out[row] = mean;
      rstd_out[row] = rstd;
    }
  }
}

template <int kNV>
__global__ void __launch_bounds__(kLnWarps * 32) add_ln_bwd_kernel(const void* dy, int dy_dtype, const float* d_res,
                                                                   const float* __restrict__ x_out,
                                                                   const float* __restrict__ mean_in,
                                                                   const float* __restrict__ rstd_in,
                                                                   const float* __restrict__ gamma, int64_t rows,
                                                                   float* dx, void* d_branch, int branch_dtype,
                                                                   float* __restrict__ partial) {
  constexpr int D = 256 * kNV;
  __shared__ float red[kLnWarps][2][32 * 8];
  grid_dependency_wait();
  grid_launch_dependents();
  const int lane = threadIdx.x & 31, w = threadIdx.x / 32;
  const int64_t stride = (int64_t)gridDim.x * kLnWarps;
  float acc_g[kNV][8], acc_b[kNV][8];  // this lane's columns: sum dy * x_hat, sum dy
#pragma unroll
  for (int c = 0; c < kNV; ++c)
#pragma unroll
    for (int e = 0; e < 8; ++e) acc_g[c][e] = acc_b[c][e] = 0.f;
  for (int64_t row = (int64_t)blockIdx.x * kLnWarps + w; row < rows; row += stride) {
    const float mean = mean_in[row], rstd = rstd_in[row];
    // every load of the row is issued before the first store (dx may alias d_res); for widths up to 512
    // the residual gradient is loaded here too, so the row's bytes are in flight together
    constexpr bool kEarly = kNV <= 2;
    float xh[kNV][8], gd[kNV][8], dd[kNV][8], rr[kEarly ? kNV : 1][8];
#pragma unroll
    for (int c = 0; c < kNV; ++c) {
      const size_t off = (size_t)row * D + c * 256 + lane * 8;
      load8(dy, dy_dtype, off, dd[c]);
      load8(x_out, DA_F32, off, xh[c]);
      if (kEarly && d_res) load8(d_res, DA_F32, off, rr[kEarly ? c : 0]);
    }
    float s1 = 0.f, s2 = 0.f;
#pragma unroll
    for (int c = 0; c < kNV; ++c) {
      const int col = c * 256 + lane * 8;
      const float* d = dd[c];
      const float4 g0 = *reinterpret_cast<const float4*>(gamma + col), g1 = *reinterpret_cast<const float4*>(gamma + col + 4);
      const float g[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        xh[c][e] = (xh[c][e] - mean) * rstd;
        gd[c][e] = d[e] * g[e];
        s1 += gd[c][e];
        s2 = fmaf(gd[c][e], xh[c][e], s2);
        acc_g[c][e] = fmaf(d[e], xh[c][e], acc_g[c][e]);
        acc_b[c][e] += d[e];
      }
    }
    const float m1 = warp_sum(s1) * (1.f / D), m2 = warp_sum(s2) * (1.f / D);
#pragma unroll
    for (int c = 0; c < kNV; ++c) {
      const size_t off = (size_t)row * D + c * 256 + lane * 8;
      float o[8];
      if (d_res && kEarly) {
#pragma unroll
        for (int e = 0; e < 8; ++e) o[e] = rr[kEarly ? c : 0][e];
      } else if (d_res) {
        load8(d_res, DA_F32, off, o);
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) o[e] = 0.f;
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) o[e] += rstd * (gd[c][e] - m1 - xh[c][e] * m2);
      store8(dx, DA_F32, off, o);
      if (d_branch) store8(d_branch, branch_dtype, off, o);
    }
  }
  // block column sums, one 256-column chunk at a time through shared memory
#pragma unroll
  for (int c = 0; c < kNV; ++c) {
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      red[w][0][lane * 8 + e] = acc_g[c][e];
      red[w][1][lane * 8 + e] = acc_b[c][e];
    }
    __syncthreads();
    for (int i = threadIdx.x; i < 2 * 256; i += blockDim.x) {
      const int which = i / 256, col = i % 256;
      float t = 0.f;
#pragma unroll
      for (int k = 0; k < kLnWarps; ++k) t += red[k][which][col];
      partial[((size_t)blockIdx.x * 2 + which) * D + c * 256 + col] = t;
    }
    __syncthreads();
  }
}

// d gamma, d beta: sums of the [blocks, 2, D] partials over blocks.  One CTA per 32 output columns
// of the 2 x D outputs: its 8 warps split the block range (lane = column, coalesced rows), then the
// 8 partial sums are added in a fixed order (deterministic).
__global__ void __launch_bounds__(256) ln_partial_sum_kernel(const float* __restrict__ partial, int blocks, int D,
                                                             float* __restrict__ dgamma, float* __restrict__ dbeta) {
  __shared__ float red[8][32];
  grid_dependency_wait();
  grid_launch_dependents();
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int i = blockIdx.x * 32 + lane;  // output index in [0, 2 D)
  const int which = i / D, col = i % D;
  float t = 0.f;
  if (i < 2 * D)
    for (int k = w; k < blocks; k += 8) t += partial[((size_t)k * 2 + which) * D + col];
  red[w][lane] = t;
  __syncthreads();
  if (w == 0 && i < 2 * D) {
    float s = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) s += red[k][lane];
    float* out = which == 0 ? dgamma : dbeta;
    if (out) out[col] = s;
  }
}

inline int ln_blocks(int64_t rows) {
  const int64_t need = (rows + kLnWarps - 1) / kLnWarps;
  const int64_t cap = 4LL * sm_count();
  return (int)(need < cap ? (need > 0 ? need : 1) : cap);
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace
}  // namespace da

extern "C" int da_layernorm_bwd_blocks(int64_t rows) { return da::ln_blocks(rows); }

extern "C" int da_add_layernorm_fwd(const float* x, const void* branch, int branch_dtype, const float* gamma,
                                    const float* beta, int64_t rows, int64_t D, float eps, float* x_out, void* y,
                                    int y_dtype, float* mean, float* rstd, void* stream) {
  using namespace da;
  if (!x || !gamma || !beta || !y || !mean || !rstd || (branch && !x_out)) return DA_ERR_NULL;
  if (rows <= 0 || (D != 256 && D != 512 && D != 768 && D != 1024)) return DA_ERR_SHAPE;
  if (y_dtype < DA_F16 || y_dtype > DA_F32 || (branch && (branch_dtype < DA_F16 || branch_dtype > DA_F32)))
    return DA_ERR_DTYPE;
  if (!aligned16(x) || !aligned16(gamma) || !aligned16(beta) || !aligned16(y) || (branch && !aligned16(branch)) ||
      (x_out && !aligned16(x_out)))
    return DA_ERR_ALIGN;
  if (int rc = bind_device(x)) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const dim3 grid((unsigned)ln_blocks(rows)), block(kLnWarps * 32);
  switch (D) {
    case 256: return launch_kernel(add_ln_fwd_kernel<1>, grid, block, 0, st, false, x, branch, branch_dtype, gamma, beta, rows, eps, x_out, y, y_dtype, mean, rstd);
    case 512: return launch_kernel(add_ln_fwd_kernel<2>, grid, block, 0, st, false, x, branch, branch_dtype, gamma, beta, rows, eps, x_out, y, y_dtype, mean, rstd);
    case 768: return launch_kernel(add_ln_fwd_kernel<3>, grid, block, 0, st, false, x, branch, branch_dtype, gamma, beta, rows, eps, x_out, y, y_dtype, mean, rstd);
    default: return launch_kernel(add_ln_fwd_kernel<4>, grid, block, 0, st, false, x, branch, branch_dtype, gamma, beta, rows, eps, x_out, y, y_dtype, mean, rstd);
  }
}

extern "C" int da_add_layernorm_bwd(const void* dy, int dy_dtype, const float* d_res, const float* x_out,
                                    const float* mean, const float* rstd, const float* gamma, int64_t rows, int64_t D,
                                    float* dx, void* d_branch, int branch_dtype, float* partial, int partial_blocks,
                                    float* dgamma, float* dbeta, void* stream) {
  using namespace da;
  if (!dy || !x_out || !mean || !rstd || !gamma || !dx || !partial) return DA_ERR_NULL;
  if (rows <= 0 || (D != 256 && D != 512 && D != 768 && D != 1024)) return DA_ERR_SHAPE;
  if (dy_dtype < DA_F16 || dy_dtype > DA_F32 || (d_branch && (branch_dtype < DA_F16 || branch_dtype > DA_F32)))
    return DA_ERR_DTYPE;
  if (partial_blocks != ln_blocks(rows)) return DA_ERR_WORKSPACE;
  if (!aligned16(dy) || !aligned16(x_out) || !aligned16(gamma) || !aligned16(dx) || (d_res && !aligned16(d_res)) ||
      (d_branch && !aligned16(d_branch)))
    return DA_ERR_ALIGN;
  if (int rc = bind_device(dy)) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const dim3 grid((unsigned)partial_blocks), block(kLnWarps * 32);
  int rc;
  switch (D) {
    case 256: rc = launch_kernel(add_ln_bwd_kernel<1>, grid, block, 0, st, false, dy, dy_dtype, d_res, x_out, mean, rstd, gamma, rows, dx, d_branch, branch_dtype, partial); break;
    case 512: rc = launch_kernel(add_ln_bwd_kernel<2>, grid, block, 0, st, false, dy, dy_dtype, d_res, x_out, mean, rstd, gamma, rows, dx, d_branch, branch_dtype, partial); break;
    case 768: rc = launch_kernel(add_ln_bwd_kernel<3>, grid, block, 0, st, false, dy, dy_dtype, d_res, x_out, mean, rstd, gamma, rows, dx, d_branch, branch_dtype, partial); break;
    default: rc = launch_kernel(add_ln_bwd_kernel<4>, grid, block, 0, st, false, dy, dy_dtype, d_res, x_out, mean, rstd, gamma, rows, dx, d_branch, branch_dtype, partial); break;
  }
  if (rc) return rc;
  if (!dgamma && !dbeta) return DA_OK;
  const int n = 2 * (int)D;
  return launch_kernel(ln_partial_sum_kernel, dim3((unsigned)((n + 31) / 32)), dim3(256), 0, st, false,
                       (const float*)partial, partial_blocks, (int)D, dgamma, dbeta);
}
