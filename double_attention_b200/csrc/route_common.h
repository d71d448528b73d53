// Shared declarations of the dictionary-route kernels.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace da {
namespace route {

struct RouteFwdArgs {
  const void* q;            // route input rows: [rows, q_cols] with row stride q_row_stride (elements)
  int64_t rows;             // rows per group
  int64_t q_cols;           // columns of the q matrix
  int64_t q_row_stride;     // elements between consecutive rows
  int groups;               // groups of R columns routed independently (module: 2*H)
  int64_t group_col_stride; // column offset between groups (elements)
  int64_t R, M;
  int dtype;                // DA_F16 / DA_BF16 of q, z and dict_key_t
  const void* dk_t;         // [M, R] normalised keys (dtype)
  const void* dv;           // [R, M] normalised values (bf16)
  const float* beta;        // device scalar
  const float* dk_max;      // device scalar
  float eps;
  int normalize_input, normalize_output;
  void* z;                  // [groups, rows, R]
  float* lse;               // [groups, rows]
  float* out_norm;          // [groups, rows]
  int* argmax;              // [groups, rows] optional
  int* work;                // [2 + repair_cap] persistent, zero-initialised once
  int repair_cap;
  int* status;
};

int route_fwd(const RouteFwdArgs& a, cudaStream_t st);

struct RouteBwdArgs {
  const void* q;            // forward input rows (same addressing as RouteFwdArgs)
  int64_t rows, q_cols, q_row_stride;
  int groups;
  int64_t group_col_stride;
  int64_t R, M;
  int dtype;
  const void* dk_t;         // [M, R] normalised keys (dtype)
  const void* dv_t;         // [M, R] normalised values (bf16)
  const float* beta;
  float eps;
  int normalize_input, normalize_output;
  const void* z;            // [groups, rows, R] forward output (dtype)
  const void* dz;           // [groups, rows, R] its gradient (dtype)
  const float* lse;         // [groups, rows] from the forward
  const float* out_norm;    // [groups, rows] from the forward
  void* dq;                 // gradient of q, layout of q (dtype)
  void* p_out;              // [groups, rows, M] bf16 assignment weights (may be null)
  void* dl_out;             // [groups, rows, M] dtype: invn * beta * dLs (may be null)
  void* g_out;              // [groups, rows, R] bf16 gradient of the reconstruction
  float* dbeta;             // accumulated, may be null
  int* status;
  // [groups, rows_pad, 4] fp32 with rows_pad = rows rounded up to 128 (optional): per row
  // {lse * log2(e), input inverse norm, delta = <P, dP>, 0}; rows past `rows` get {+inf, 0, 0, 0}
  float* row_stats = nullptr;
  float* dbeta_part = nullptr; // [8 * pairs] per-(CTA, warp) dbeta partials, summed in order (optional)
};

int route_bwd(const RouteBwdArgs& a, cudaStream_t st);

// The whole route backward with deterministic dictionary gradients (route_dict_grad.cu): the row pass
// above (dq, g and row_stats into the workspace, no [rows, M] outputs), then the atom-parallel
// dictionary-gradient kernel and the fixed-order reduction of its partial sums.
bool route_bwd_fused_supported(const RouteBwdArgs& a);
int64_t route_bwd_workspace_bytes(int64_t rows, int groups, int64_t R, int64_t M);
int route_bwd_fused(RouteBwdArgs a, void* workspace, int64_t workspace_bytes, float* d_key, float* d_value,
                    float* dbeta, cudaStream_t st);

}  // namespace route
}  // namespace da
