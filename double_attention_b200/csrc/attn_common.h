// Shared declarations of the outer routed-attention kernels.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace da {
namespace attn {

constexpr int kMaxMaps = 4;

// Row addressing of a [rows, R] matrix holding per-(batch, branch) sequences:
//   row(b, branch, t) = base + b * sb + branch * sbr + t
struct RowMap {
  const void* ptr;
  int64_t rows;   // total rows of the matrix
  int64_t base, sb, sbr;
};

struct AttnFwdArgs {
  RowMap q, k;               // routed queries / keys, [rows, R] each, dtype
  const void* v;             // [B, T, D] (dtype)
  int B, T, R, D;
  int maps;                  // S outer maps (1..4)
  int group;                 // branches concatenated per map (H / S when H >= S, else 1)
  int branch0[kMaxMaps];     // first branch of each map
  int causal;
  int dtype;
  const float* scales;       // [maps] gamma_s (device)
  const float* weights;      // [maps] alpha_s (device) or null when maps == 1
  const float* key_norm_max; // [B * maps] upper bound of ||k|| per (b, map), or null -> key_norm_bound
  float key_norm_bound;
  void* y;                   // [B, T, D] output (dtype)
  float* lse;                // [B, maps, T] natural-log sum of exp(gamma_s q.k) per map
  int* status;
  float* part_sum = nullptr;  // key-split workspace (mixed maps, few query tiles), or null: no split
  float* part_o = nullptr;
};

// Key shares per query tile of the mixed-map forward: 2 when the tiles' CTAs (two per pair) fit on the
// SMs at once (the longest tile's chain of score products is then halved), else 1.
inline int key_split(int maps, long pairs, int sms) { return (maps > 1 && 2 * pairs <= sms) ? 2 : 1; }

int attn_fwd(const AttnFwdArgs& a, cudaStream_t st);

}  // namespace attn
}  // namespace da
