// Host-side helpers shared by the C-ABI entry points: status codes, the
// thread-local record of the last CUDA error, and TMA descriptor creation
// through the driver entry point (so the library does not link libcuda).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/da_b200.h"

namespace da {

// Records the pending CUDA runtime error (clearing it) and returns DA_ERR_CUDA.
int record_cuda_error();
// Records an explicit CUDA error code and returns DA_ERR_CUDA.
int record_cuda_error_code(int code);

// Encodes a 2-D tiled tensor map over a row-major matrix [outer, inner]
// with the given row stride, a box of [box_outer, box_inner] elements and
// 128-byte swizzling (box_inner * elem_bytes must be 128) unless
// `swizzle128` is false.  Returns DA_OK or a DA_ERR_* status.
int make_tmap_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, int elem_bytes,
                 uint64_t inner, uint64_t outer, uint64_t row_stride_bytes, uint32_t box_inner,
                 uint32_t box_outer, bool swizzle128 = true);

// Encodes a tiled tensor map of rank 3..5 with 128-byte swizzling whose box is
// 128 bytes wide in the innermost dimension (box[0] = 128 / elem_bytes);
// strides_bytes[i] is the byte stride of dims[i + 1] in any order, so a
// dimension may step across 64-column blocks of the same rows (dims[0] = 64)
// or across row groups, and one box gathers several [box[1] x 128 B] blocks,
// each laid out in shared memory exactly like a separate 2-D box.  Returns
// DA_OK or a DA_ERR_* status.
int make_tmap_blocks(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, int elem_bytes, int rank,
                     const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box);

// Optional debug progress buffer (pinned host memory) set by
// da_set_debug_trace; kernels that support it write per-CTA markers there.
int* debug_trace();

// Makes the primary context of the device owning `ptr` current on the
// calling thread (autograd runs backward on its own threads, where the
// runtime this library links may not have a context yet).  Returns DA_OK
// or DA_ERR_CUDA.
int bind_device(const void* ptr);

// Number of SMs of the current device (cached per device).
int sm_count();

// Count one kernel launched by this library (process-wide counter).
void note_launch();

// Launch with programmatic dependent launch allowed (the kernel waits for its
// predecessors with griddepcontrol.wait) and, when `pair` is set, as 2-CTA
// clusters.
template <typename... KArgs, typename... Args>
int launch_kernel(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, bool pair,
                  Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[2];
  int n = 0;
  attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[n].val.programmaticStreamSerializationAllowed = 1;
  ++n;
  if (pair) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = 2;
    attr[n].val.clusterDim.y = 1;
    attr[n].val.clusterDim.z = 1;
    ++n;
  }
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = n;
  if (cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...) != cudaSuccess) return record_cuda_error();
  note_launch();
  return DA_OK;
}

}  // namespace da
