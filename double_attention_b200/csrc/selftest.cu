// Building-block check for the tensor-core path: one output tile
// D[M=128, N] = A[128, K] * B[N, K]^T computed with TMA-staged operands and
// tcgen05 MMAs, read back from TMEM.  It exercises exactly the pieces the
// route and attention kernels are built from (128-byte swizzled TMA tiles,
// K-major and MN-major shared-memory descriptors, single-CTA and paired
// CTA MMAs, the paired "folded" TMEM accumulator layout) on a case small
// enough to compare element by element.
#include "common.cuh"
#include "host_util.h"

namespace da {
namespace {

// kCG = 1: one CTA owns all 128 rows; TMEM lane = row.
// kCG = 2: a CTA pair; CTA c owns rows [64c, 64c+64) and B rows (or, when B
//          is MN-major, B columns) [c*N/2, (c+1)*N/2).  Each CTA's TMEM holds
//          its 64 rows folded over 128 lanes: lane l = row + 64*h holds
//          columns [h*N/2, (h+1)*N/2).
template <int kCG, int kN, bool kBmn>
__global__ void __launch_bounds__(128) selftest_mma_kernel(const __grid_constant__ CUtensorMap ta,
                                                          const __grid_constant__ CUtensorMap tb,
                                                          int K, float* D, int* status) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  constexpr int kRowsCta = 128 / kCG;           // A rows held by this CTA
  constexpr int kNCta = kN / kCG;               // B rows (or columns) held by this CTA
  const int kblocks = K / 64;
  uint8_t* sA = smem;                           // kblocks x [kRowsCta x 128 B]
  uint8_t* sB = smem + kblocks * kRowsCta * 128;
  __shared__ uint64_t full_bar, done_bar;
  __shared__ uint32_t tmem_base;
  __shared__ int abort_flag;

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const uint32_t rank = (kCG == 2) ? cluster_ctarank() : 0;
  Abort ab{&abort_flag, status};

  if (threadIdx.x == 0) {
    abort_flag = 0;
    mbar_init(&full_bar, 1);
    mbar_init(&done_bar, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc<kCG>(&tmem_base, kCG == 1 ? (kN < 32 ? 32 : kN) : (kN / 2 < 32 ? 32 : kN / 2));
    tmem_relinquish<kCG>();
  }
  tc_fence_before();
  __syncthreads();
  if constexpr (kCG == 2) cluster_sync();
  tc_fence_after();
  const uint32_t tmem = tmem_base;

  // Bytes this CTA loads; the leader expects both CTAs' bytes.
  const uint32_t bytes_cta = kblocks * kRowsCta * 128 + (kBmn ? (kNCta / 64) * K * 128 : kblocks * kNCta * 128);

  if (threadIdx.x == 0) {
    const uint32_t full_addr = kCG == 2 ? mapa_shared(smem_u32(&full_bar), 0) : smem_u32(&full_bar);
    if (rank == 0) mbar_arrive_expect_tx(&full_bar, bytes_cta * kCG);
    for (int kb = 0; kb < kblocks; ++kb) {
      void* dstA = sA + kb * kRowsCta * 128;
      if (kCG == 2) tma_load_2d_pair(&ta, full_addr, dstA, kb * 64, rank * kRowsCta);
      else tma_load_2d(&ta, &full_bar, dstA, kb * 64, 0);
    }
    if (!kBmn) {
      for (int kb = 0; kb < kblocks; ++kb) {
        void* dstB = sB + kb * kNCta * 128;
        if (kCG == 2) tma_load_2d_pair(&tb, full_addr, dstB, kb * 64, rank * kNCta);
        else tma_load_2d(&tb, &full_bar, dstB, kb * 64, 0);
      }
    } else {
      // B stored [K, N]: boxes of [K rows x 64 columns], one per 64 columns.
      for (int nb = 0; nb < kNCta / 64; ++nb) {
        void* dstB = sB + nb * K * 128;
        if (kCG == 2) tma_load_2d_pair(&tb, full_addr, dstB, rank * kNCta + nb * 64, 0);
        else tma_load_2d(&tb, &full_bar, dstB, nb * 64, 0);
      }
    }
  }

  if (rank == 0 && threadIdx.x == 32) {
    if (mbar_wait(&full_bar, 0, ab)) {
      tc_fence_after();
      const uint32_t idesc = idesc_f16(128, kN, true, false, kBmn);
      for (int k = 0; k < K / 16; ++k) {
        const int kb = k / 4, kin = k % 4;
        const uint64_t adesc = sdesc_sw128(smem_u32(sA + kb * kRowsCta * 128) + kin * 32, 16, 1024);
        uint64_t bdesc;
        if (!kBmn) bdesc = sdesc_sw128(smem_u32(sB + kb * kNCta * 128) + kin * 32, 16, 1024);
        else bdesc = sdesc_sw128(smem_u32(sB) + k * 16 * 128, K * 128, 1024);
        mma_f16_ss<kCG>(tmem, adesc, bdesc, idesc, k > 0 ? 1u : 0u);
      }
      mma_commit<kCG>(smem_u32(&done_bar));
      if (kCG == 2) mma_commit<kCG>(mapa_shared(smem_u32(&done_bar), 1));
    }
  }

  // Epilogue: every warp reads its 32 TMEM lanes.
  if (mbar_wait(&done_bar, 0, ab)) {
    tc_fence_after();
    const int lane_id = warp * 32 + lane;
    constexpr int kCols = kCG == 1 ? kN : kN / 2;
    int row, col0;
    if (kCG == 1) { row = lane_id; col0 = 0; }
    else { row = rank * 64 + (lane_id % 64); col0 = (lane_id / 64) * (kN / 2); }
    for (int c = 0; c < kCols; c += 16) {
      float v[16];
      tmem_ld16(tmem + ((uint32_t)(warp * 32) << 16) + c, v);
      tmem_wait_ld();
#pragma unroll
      for (int i = 0; i < 16; ++i) D[row * kN + col0 + c + i] = v[i];
    }
  }
  tc_fence_before();
  __syncthreads();
  if constexpr (kCG == 2) cluster_sync();
  if (warp == 1) tmem_dealloc<kCG>(tmem, kCG == 1 ? (kN < 32 ? 32 : kN) : (kN / 2 < 32 ? 32 : kN / 2));
}

template <int kCG, int kN, bool kBmn>
int launch_selftest(const void* A, const void* B, int K, float* D, int* status, cudaStream_t st) {
  constexpr int kRowsCta = 128 / kCG;
  constexpr int kNCta = kN / kCG;
  CUtensorMap ta, tb;
  int rc = make_tmap_2d(&ta, A, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, K, 128, (uint64_t)K * 2, 64, kRowsCta);
  if (rc) return rc;
  if (!kBmn) rc = make_tmap_2d(&tb, B, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, K, kN, (uint64_t)K * 2, 64, kNCta);
  else rc = make_tmap_2d(&tb, B, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, kN, K, (uint64_t)kN * 2, 64, K);
  if (rc) return rc;
  const int kblocks = K / 64;
  const size_t smem = 1024 + kblocks * kRowsCta * 128 + (kBmn ? (kNCta / 64) * K * 128 : kblocks * kNCta * 128);
  auto kern = selftest_mma_kernel<kCG, kN, kBmn>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return record_cuda_error();
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  cfg.gridDim = dim3(kCG, 1, 1);
  cfg.blockDim = dim3(128, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = kCG;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, kern, ta, tb, K, D, status) != cudaSuccess) return record_cuda_error();
  note_launch();
  return DA_OK;
}

// Failure-detection check: warp 0 waits on a barrier that nothing arrives on,
// bounded by `timeout_ns`; when the wait gives up it records DA_DEV_TIMEOUT
// and `site` in the status words and sets the CTA's abort flag.  Warp 1
// waits on a second barrier that nothing arrives on either, with the regular
// limit, and must leave as soon as the abort flag is set.  Both then return
// normally, so the context stays usable.  (The limits are the only way these
// waits end; the barriers are never signalled.)
__global__ void __launch_bounds__(64) selftest_wait_kernel(unsigned long long timeout_ns, int site, int* status,
                                                           unsigned long long* elapsed_ns) {
  __shared__ uint64_t never_a, never_b;
  __shared__ int abort_flag;
  Abort ab{&abort_flag, status};
  if (threadIdx.x == 0) {
    abort_flag = 0;
    mbar_init(&never_a, 1);
    mbar_init(&never_b, 1);
    fence_mbar_init();
  }
  __syncthreads();
  const unsigned long long t0 = globaltimer();
  bool ok = true;
  if (threadIdx.x == 0) ok = mbar_wait(&never_a, 0, ab, site, timeout_ns);
  if (threadIdx.x == 32) ok = mbar_wait(&never_b, 0, ab, site + 1);
  if (threadIdx.x == 32 && elapsed_ns) elapsed_ns[1] = globaltimer() - t0;
  if (threadIdx.x == 0 && elapsed_ns) elapsed_ns[0] = globaltimer() - t0;
  (void)ok;
}

}  // namespace
}  // namespace da

extern "C" int da_selftest_wait_timeout(int64_t timeout_ns, int site, int* status, uint64_t* elapsed_ns,
                                        void* stream) {
  using namespace da;
  if (!status) return DA_ERR_NULL;
  if (int rc = bind_device(status)) return rc;
  if (timeout_ns <= 0 || timeout_ns > 100000000ll || site <= 0) return DA_ERR_SHAPE;  // at most 0.1 s
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  selftest_wait_kernel<<<1, 64, 0, st>>>(static_cast<unsigned long long>(timeout_ns), site, status,
                                         reinterpret_cast<unsigned long long*>(elapsed_ns));
  if (cudaGetLastError() != cudaSuccess) return record_cuda_error();
  note_launch();
  return DA_OK;
}

extern "C" int da_selftest_mma(int cta_group, int n, int b_mn_major, int k, const void* A, const void* B,
                               float* D, int* status, void* stream) {
  using namespace da;
  if (!A || !B || !D) return DA_ERR_NULL;
  if (int rc = bind_device(A)) return rc;
  if (k <= 0 || k % 64 || k > 256) return DA_ERR_SHAPE;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
#define DA_SELFTEST_CASE(CG, N, MN) \
  if (cta_group == CG && n == N && (b_mn_major != 0) == MN) return launch_selftest<CG, N, MN>(A, B, k, D, status, st);
  DA_SELFTEST_CASE(1, 64, false)
  DA_SELFTEST_CASE(1, 128, false)
  DA_SELFTEST_CASE(1, 256, false)
  DA_SELFTEST_CASE(1, 128, true)
  DA_SELFTEST_CASE(1, 256, true)
  DA_SELFTEST_CASE(2, 64, false)
  DA_SELFTEST_CASE(2, 128, false)
  DA_SELFTEST_CASE(2, 256, false)
  DA_SELFTEST_CASE(2, 128, true)
  DA_SELFTEST_CASE(2, 256, true)
#undef DA_SELFTEST_CASE
  return DA_ERR_UNSUPPORTED;
}
