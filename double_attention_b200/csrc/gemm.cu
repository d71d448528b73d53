// Dense GEMM on tcgen05: C[M, N] (+)= sum_k A(m, k) B(n, k).
//
// Used for the fused Q/K projection of SharedDictionaryAttention
// (modules.py:143-157: x . cat(W_q, W_k)^T) and for its backward (dX = dC W,
// dW = dC^T X).  A and B are each either K-major (row-major [M, K] /
// [N, K]) or MN-major (row-major [K, M] / [K, N]); both layouts are staged
// by TMA into 128-byte swizzled tiles that the tensor core reads directly.
// One CTA computes a 128 x kN tile, streaming K in 64-wide stages through a
// kStages-deep TMA -> MMA pipeline, accumulating in TMEM; four epilogue
// warps read the accumulator back (one row per thread) and store it.
#include "common.cuh"
#include "host_util.h"

namespace da {
namespace gemm {

constexpr int kBM = 128;
constexpr int kBK = 64;
constexpr int kThreads = 192;  // warp0 TMA, warp1 MMA, warps2-5 epilogue

template <int kN>
struct Cfg {
  static constexpr int kABytes = kBM * kBK * 2;
  static constexpr int kBBytes = kN * kBK * 2;
  static constexpr int kStages = kN == 256 ? 4 : 6;
  static constexpr int kSmem = kStages * (kABytes + kBBytes);
};

// The segmented GEMM runs two CTAs per SM: one CTA's product (a chain of dependent K = 16 instructions
// into its TMEM accumulator) interleaves in the tensor pipe with the other's, and each CTA's epilogue
// overlaps the other's K loop.  Two 48 KB stages each (128 x 256 tiles), 256 TMEM columns each.
template <int kN>
struct SegCfg {
  static constexpr int kABytes = kBM * kBK * 2;
  static constexpr int kBBytes = kN * kBK * 2;
  static constexpr int kStages = kN == 256 ? 2 : 3;
  static constexpr int kSmem = kStages * (kABytes + kBBytes);
};

struct Params {
  int M, N, K;
  void* c;
  int64_t ldc;
  int out_f32;     // C is fp32 (else the input dtype)
  int accumulate;  // C += A.B (else C = A.B)
  int* status;
  int kps;         // K stages per split (split-K when gridDim.z > 1), 0 = all
  // grouped K (MN-major A only): K stage kb belongs to group kb / kseg, whose A columns start
  // a_goff further right and whose A rows restart at 0; 0 = one group
  int kseg = 0, a_goff = 0, a_inner = 0;
  // split-K partial sums: with `partial` set every split stores its [M, N] partial (dense, row stride N) at
  // partial + split * M * N and splitk_reduce_kernel adds them in split order (deterministic); null: each
  // split adds its partial into C with fp32 atomics (order-dependent rounding)
  float* partial = nullptr;
  // a second K segment: K stages kb >= nk1 come from the second pair of tensor maps (C = A.B^T + A2.B2^T);
  // nk1 = 0: one segment
  int nk1 = 0;
  // epilogue of the operand-dtype output: + bias[n] (operand dtype, or null), then act 1: GELU (the
  // pre-activation also stored in aux when aux is set), act 2: times GELU'(aux[m, n]); aux [M, N] with row
  // stride ldaux in the operand dtype
  const void* bias = nullptr;
  int act = 0;
  void* aux = nullptr;
  int64_t ldaux = 0;
};

// GELU with the exact erf form (nn.GELU's default) and its derivative.
DA_DEV float gelu_f(float z) { return 0.5f * z * (1.f + erff(z * 0.70710678118654752f)); }
DA_DEV float gelu_grad_f(float z) {
  return 0.5f * (1.f + erff(z * 0.70710678118654752f)) + z * 0.39894228040143268f * expf(-0.5f * z * z);
}

template <typename T, int kN, bool kAmn, bool kBmn>
__global__ void __launch_bounds__(kThreads, 1) gemm_kernel(const __grid_constant__ CUtensorMap ta,
                                                           const __grid_constant__ CUtensorMap tb,
                                                           const __grid_constant__ CUtensorMap ta2,
                                                           const __grid_constant__ CUtensorMap tb2, const Params p) {
  using C = Cfg<kN>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ uint64_t full[C::kStages], empty[C::kStages], done;
  __shared__ uint32_t tmem_base;
  __shared__ int abort_flag;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int m0 = blockIdx.x * kBM, n0 = blockIdx.y * kN;
  const int nk_all = p.nk1 ? p.nk1 + (p.K - p.nk1 * kBK + kBK - 1) / kBK  // two segments (K = K1 + K2)
                           : (p.K + kBK - 1) / kBK;  // TMA zero-fills the ragged last K stage
  // split-K: this CTA reduces K stages [kb0, kb0 + nk) and adds its partial sum atomically
  const bool split = gridDim.z > 1;
  const int kb0 = split ? (int)blockIdx.z * p.kps : 0;
  const int nk = split ? min(p.kps, nk_all - kb0) : nk_all;  // >= 1 (the host sizes the splits)
  Abort ab{&abort_flag, p.status};

  if (threadIdx.x == 0) {
    abort_flag = 0;
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(&done, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc<1>(&tmem_base, kN);
    tmem_relinquish<1>();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  grid_dependency_wait();  // predecessors' outputs are visible from here on
  grid_launch_dependents();
  const uint32_t tmem = tmem_base;

  if (warp == 0) {
    if (lane == 0) {
      prefetch_tmap(&ta);
      prefetch_tmap(&tb);
      if (p.nk1) {
        prefetch_tmap(&ta2);
        prefetch_tmap(&tb2);
      }
      int issued = 0;
      for (int kb = 0; kb < nk; ++kb) {
        const int s = kb % C::kStages;
        if (!mbar_wait(&empty[s], ((kb / C::kStages) & 1u) ^ 1u, ab, 41)) break;
        mbar_arrive_expect_tx(&full[s], C::kABytes + C::kBBytes);
        uint8_t* sa = smem + s * (C::kABytes + C::kBBytes);
        uint8_t* sb = sa + C::kABytes;
        const bool second = p.nk1 && kb0 + kb >= p.nk1;
        const CUtensorMap* tA = second ? &ta2 : &ta;
        const CUtensorMap* tB = second ? &tb2 : &tb;
        const int kk = second ? kb0 + kb - p.nk1 : kb0 + kb;  // K stage inside its segment
        if (!kAmn) {
          tma_load_2d(tA, &full[s], sa, kk * kBK, m0);
        } else {
          const int grp = p.kseg ? kk / p.kseg : 0;
          const int ax = m0 + grp * p.a_goff, ay = (kk - grp * p.kseg) * kBK;
          tma_load_2d(tA, &full[s], sa, ax, ay);
          tma_load_2d(tA, &full[s], sa + kBK * 128, ax + 64, ay);
        }
        if (!kBmn) {
          tma_load_2d(tB, &full[s], sb, kk * kBK, n0);
        } else {
          for (int i = 0; i < kN / 64; ++i)
            tma_load_2d(tB, &full[s], sb + i * kBK * 128, n0 + i * 64, kk * kBK);
        }
        issued = kb + 1;
      }
      for (int kb = (issued > C::kStages ? issued - C::kStages : 0); kb < issued; ++kb)
        mbar_wait_drain(&full[kb % C::kStages], (kb / C::kStages) & 1u);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = idesc_f16(kBM, kN, std::is_same<T, __nv_bfloat16>::value, kAmn, kBmn);
      bool ok = true;
      for (int kb = 0; ok && kb < nk; ++kb) {
        const int s = kb % C::kStages;
        ok = mbar_wait(&full[s], (kb / C::kStages) & 1u, ab, 42);
        if (!ok) break;
        tc_fence_after();
        const uint32_t sa = smem_u32(smem + s * (C::kABytes + C::kBBytes));
        const uint32_t sb = sa + C::kABytes;
#pragma unroll
        for (int k = 0; k < kBK / 16; ++k) {
          const uint64_t ad = kAmn ? sdesc_sw128(sa + k * 16 * 128, kBK * 128, 1024)
                                   : sdesc_sw128(sa + k * 32, 16, 1024);
          const uint64_t bd = kBmn ? sdesc_sw128(sb + k * 16 * 128, kBK * 128, 1024)
                                   : sdesc_sw128(sb + k * 32, 16, 1024);
          mma_f16_ss<1>(tmem, ad, bd, idesc, (kb > 0 || k > 0) ? 1u : 0u);
        }
        mma_commit<1>(smem_u32(&empty[s]));
      }
      mma_commit<1>(smem_u32(&done));
      mbar_wait_drain(&done, 0);
    }
  } else {
    const int quad = warp & 3;
    const int row = m0 + quad * 32 + lane;
    bool ok = mbar_wait(&done, 0, ab, 43);
    ok = __all_sync(0xffffffffu, ok);
    tc_fence_after();
    if (ok) {
      const bool live = row < p.M;
      for (int c = 0; c < kN; c += 32) {
        float v[32];
        tmem_ld32(tmem + ((uint32_t)(quad * 32) << 16) + c, v);
        tmem_wait_ld();
        if (!live || n0 + c >= p.N) continue;
        if (split && p.partial) {
          float4* dst = reinterpret_cast<float4*>(p.partial + ((size_t)blockIdx.z * p.M + row) * p.N + n0 + c);
#pragma unroll
          for (int e = 0; e < 8; ++e) dst[e] = make_float4(v[4 * e], v[4 * e + 1], v[4 * e + 2], v[4 * e + 3]);
        } else if (split) {
          float4* dst = reinterpret_cast<float4*>(reinterpret_cast<float*>(p.c) + (size_t)row * p.ldc + n0 + c);
#pragma unroll
          for (int e = 0; e < 8; ++e) atomicAdd(dst + e, make_float4(v[4 * e], v[4 * e + 1], v[4 * e + 2], v[4 * e + 3]));
        } else if (p.out_f32) {
          float* dst = reinterpret_cast<float*>(p.c) + (size_t)row * p.ldc + n0 + c;
#pragma unroll
          for (int e = 0; e < 32; e += 4) {
            float4 w = make_float4(v[e], v[e + 1], v[e + 2], v[e + 3]);
            if (p.accumulate) {
              const float4 o = *reinterpret_cast<float4*>(dst + e);
              w.x += o.x; w.y += o.y; w.z += o.z; w.w += o.w;
            }
            *reinterpret_cast<float4*>(dst + e) = w;
          }
        } else {
          T* dst = reinterpret_cast<T*>(p.c) + (size_t)row * p.ldc + n0 + c;
          if (p.bias) {
            const uint4* b4 = reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(p.bias) + n0 + c);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const uint4 bv = __ldg(b4 + e);
              const uint32_t bw[4] = {bv.x, bv.y, bv.z, bv.w};
#pragma unroll
              for (int h = 0; h < 4; ++h) {
                const float2 f = unpack2<T>(bw[h]);
                v[8 * e + 2 * h] += f.x;
                v[8 * e + 2 * h + 1] += f.y;
              }
            }
          }
          if (p.act == 1) {  // GELU; the pre-activation (rounded as stored) kept for the backward
            if (p.aux) {
              T* za = reinterpret_cast<T*>(p.aux) + (size_t)row * p.ldaux + n0 + c;
              uint32_t zw[16];
#pragma unroll
              for (int e = 0; e < 16; ++e) zw[e] = pack2<T>(v[2 * e], v[2 * e + 1]);
#pragma unroll
              for (int e = 0; e < 4; ++e)
                reinterpret_cast<uint4*>(za)[e] = make_uint4(zw[4 * e], zw[4 * e + 1], zw[4 * e + 2], zw[4 * e + 3]);
            }
#pragma unroll
            for (int e = 0; e < 32; ++e) v[e] = gelu_f(v[e]);
          } else if (p.act == 2) {  // times GELU' of the stored pre-activation
            const uint4* z4 = reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(p.aux) + (size_t)row * p.ldaux + n0 + c);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const uint4 zv = z4[e];
              const uint32_t zw[4] = {zv.x, zv.y, zv.z, zv.w};
#pragma unroll
              for (int h = 0; h < 4; ++h) {
                const float2 f = unpack2<T>(zw[h]);
                v[8 * e + 2 * h] *= gelu_grad_f(f.x);
                v[8 * e + 2 * h + 1] *= gelu_grad_f(f.y);
              }
            }
          }
          uint32_t w[16];
#pragma unroll
          for (int e = 0; e < 16; ++e) w[e] = pack2<T>(v[2 * e], v[2 * e + 1]);
#pragma unroll
          for (int e = 0; e < 4; ++e)
            reinterpret_cast<uint4*>(dst)[e] = make_uint4(w[4 * e], w[4 * e + 1], w[4 * e + 2], w[4 * e + 3]);
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc<1>(tmem, kN);
}

// Several GEMMs that share the A operand, one launch: output columns are
// split into segments, each with its own weight matrix B_s [N_s, K] (K-major),
// output C_s (its own leading dimension and dtype) and optional bias.  Used for
// the Q, K and V projections of one input (modules.py:143-157 and the value
// projection): x is read once and V is written directly in the bf16 the
// attention's P.V product reads.  Every segment width is a multiple of kN, so
// a CTA's tile lies inside one segment.
constexpr int kMaxSeg = 3;

struct SegParams {
  int M, K, nseg;
  int seg_n0[kMaxSeg + 1];  // first global column of each segment; seg_n0[nseg] = total columns
  void* c[kMaxSeg];
  int64_t ldc[kMaxSeg];
  int out_dtype[kMaxSeg];   // DA_F16 / DA_BF16 / DA_F32
  const void* bias[kMaxSeg];  // [N_s] in the operand dtype, or null
  int* status;
};

template <typename T, int kN>
__global__ void __launch_bounds__(kThreads, 2) gemm_seg_kernel(const __grid_constant__ CUtensorMap ta,
                                                               const __grid_constant__ CUtensorMap tb0,
                                                               const __grid_constant__ CUtensorMap tb1,
                                                               const __grid_constant__ CUtensorMap tb2,
                                                               const SegParams p) {
  using C = SegCfg<kN>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ uint64_t full[C::kStages], empty[C::kStages], done;
  __shared__ uint32_t tmem_base;
  __shared__ int abort_flag;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int m0 = blockIdx.x * kBM, gn0 = blockIdx.y * kN;
  int seg = 0;
  while (seg + 1 < p.nseg && gn0 >= p.seg_n0[seg + 1]) ++seg;
  const int n0 = gn0 - p.seg_n0[seg];  // column inside the segment
  const CUtensorMap* tb = seg == 0 ? &tb0 : (seg == 1 ? &tb1 : &tb2);
  const int nk = (p.K + kBK - 1) / kBK;
  Abort ab{&abort_flag, p.status};

  if (threadIdx.x == 0) {
    abort_flag = 0;
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(&done, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc<1>(&tmem_base, kN);
    tmem_relinquish<1>();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  grid_dependency_wait();  // predecessors' outputs are visible from here on
  grid_launch_dependents();
  const uint32_t tmem = tmem_base;

  if (warp == 0) {
    if (lane == 0) {
      prefetch_tmap(&ta);
      prefetch_tmap(tb);
      int issued = 0;
      for (int kb = 0; kb < nk; ++kb) {
        const int s = kb % C::kStages;
        if (!mbar_wait(&empty[s], ((kb / C::kStages) & 1u) ^ 1u, ab, 41)) break;
        mbar_arrive_expect_tx(&full[s], C::kABytes + C::kBBytes);
        uint8_t* sa = smem + s * (C::kABytes + C::kBBytes);
        tma_load_2d(&ta, &full[s], sa, kb * kBK, m0);
        tma_load_2d(tb, &full[s], sa + C::kABytes, kb * kBK, n0);
        issued = kb + 1;
      }
      for (int kb = (issued > C::kStages ? issued - C::kStages : 0); kb < issued; ++kb)
        mbar_wait_drain(&full[kb % C::kStages], (kb / C::kStages) & 1u);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = idesc_f16(kBM, kN, std::is_same<T, __nv_bfloat16>::value, false, false);
      bool ok = true;
      for (int kb = 0; ok && kb < nk; ++kb) {
        const int s = kb % C::kStages;
        ok = mbar_wait(&full[s], (kb / C::kStages) & 1u, ab, 42);
        if (!ok) break;
        tc_fence_after();
        const uint32_t sa = smem_u32(smem + s * (C::kABytes + C::kBBytes));
        const uint32_t sb = sa + C::kABytes;
#pragma unroll
        for (int k = 0; k < kBK / 16; ++k)
          mma_f16_ss<1>(tmem, sdesc_sw128(sa + k * 32, 16, 1024), sdesc_sw128(sb + k * 32, 16, 1024), idesc,
                        (kb > 0 || k > 0) ? 1u : 0u);
        mma_commit<1>(smem_u32(&empty[s]));
      }
      mma_commit<1>(smem_u32(&done));
      mbar_wait_drain(&done, 0);
    }
  } else {
    const int quad = warp & 3;
    const int row = m0 + quad * 32 + lane;
    bool ok = mbar_wait(&done, 0, ab, 43);
    ok = __all_sync(0xffffffffu, ok);
    tc_fence_after();
    if (ok) {
      const bool live = row < p.M;
      const int od = p.out_dtype[seg];
      const T* bias = static_cast<const T*>(p.bias[seg]);
      for (int c = 0; c < kN; c += 32) {
        float v[32];
        tmem_ld32(tmem + ((uint32_t)(quad * 32) << 16) + c, v);
        tmem_wait_ld();
        if (!live) continue;
        if (bias) {
#pragma unroll
          for (int e = 0; e < 32; ++e) v[e] += static_cast<float>(bias[n0 + c + e]);
        }
        char* base = static_cast<char*>(p.c[seg]);
        if (od == DA_F32) {
          float4* dst = reinterpret_cast<float4*>(reinterpret_cast<float*>(base) + (size_t)row * p.ldc[seg] + n0 + c);
#pragma unroll
          for (int e = 0; e < 8; ++e) dst[e] = make_float4(v[4 * e], v[4 * e + 1], v[4 * e + 2], v[4 * e + 3]);
        } else {
          uint32_t w[16];
          if (od == DA_BF16) {
#pragma unroll
            for (int e = 0; e < 16; ++e) w[e] = pack_bf16x2(v[2 * e], v[2 * e + 1]);
          } else {
#pragma unroll
            for (int e = 0; e < 16; ++e) w[e] = pack_f16x2(v[2 * e], v[2 * e + 1]);
          }
          uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(base) + (size_t)row * p.ldc[seg] + n0 + c);
#pragma unroll
          for (int e = 0; e < 4; ++e) dst[e] = make_uint4(w[4 * e], w[4 * e + 1], w[4 * e + 2], w[4 * e + 3]);
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc<1>(tmem, kN);
}

// ----------------------------------------------------------------------------------------------- persistent
// The operand-dtype GEMM of the layers around the routed attention (da_gemm_ex), persistent: one CTA per
// SM walks the 128 x 256 output tiles (N fastest, so CTAs running side by side read the same A rows from
// L2).  Two producer warps take alternate 48 KB stages (each completes about one stage per 0.4 us, and a
// stage feeds 4.2 MFLOP, 0.27 us of the SM's tensor pipe), and the accumulator is double-buffered in TMEM
// (2 x 256 columns), so the epilogue of one tile (bias, GELU or GELU', conversion, stores) runs while the
// tensor core computes the next.
namespace pk {
constexpr int kN = 256;
constexpr int kStages = 4;
constexpr int kABytes = kBM * kBK * 2;          // 16 KB
constexpr int kBBytes = kN * kBK * 2;           // 32 KB
constexpr int kStageBytes = kABytes + kBBytes;  // 48 KB
constexpr int kSmem = kStages * kStageBytes;
constexpr int kThreads = 224;                   // warps 0 and 6 TMA, 1 MMA, 2-5 epilogue
constexpr int kProducer2 = 6;
}  // namespace pk

template <typename T>
DA_DEV void epilogue_tile_chunk(const Params& p, int row, int col, float (&v)[32]) {
  T* dst = reinterpret_cast<T*>(p.c) + (size_t)row * p.ldc + col;
  if (p.bias) {
    const uint4* b4 = reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(p.bias) + col);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const uint4 bv = __ldg(b4 + e);
      const uint32_t bw[4] = {bv.x, bv.y, bv.z, bv.w};
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        const float2 f = unpack2<T>(bw[h]);
        v[8 * e + 2 * h] += f.x;
        v[8 * e + 2 * h + 1] += f.y;
      }
    }
  }
  if (p.act == 1) {
    if (p.aux) {
      T* za = reinterpret_cast<T*>(p.aux) + (size_t)row * p.ldaux + col;
#pragma unroll
      for (int e = 0; e < 4; ++e)
        reinterpret_cast<uint4*>(za)[e] = make_uint4(pack2<T>(v[8 * e], v[8 * e + 1]), pack2<T>(v[8 * e + 2], v[8 * e + 3]),
                                                     pack2<T>(v[8 * e + 4], v[8 * e + 5]), pack2<T>(v[8 * e + 6], v[8 * e + 7]));
    }
#pragma unroll
    for (int e = 0; e < 32; ++e) v[e] = gelu_f(v[e]);
  } else if (p.act == 2) {
    const uint4* z4 = reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(p.aux) + (size_t)row * p.ldaux + col);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const uint4 zv = z4[e];
      const uint32_t zw[4] = {zv.x, zv.y, zv.z, zv.w};
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        const float2 f = unpack2<T>(zw[h]);
        v[8 * e + 2 * h] *= gelu_grad_f(f.x);
        v[8 * e + 2 * h + 1] *= gelu_grad_f(f.y);
      }
    }
  }
#pragma unroll
  for (int e = 0; e < 4; ++e)
    reinterpret_cast<uint4*>(dst)[e] = make_uint4(pack2<T>(v[8 * e], v[8 * e + 1]), pack2<T>(v[8 * e + 2], v[8 * e + 3]),
                                                  pack2<T>(v[8 * e + 4], v[8 * e + 5]), pack2<T>(v[8 * e + 6], v[8 * e + 7]));
}

template <typename T, bool kAmn, bool kBmn>
__global__ void __launch_bounds__(pk::kThreads, 1) gemm_pk_kernel(const __grid_constant__ CUtensorMap ta,
                                                                  const __grid_constant__ CUtensorMap tb,
                                                                  const __grid_constant__ CUtensorMap ta2,
                                                                  const __grid_constant__ CUtensorMap tb2,
                                                                  const Params p) {
  using namespace pk;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ uint64_t full[kStages], empty[kStages], acc_full[2], acc_empty[2];
  __shared__ uint32_t tmem_base;
  __shared__ int abort_flag;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  // work items: output tiles, each split into `splits` K ranges of p.kps stages (split-K, fp32 partial tiles
  // into p.partial); splits = 1 writes the epilogue output
  const int n_tiles = (p.N + kN - 1) / kN, m_tiles = (p.M + kBM - 1) / kBM;
  const int nk_all = p.nk1 ? p.nk1 + (p.K - p.nk1 * kBK + kBK - 1) / kBK : (p.K + kBK - 1) / kBK;
  const int splits = p.partial ? (nk_all + p.kps - 1) / p.kps : 1;
  const int tiles = n_tiles * m_tiles * splits;
  const int my_tiles = blockIdx.x < tiles ? (tiles - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
  Abort ab{&abort_flag, p.status};

  if (threadIdx.x == 0) {
    abort_flag = 0;
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 4);  // one arrival per epilogue warp
    }
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc<1>(&tmem_base, 2 * kN);
    tmem_relinquish<1>();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  grid_dependency_wait();
  grid_launch_dependents();
  const uint32_t tmem = tmem_base;
  auto tile_mn = [&](int i, int& m0, int& n0, int& kb0, int& nk) {
    const int w = (int)blockIdx.x + i * (int)gridDim.x;
    const int t = w / splits, z = w % splits;  // splits of one tile run side by side
    m0 = (t / n_tiles) * kBM;
    n0 = (t % n_tiles) * kN;
    kb0 = z * (splits > 1 ? p.kps : 0);
    nk = splits > 1 ? min(p.kps, nk_all - kb0) : nk_all;
  };

  if ((warp == 0 || warp == kProducer2) && lane == 0) {
    // ---------------------------------------------------------------- TMA producers (alternate stages)
    const int pi = warp == 0 ? 0 : 1;
    prefetch_tmap(&ta);
    prefetch_tmap(&tb);
    if (p.nk1) {
      prefetch_tmap(&ta2);
      prefetch_tmap(&tb2);
    }
    bool ok = true;
    int it = 0, last = -1;
    for (int i = 0; ok && i < my_tiles; ++i) {
      int m0, n0, kb0, nk;
      tile_mn(i, m0, n0, kb0, nk);
      for (int kb = kb0; kb < kb0 + nk; ++kb, ++it) {
        if ((it & 1) != pi) continue;
        const int s = it % kStages;
        if (!mbar_wait(&empty[s], ((it / kStages) & 1u) ^ 1u, ab, 44)) { ok = false; break; }
        mbar_arrive_expect_tx(&full[s], kStageBytes);
        uint8_t* sa = smem + s * kStageBytes;
        uint8_t* sb = sa + kABytes;
        const bool second = p.nk1 && kb >= p.nk1;
        const CUtensorMap* tA = second ? &ta2 : &ta;
        const CUtensorMap* tB = second ? &tb2 : &tb;
        const int kk = second ? kb - p.nk1 : kb;
        if (!kAmn) {
          tma_load_2d(tA, &full[s], sa, kk * kBK, m0);
        } else {  // A stored [K, M]: this stage's 64 K rows, the tile's 128 M columns as two boxes
          tma_load_2d(tA, &full[s], sa, m0, kk * kBK);
          tma_load_2d(tA, &full[s], sa + kBK * 128, m0 + 64, kk * kBK);
        }
        if (!kBmn) {
          tma_load_2d(tB, &full[s], sb, kk * kBK, n0);
        } else {
          for (int j = 0; j < kN / 64; ++j) tma_load_2d(tB, &full[s], sb + j * kBK * 128, n0 + j * 64, kk * kBK);
        }
        last = it;
      }
    }
    // drain this producer's last loads (at most kStages / 2 of them can be in flight)
    for (int j = (last - kStages + 1 > 0 ? last - kStages + 1 : 0); j <= last; ++j)
      if ((j & 1) == pi) mbar_wait_drain(&full[j % kStages], (j / kStages) & 1u);
  } else if (warp == 1 && lane == 0) {
    // ---------------------------------------------------------------- MMA issuer
    const uint32_t idesc = idesc_f16(kBM, kN, std::is_same<T, __nv_bfloat16>::value, kAmn, kBmn);
    bool ok = true;
    int it = 0;
    for (int i = 0; ok && i < my_tiles; ++i) {
      const int buf = i & 1;
      int m0, n0, kb0, nk;
      tile_mn(i, m0, n0, kb0, nk);
      if (i >= 2 && !mbar_wait(&acc_empty[buf], ((i >> 1) - 1) & 1u, ab, 45)) break;
      tc_fence_after();
      const uint32_t d = tmem + buf * kN;
      for (int kb = 0; kb < nk; ++kb, ++it) {
        const int s = it % kStages;
        if (!mbar_wait(&full[s], (it / kStages) & 1u, ab, 46)) { ok = false; break; }
        tc_fence_after();
        const uint32_t sa = smem_u32(smem + s * kStageBytes);
        const uint32_t sb = sa + kABytes;
#pragma unroll
        for (int k = 0; k < kBK / 16; ++k) {
          const uint64_t ad = kAmn ? sdesc_sw128(sa + k * 16 * 128, kBK * 128, 1024) : sdesc_sw128(sa + k * 32, 16, 1024);
          const uint64_t bd = kBmn ? sdesc_sw128(sb + k * 16 * 128, kBK * 128, 1024) : sdesc_sw128(sb + k * 32, 16, 1024);
          mma_f16_ss<1>(d, ad, bd, idesc, (kb > 0 || k > 0) ? 1u : 0u);
        }
        mma_commit<1>(smem_u32(&empty[s]));
      }
      if (ok) mma_commit<1>(smem_u32(&acc_full[buf]));
    }
  } else if (warp >= 2 && warp <= 5) {
    // ---------------------------------------------------------------- epilogue (thread = output row)
    const int quad = warp & 3;
    bool ok = true;
    for (int i = 0; i < my_tiles; ++i) {
      const int buf = i & 1;
      int m0, n0, kb0, nk;
      tile_mn(i, m0, n0, kb0, nk);
      if (ok) ok = mbar_wait(&acc_full[buf], (i >> 1) & 1u, ab, 47);
      ok = __all_sync(0xffffffffu, ok);
      tc_fence_after();
      const int row = m0 + quad * 32 + lane;
      if (ok) {
        for (int c = 0; c < kN; c += 32) {
          float v[32];
          tmem_ld32(tmem + ((uint32_t)(quad * 32) << 16) + buf * kN + c, v);
          tmem_wait_ld();
          if (row >= p.M || n0 + c >= p.N) continue;
          if (splits > 1) {  // this split's fp32 partial tile (added in split order by splitk_reduce_kernel)
            const int z = kb0 / p.kps;
            float4* dst = reinterpret_cast<float4*>(p.partial + ((size_t)z * p.M + row) * p.N + n0 + c);
#pragma unroll
            for (int e = 0; e < 8; ++e) dst[e] = make_float4(v[4 * e], v[4 * e + 1], v[4 * e + 2], v[4 * e + 3]);
          } else {
            epilogue_tile_chunk<T>(p, row, n0 + c, v);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[buf]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc<1>(tmem, 2 * kN);
}

template <typename T, bool kAmn, bool kBmn>
int launch_pk(const void* A, int64_t lda, const void* B, int64_t ldb, const void* A2, int64_t lda2, const void* B2,
              int64_t ldb2, int64_t K2, const Params& p, cudaStream_t st) {
  const CUtensorMapDataType dt =
      std::is_same<T, __nv_bfloat16>::value ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  const int64_t K1 = A2 ? (int64_t)p.nk1 * kBK : p.K;
  CUtensorMap ta, tb, ta2, tb2;
  if (kAmn) {  // A stored [K, M]
    if (int rc = make_tmap_2d(&ta, A, dt, 2, p.M, K1, (uint64_t)lda * 2, 64, kBK)) return rc;
  } else {
    if (int rc = make_tmap_2d(&ta, A, dt, 2, K1, p.M, (uint64_t)lda * 2, 64, kBM)) return rc;
  }
  if (kBmn) {
    if (int rc = make_tmap_2d(&tb, B, dt, 2, p.N, K1, (uint64_t)ldb * 2, 64, kBK)) return rc;
  } else {
    if (int rc = make_tmap_2d(&tb, B, dt, 2, K1, p.N, (uint64_t)ldb * 2, 64, pk::kN)) return rc;
  }
  ta2 = ta;
  tb2 = tb;
  if (A2) {
    if (int rc = make_tmap_2d(&ta2, A2, dt, 2, K2, p.M, (uint64_t)lda2 * 2, 64, kBM)) return rc;
    if (kBmn) {
      if (int rc = make_tmap_2d(&tb2, B2, dt, 2, p.N, K2, (uint64_t)ldb2 * 2, 64, kBK)) return rc;
    } else {
      if (int rc = make_tmap_2d(&tb2, B2, dt, 2, K2, p.N, (uint64_t)ldb2 * 2, 64, pk::kN)) return rc;
    }
  }
  auto kern = gemm_pk_kernel<T, kAmn, kBmn>;
  const int smem = pk::kSmem + 1024;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
    return record_cuda_error();
  const int nk_all = p.nk1 ? p.nk1 + (int)((p.K - p.nk1 * kBK + kBK - 1) / kBK) : (int)((p.K + kBK - 1) / kBK);
  const int splits = p.partial ? (nk_all + p.kps - 1) / p.kps : 1;
  const int tiles = (int)(((p.M + kBM - 1) / kBM) * ((p.N + pk::kN - 1) / pk::kN)) * splits;
  const int grid = tiles < sm_count() ? tiles : sm_count();
  return launch_kernel(kern, dim3((unsigned)grid), dim3(pk::kThreads), smem, st, false, ta, tb, ta2, tb2, p);
}

// C[m, n] += sum over splits z, in index order, of partial[z, m, n] (four columns per thread).
// C (+)= the splits' partial sums, added in split order: fp32 C added to (accumulate) or overwritten, or
// C in a 16-bit type TO, stored once.
template <typename TO>
__global__ void __launch_bounds__(256) splitk_reduce_kernel(const float* partial, int splits, int M, int N, void* c,
                                                            int64_t ldc, int accumulate) {
  grid_dependency_wait();
  grid_launch_dependents();
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;  // float4 index
  const int64_t per_row = N / 4;
  if (i >= (int64_t)M * per_row) return;
  const int64_t row = i / per_row, col = (i % per_row) * 4;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int z = 0; z < splits; ++z) {
    const float4 v = *reinterpret_cast<const float4*>(partial + ((size_t)z * M + row) * N + col);
    acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
  }
  if constexpr (std::is_same<TO, float>::value) {
    float4* dst = reinterpret_cast<float4*>(static_cast<float*>(c) + row * ldc + col);
    if (accumulate) {
      const float4 o = *dst;
      acc.x += o.x; acc.y += o.y; acc.z += o.z; acc.w += o.w;
    }
    *dst = acc;
  } else {
    *reinterpret_cast<uint2*>(static_cast<TO*>(c) + row * ldc + col) =
        make_uint2(pack2<TO>(acc.x, acc.y), pack2<TO>(acc.z, acc.w));
  }
}

// Split count and K stages per split of a split-K product (the same plan for the workspace query and the
// launch): about two CTAs per SM-sized wave of 128 x 128 output tiles unless `splits` asks otherwise.
inline void splitk_plan(int64_t M, int64_t N, int64_t K, int splits, int* out_splits, int* out_kps) {
  const int nk = (int)((K + kBK - 1) / kBK);
  if (splits <= 0) {
    const int tiles = (int)((M / 128) * (N / 128));
    splits = (2 * sm_count() + tiles - 1) / tiles;
  }
  int kps = (nk + splits - 1) / splits;
  if (kps < 1) kps = 1;
  *out_splits = (nk + kps - 1) / kps;  // every split gets at least one K stage
  *out_kps = kps;
}

// out_dtype: DA_F32 (p.accumulate: added to C, else overwritten), or the 16-bit type C is stored in
inline int splitk_reduce(const Params& p, int splits, cudaStream_t st, int out_dtype = DA_F32) {
  const int64_t n4 = (int64_t)p.M * (p.N / 4);
  const dim3 grid((unsigned)((n4 + 255) / 256));
  if (out_dtype == DA_BF16)
    return launch_kernel(splitk_reduce_kernel<__nv_bfloat16>, grid, dim3(256), 0, st, false, (const float*)p.partial,
                         splits, p.M, p.N, p.c, p.ldc, 0);
  if (out_dtype == DA_F16)
    return launch_kernel(splitk_reduce_kernel<__half>, grid, dim3(256), 0, st, false, (const float*)p.partial, splits,
                         p.M, p.N, p.c, p.ldc, 0);
  return launch_kernel(splitk_reduce_kernel<float>, grid, dim3(256), 0, st, false, (const float*)p.partial, splits,
                       p.M, p.N, p.c, p.ldc, p.accumulate);
}

template <typename T, int kN, bool kAmn, bool kBmn>
int launch(const void* A, int64_t lda, const void* B, int64_t ldb, const Params& p, int splits, cudaStream_t st) {
  using C = Cfg<kN>;
  const CUtensorMapDataType dt =
      std::is_same<T, __nv_bfloat16>::value ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUtensorMap ta, tb;
  int rc = kAmn ? (p.kseg ? make_tmap_2d(&ta, A, dt, 2, p.a_inner, (uint64_t)p.kseg * kBK, (uint64_t)lda * 2, 64, kBK)
                          : make_tmap_2d(&ta, A, dt, 2, p.M, p.K, (uint64_t)lda * 2, 64, kBK))
                : make_tmap_2d(&ta, A, dt, 2, p.K, p.M, (uint64_t)lda * 2, 64, kBM);
  if (rc) return rc;
  rc = kBmn ? make_tmap_2d(&tb, B, dt, 2, p.N, p.K, (uint64_t)ldb * 2, 64, kBK)
            : make_tmap_2d(&tb, B, dt, 2, p.K, p.N, (uint64_t)ldb * 2, 64, kN);
  if (rc) return rc;
  auto kern = gemm_kernel<T, kN, kAmn, kBmn>;
  const int smem = C::kSmem + 1024;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
    return record_cuda_error();
  dim3 grid((unsigned)((p.M + kBM - 1) / kBM), (unsigned)((p.N + kN - 1) / kN), (unsigned)splits);
  return launch_kernel(kern, grid, dim3(kThreads), smem, st, false, ta, tb, ta, tb, p);
}

// The same with a second K segment (A2 [M, K2] / B2 in the modes of A / B): C = A.B^T + A2.B2^T.
template <typename T, int kN, bool kAmn, bool kBmn>
int launch2(const void* A, int64_t lda, const void* B, int64_t ldb, const void* A2, int64_t lda2, const void* B2,
            int64_t ldb2, int64_t K2, const Params& p, cudaStream_t st) {
  static_assert(!kAmn, "the second segment takes a K-major A");
  using C = Cfg<kN>;
  const CUtensorMapDataType dt =
      std::is_same<T, __nv_bfloat16>::value ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  const int64_t K1 = (int64_t)p.nk1 * kBK;
  CUtensorMap ta, tb, ta2, tb2;
  if (int rc = make_tmap_2d(&ta, A, dt, 2, K1, p.M, (uint64_t)lda * 2, 64, kBM)) return rc;
  if (int rc = make_tmap_2d(&ta2, A2, dt, 2, K2, p.M, (uint64_t)lda2 * 2, 64, kBM)) return rc;
  if (kBmn) {
    if (int rc = make_tmap_2d(&tb, B, dt, 2, p.N, K1, (uint64_t)ldb * 2, 64, kBK)) return rc;
    if (int rc = make_tmap_2d(&tb2, B2, dt, 2, p.N, K2, (uint64_t)ldb2 * 2, 64, kBK)) return rc;
  } else {
    if (int rc = make_tmap_2d(&tb, B, dt, 2, K1, p.N, (uint64_t)ldb * 2, 64, kN)) return rc;
    if (int rc = make_tmap_2d(&tb2, B2, dt, 2, K2, p.N, (uint64_t)ldb2 * 2, 64, kN)) return rc;
  }
  auto kern = gemm_kernel<T, kN, kAmn, kBmn>;
  const int smem = C::kSmem + 1024;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
    return record_cuda_error();
  dim3 grid((unsigned)((p.M + kBM - 1) / kBM), (unsigned)((p.N + kN - 1) / kN), 1);
  return launch_kernel(kern, grid, dim3(kThreads), smem, st, false, ta, tb, ta2, tb2, p);
}

template <typename T>
int dispatch(int a_mn, int b_mn, int n_tile, const void* A, int64_t lda, const void* B, int64_t ldb, const Params& p,
             int splits, cudaStream_t st) {
#define DA_GEMM_CASE(NT, AMN, BMN) \
  if (n_tile == NT && a_mn == AMN && b_mn == BMN) return launch<T, NT, AMN, BMN>(A, lda, B, ldb, p, splits, st);
  DA_GEMM_CASE(128, 0, 0)
  DA_GEMM_CASE(256, 0, 0)
  DA_GEMM_CASE(128, 0, 1)
  DA_GEMM_CASE(256, 0, 1)
  DA_GEMM_CASE(128, 1, 1)
  DA_GEMM_CASE(256, 1, 1)
#undef DA_GEMM_CASE
  return DA_ERR_UNSUPPORTED;
}

}  // namespace gemm
}  // namespace da

extern "C" int da_gemm(const void* A, int64_t lda, int a_mn_major, const void* B, int64_t ldb, int b_mn_major,
                       void* C, int64_t ldc, int64_t M, int64_t N, int64_t K, int dtype, int out_f32, int accumulate,
                       int* status, void* stream) {
  using namespace da;
  if (!A || !B || !C || !status) return DA_ERR_NULL;
  if (int rc = bind_device(A)) return rc;
  if (dtype != DA_BF16 && dtype != DA_F16) return DA_ERR_DTYPE;
  if (M <= 0 || N <= 0 || K <= 0 || N % 128) return DA_ERR_SHAPE;
  if ((lda % 8) || (ldb % 8)) return DA_ERR_ALIGN;  // 16-byte row strides for TMA
  if (a_mn_major && M % 128) return DA_ERR_SHAPE;   // every A box starts inside the matrix
  if (accumulate && !out_f32) return DA_ERR_UNSUPPORTED;
  if ((reinterpret_cast<uintptr_t>(C) & 15) || (ldc % 8)) return DA_ERR_ALIGN;
  gemm::Params p{(int)M, (int)N, (int)K, C, ldc, out_f32, accumulate, status, 0};
  const int n_tile = (N % 256 == 0 && (M / 128) * (N / 256) >= 120) ? 256 : 128;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (dtype == DA_BF16)
    return gemm::dispatch<__nv_bfloat16>(a_mn_major, b_mn_major, n_tile, A, lda, B, ldb, p, 1, st);
  return gemm::dispatch<__half>(a_mn_major, b_mn_major, n_tile, A, lda, B, ldb, p, 1, st);
}

extern "C" int da_gemm_ex(const void* A, int64_t lda, const void* B, int64_t ldb, int b_mn_major, int64_t K,
                          const void* A2, int64_t lda2, const void* B2, int64_t ldb2, int64_t K2, void* C,
                          int64_t ldc, int64_t M, int64_t N, int dtype, const void* bias, int act, void* aux,
                          int64_t ldaux, int* status, void* stream) {
  using namespace da;
  if (!A || !B || !C || !status) return DA_ERR_NULL;
  if ((A2 == nullptr) != (B2 == nullptr)) return DA_ERR_NULL;
  if (act < 0 || act > 2) return DA_ERR_UNSUPPORTED;
  if (act == 2 && !aux) return DA_ERR_NULL;
  if (int rc = bind_device(A)) return rc;
  if (dtype != DA_BF16 && dtype != DA_F16) return DA_ERR_DTYPE;
  if (M <= 0 || N <= 0 || K <= 0 || N % 128 || (A2 && (K2 <= 0 || K % gemm::kBK))) return DA_ERR_SHAPE;
  if ((lda % 8) || (ldb % 8) || (A2 && ((lda2 % 8) || (ldb2 % 8))) || (ldc % 8) || (aux && (ldaux % 8)))
    return DA_ERR_ALIGN;
  const uintptr_t any = reinterpret_cast<uintptr_t>(C) | reinterpret_cast<uintptr_t>(bias) |
                        reinterpret_cast<uintptr_t>(aux);
  if (any & 15) return DA_ERR_ALIGN;
  gemm::Params p{(int)M, (int)N, (int)(K + (A2 ? K2 : 0)), C, ldc, 0, 0, status, 0};
  p.nk1 = A2 ? (int)(K / gemm::kBK) : 0;
  p.bias = bias;
  p.act = act;
  p.aux = aux;
  p.ldaux = ldaux;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const bool bf = dtype == DA_BF16;
  if (N % 256 == 0) {  // the persistent kernel (256-column tiles)
    if (bf) return b_mn_major ? gemm::launch_pk<__nv_bfloat16, false, true>(A, lda, B, ldb, A2, lda2, B2, ldb2, K2, p, st)
                              : gemm::launch_pk<__nv_bfloat16, false, false>(A, lda, B, ldb, A2, lda2, B2, ldb2, K2, p, st);
    return b_mn_major ? gemm::launch_pk<__half, false, true>(A, lda, B, ldb, A2, lda2, B2, ldb2, K2, p, st)
                      : gemm::launch_pk<__half, false, false>(A, lda, B, ldb, A2, lda2, B2, ldb2, K2, p, st);
  }
  const int n_tile = (N % 256 == 0 && (M / 128) * (N / 256) >= 120) ? 256 : 128;
  if (!A2) {
    if (bf) return gemm::dispatch<__nv_bfloat16>(0, b_mn_major, n_tile, A, lda, B, ldb, p, 1, st);
    return gemm::dispatch<__half>(0, b_mn_major, n_tile, A, lda, B, ldb, p, 1, st);
  }
#define DA_GEMM2_CASE(TT, NT, BMN)                                                                       \
  if (n_tile == NT && (b_mn_major != 0) == BMN)                                                         \
    return gemm::launch2<TT, NT, false, BMN>(A, lda, B, ldb, A2, lda2, B2, ldb2, K2, p, st);
  if (bf) {
    DA_GEMM2_CASE(__nv_bfloat16, 128, false)
    DA_GEMM2_CASE(__nv_bfloat16, 256, false)
    DA_GEMM2_CASE(__nv_bfloat16, 128, true)
    DA_GEMM2_CASE(__nv_bfloat16, 256, true)
  } else {
    DA_GEMM2_CASE(__half, 128, false)
    DA_GEMM2_CASE(__half, 256, false)
    DA_GEMM2_CASE(__half, 128, true)
    DA_GEMM2_CASE(__half, 256, true)
  }
#undef DA_GEMM2_CASE
  return DA_ERR_UNSUPPORTED;
}

extern "C" int64_t da_gemm_splitk_workspace_elems(int64_t M, int64_t N, int64_t K, int splits) {
  if (M <= 0 || N <= 0 || K <= 0 || M % 128 || N % 128) return -1;
  int s = 0, kps = 0;
  da::gemm::splitk_plan(M, N, K, splits, &s, &kps);
  return (int64_t)s * M * N;
}

namespace {

// C (fp32, += when accumulate, else =; or c_dtype = the operand dtype, stored once) = A.B^T over a K split
// across CTAs; with a workspace the splits' partials are added in split order.
int splitk_entry(const void* A, int64_t lda, int a_mn_major, const void* B, int64_t ldb, int b_mn_major, void* C,
                 int64_t ldc, int c_dtype, int accumulate, int64_t M, int64_t N, int64_t K, int dtype, int splits,
                 float* workspace, int64_t workspace_elems, int* status, void* stream) {
  using namespace da;
  if (!A || !B || !C || !status) return DA_ERR_NULL;
  if (int rc = bind_device(A)) return rc;
  if (dtype != DA_BF16 && dtype != DA_F16) return DA_ERR_DTYPE;
  if (c_dtype != DA_F32 && c_dtype != dtype) return DA_ERR_DTYPE;
  if (M <= 0 || N <= 0 || K <= 0 || N % 128 || M % 128) return DA_ERR_SHAPE;
  if ((lda % 8) || (ldb % 8)) return DA_ERR_ALIGN;
  if ((reinterpret_cast<uintptr_t>(C) & 15) || (ldc % 4)) return DA_ERR_ALIGN;
  const int n_tile = 128;
  int kps = 0;
  gemm::splitk_plan(M, N, K, splits, &splits, &kps);
  gemm::Params p{(int)M, (int)N, (int)K, C, ldc, c_dtype == DA_F32 ? 1 : 0, accumulate, status, kps};
  if (workspace) {
    if (workspace_elems < (int64_t)splits * M * N) return DA_ERR_WORKSPACE;
    if (reinterpret_cast<uintptr_t>(workspace) & 15) return DA_ERR_ALIGN;
    p.partial = workspace;
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (p.partial && splits > 1 && a_mn_major && b_mn_major && N % 256 == 0) {
    // the weight gradients of the block's layers: the persistent kernel's split-K work items
    const int rc = dtype == DA_BF16
                       ? gemm::launch_pk<__nv_bfloat16, true, true>(A, lda, B, ldb, nullptr, 0, nullptr, 0, 0, p, st)
                       : gemm::launch_pk<__half, true, true>(A, lda, B, ldb, nullptr, 0, nullptr, 0, 0, p, st);
    if (rc) return rc;
    return gemm::splitk_reduce(p, splits, st, c_dtype);
  }
  int rc = dtype == DA_BF16
               ? gemm::dispatch<__nv_bfloat16>(a_mn_major, b_mn_major, n_tile, A, lda, B, ldb, p, splits, st)
               : gemm::dispatch<__half>(a_mn_major, b_mn_major, n_tile, A, lda, B, ldb, p, splits, st);
  // one split writes C itself (the kernel's non-split epilogue)
  if (rc || !p.partial || splits == 1) return rc;
  return gemm::splitk_reduce(p, splits, st, c_dtype);
}

}  // namespace

extern "C" int da_gemm_splitk(const void* A, int64_t lda, int a_mn_major, const void* B, int64_t ldb, int b_mn_major,
                              float* C, int64_t ldc, int64_t M, int64_t N, int64_t K, int dtype, int splits,
                              float* workspace, int64_t workspace_elems, int* status, void* stream) {
  return splitk_entry(A, lda, a_mn_major, B, ldb, b_mn_major, C, ldc, DA_F32, 1, M, N, K, dtype, splits, workspace,
                      workspace_elems, status, stream);
}

extern "C" int da_gemm_splitk_store(const void* A, int64_t lda, int a_mn_major, const void* B, int64_t ldb,
                                    int b_mn_major, void* C, int64_t ldc, int c_dtype, int64_t M, int64_t N, int64_t K,
                                    int dtype, int splits, float* workspace, int64_t workspace_elems, int* status,
                                    void* stream) {
  if (!workspace) return DA_ERR_WORKSPACE;
  return splitk_entry(A, lda, a_mn_major, B, ldb, b_mn_major, C, ldc, c_dtype, 0, M, N, K, dtype, splits, workspace,
                      workspace_elems, status, stream);
}

extern "C" int da_gemm_segments(const void* A, int64_t lda, int64_t M, int64_t K, int dtype, int nseg,
                                const void* const* B, const int64_t* ldb, const int64_t* N, void* const* C,
                                const int64_t* ldc, const int* out_dtype, const void* const* bias, int* status,
                                void* stream) {
  using namespace da;
  using namespace da::gemm;
  if (!A || !B || !N || !C || !ldc || !ldb || !out_dtype || !status) return DA_ERR_NULL;
  if (int rc = bind_device(A)) return rc;
  if (dtype != DA_BF16 && dtype != DA_F16) return DA_ERR_DTYPE;
  if (nseg < 1 || nseg > kMaxSeg || M <= 0 || K <= 0) return DA_ERR_SHAPE;
  if (lda % 8) return DA_ERR_ALIGN;
  SegParams p;
  p.M = (int)M;
  p.K = (int)K;
  p.nseg = nseg;
  p.status = status;
  int64_t total = 0;
  bool all256 = true;
  for (int s = 0; s < nseg; ++s) {
    if (!B[s] || !C[s]) return DA_ERR_NULL;
    if (N[s] <= 0 || N[s] % 128) return DA_ERR_SHAPE;
    if (N[s] % 256) all256 = false;
    if (ldb[s] % 8) return DA_ERR_ALIGN;
    const int od = out_dtype[s];
    if (od != DA_F16 && od != DA_BF16 && od != DA_F32) return DA_ERR_DTYPE;
    if ((reinterpret_cast<uintptr_t>(C[s]) & 15) || (ldc[s] % 8)) return DA_ERR_ALIGN;
    p.seg_n0[s] = (int)total;
    p.c[s] = C[s];
    p.ldc[s] = ldc[s];
    p.out_dtype[s] = od;
    p.bias[s] = bias ? bias[s] : nullptr;
    total += N[s];
  }
  p.seg_n0[nseg] = (int)total;
  for (int s = nseg; s < kMaxSeg; ++s) {
    p.seg_n0[s + 1 <= kMaxSeg ? s + 1 : kMaxSeg] = (int)total;
    p.c[s] = nullptr;
    p.ldc[s] = 0;
    p.out_dtype[s] = DA_F32;
    p.bias[s] = nullptr;
  }
  const CUtensorMapDataType dt = dtype == DA_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  const int n_tile = (all256 && (M / 128) * (total / 256) >= 120) ? 256 : 128;
  CUtensorMap ta, tb[kMaxSeg];
  int rc = make_tmap_2d(&ta, A, dt, 2, K, M, (uint64_t)lda * 2, 64, kBM);
  if (rc) return rc;
  for (int s = 0; s < kMaxSeg; ++s) {
    const int si = s < nseg ? s : 0;
    rc = make_tmap_2d(&tb[s], B[si], dt, 2, K, N[si], (uint64_t)ldb[si] * 2, 64, n_tile);
    if (rc) return rc;
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  dim3 grid((unsigned)((M + kBM - 1) / kBM), (unsigned)(total / n_tile), 1);
  auto run = [&](auto kern, int smem_bytes) -> int {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes) != cudaSuccess)
      return record_cuda_error();
    return launch_kernel(kern, grid, dim3(kThreads), smem_bytes, st, false, ta, tb[0], tb[1], tb[2], p);
  };
  const bool bf16 = dtype == DA_BF16;
  if (n_tile == 256)
    return bf16 ? run(gemm_seg_kernel<__nv_bfloat16, 256>, SegCfg<256>::kSmem + 1024)
                : run(gemm_seg_kernel<__half, 256>, SegCfg<256>::kSmem + 1024);
  return bf16 ? run(gemm_seg_kernel<__nv_bfloat16, 128>, SegCfg<128>::kSmem + 1024)
              : run(gemm_seg_kernel<__half, 128>, SegCfg<128>::kSmem + 1024);
}

extern "C" int da_gemm_splitk_grouped(const void* A, int64_t lda, int64_t a_group_cols, const void* B, int64_t ldb,
                                      float* C, int64_t ldc, int64_t M, int64_t N, int64_t K_group, int groups,
                                      int dtype, int splits, float* workspace, int64_t workspace_elems,
                                      int* status, void* stream) {
  using namespace da;
  if (!A || !B || !C || !status) return DA_ERR_NULL;
  if (int rc = bind_device(A)) return rc;
  if (dtype != DA_BF16 && dtype != DA_F16) return DA_ERR_DTYPE;
  if (M <= 0 || N <= 0 || K_group <= 0 || groups <= 0 || N % 128 || M % 128 || K_group % gemm::kBK)
    return DA_ERR_SHAPE;
  if (a_group_cols < 0 || a_group_cols % 8 || (lda % 8) || (ldb % 8)) return DA_ERR_ALIGN;
  if ((int64_t)(groups - 1) * a_group_cols + M > lda) return DA_ERR_SHAPE;
  if ((reinterpret_cast<uintptr_t>(C) & 15) || (ldc % 4)) return DA_ERR_ALIGN;
  const int64_t K = K_group * groups;
  int kps = 0;
  gemm::splitk_plan(M, N, K, splits, &splits, &kps);
  gemm::Params p{(int)M, (int)N, (int)K, C, ldc, 1, 1, status, kps};
  p.kseg = (int)(K_group / gemm::kBK);
  p.a_goff = (int)a_group_cols;
  p.a_inner = (int)((groups - 1) * a_group_cols + M);
  if (workspace) {
    if (workspace_elems < (int64_t)splits * M * N) return DA_ERR_WORKSPACE;
    if (reinterpret_cast<uintptr_t>(workspace) & 15) return DA_ERR_ALIGN;
    p.partial = workspace;
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int rc = dtype == DA_BF16 ? gemm::dispatch<__nv_bfloat16>(1, 1, 128, A, lda, B, ldb, p, splits, st)
                            : gemm::dispatch<__half>(1, 1, 128, A, lda, B, ldb, p, splits, st);
  if (rc || !p.partial || splits == 1) return rc;
  return gemm::splitk_reduce(p, splits, st);
}
