// Dictionary route, forward.
//
// Reference: src/double_attention/ops.py:16-62 (dictionary_route_reference)
// and the Triton path it replaces, triton_kernels.py:1717-1802 / :126-292.
//
//   q_hat = q / max(||q||, eps)                         (normalize_input)
//   p     = softmax(beta * q_hat . Dk)  over M atoms
//   r     = p . Dv^T
//   z     = r / max(||r||, eps)                         (normalize_output)
//
// The route is a non-causal attention whose "keys" and "values" are the M
// dictionary atoms, shared by every row.  One CTA pair (a 2-CTA cluster
// running cta_group::2 MMAs) owns 128 route rows, 64 per CTA:
//   * S_j = q . Dk_j for atom tiles of 64 (paired M=128 MMA, N=64) lands in
//     TMEM "folded": lane l holds row l%64, atoms (l/64)*32 + [0,32);
//   * the softmax warpgroup turns S_j into bf16 probabilities P_j in shared
//     memory (each CTA writes its own 64 rows);
//   * O += P_j . Dv_j^T accumulates the reconstruction in TMEM (R/2 columns
//     per CTA thanks to the folded paired layout, so R = 512 fits).
// Nothing of size [rows, M] ever reaches HBM; q is read once, z written once.
//
// Softmax without rescaling: every score obeys
//   beta * q_hat . dk_j  <=  beta * ||q_hat|| * max_j ||dk_j|| =: c_row,
// so p_j = 2^(log2e * beta q_hat.dk_j - log2e * c_row) never exceeds 1 and the
// accumulator never needs the online-softmax correction.  The exact row
// maximum is tracked too; a row whose largest term fell below 2^-100 (which
// cannot happen for normalised inputs with beta * max||dk|| < 34) is listed
// and recomputed exactly in fp32 by the last CTA of the grid.
#include "common.cuh"
#include "host_util.h"
#include "route_common.h"

namespace da {
namespace route {

template <int kR>
struct FwdCfg {
  static constexpr int kRows = 64;                 // rows per CTA (128 per pair)
  static constexpr int kNA = 64;                   // atoms per tile
  static constexpr int kNc = kR < 256 ? kR : 256;  // N of one P.Dv^T instruction
  static constexpr int kPV = kR / kNc;             // P.Dv^T instructions per tile
  static constexpr int kStages = kR == 512 ? 2 : (kR == 256 ? 4 : 8);
  static constexpr int kB = 4;                     // S (TMEM) and P (smem) buffers in flight
  static constexpr int kQBytes = kRows * kR * 2;         // this CTA's q rows
  static constexpr int kDkBytes = (kNA / 2) * kR * 2;    // this CTA's half of a Dk tile
  static constexpr int kDvBytes = (kR / 2) * kNA * 2;    // this CTA's half of a Dv tile
  static constexpr int kPBytes = kRows * kNA * 2;
  static constexpr int kOffQ = 0;
  static constexpr int kOffDk = kOffQ + kQBytes;
  static constexpr int kOffDv = kOffDk + kStages * kDkBytes;
  static constexpr int kOffP = kOffDv + kStages * kDvBytes;
  static constexpr int kOffRed = kOffP + kB * kPBytes;     // 2 x 128 floats for row reductions
  // At least 120 KB so that exactly one CTA of a pair lives on each SM.
  static constexpr int kSmemUsed = kOffRed + 2 * 128 * 4;
  static_assert(kSmemUsed + 1024 + 512 <= 232448, "route tile does not fit in shared memory");
  static constexpr int kSmem = kSmemUsed < 120 * 1024 ? 120 * 1024 : kSmemUsed;
  static constexpr int kTmemO = 0;
  static constexpr int kTmemS = kR / 2;
  static constexpr int kTmemCols = (kR / 2 + 32 * kB) <= 128 ? 128 : ((kR / 2 + 32 * kB) <= 256 ? 256 : 512);
  static constexpr int kThreads = 192;             // warp0 TMA, warp1 MMA, warps2-5 softmax
};

struct FwdParams {
  const void* q;        // raw pointers (repair path)
  int64_t q_row_stride;
  const void* dk_t;
  const void* dv;
  int rows;             // route rows per group
  int groups;
  int col_stride;       // column offset between groups inside the q matrix (elements)
  int M;                // atoms (multiple of 64)
  const float* beta;    // device scalar
  const float* dk_max;  // device scalar: max column norm of Dk as rounded
  float eps;
  int normalize_input, normalize_output;
  void* z;              // [groups, rows, R] output (q dtype)
  float* lse;           // [groups, rows]  ln sum_j exp(beta q_hat.dk_j)
  float* out_norm;      // [groups, rows]  ||p . Dv^T|| (p normalised)
  int* argmax;          // [groups, rows]  index of the largest assignment weight (optional)
  int* work;            // [0] CTA tickets, [1] repair count, [2..] repair rows
  int repair_cap;
  int* status;
  int* trace;           // optional progress markers (debug)
};

// Exact fp32 recomputation of the listed rows by one CTA (rare path).
template <int kR, typename T>
__device__ void repair_listed_rows(const FwdParams& p, float* buf) {
  const int nthr = blockDim.x, tid = threadIdx.x;
  const int count = min(p.work[1], p.repair_cap);
  float* prob = buf;            // [M]
  float* vec = prob + p.M;      // [kR]
  float* red = vec + kR;        // [32]
  auto block_sum = [&](float v) -> float {
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    __syncthreads();
    if ((tid & 31) == 0) red[tid >> 5] = v;
    __syncthreads();
    float t = 0.f;
    for (int w = 0; w < nthr / 32; ++w) t += red[w];
    return t;
  };
  auto block_max = [&](float v) -> float {
    for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    __syncthreads();
    if ((tid & 31) == 0) red[tid >> 5] = v;
    __syncthreads();
    float t = -INFINITY;
    for (int w = 0; w < nthr / 32; ++w) t = fmaxf(t, red[w]);
    return t;
  };
  const float beta = *p.beta;
  const T* dkt = reinterpret_cast<const T*>(p.dk_t);
  const __nv_bfloat16* dv = reinterpret_cast<const __nv_bfloat16*>(p.dv);
  for (int it = 0; it < count; ++it) {
    const int idx = p.work[2 + it];
    const int g = idx / p.rows, row = idx % p.rows;
    const T* qrow = reinterpret_cast<const T*>(p.q) + (size_t)row * p.q_row_stride + (size_t)g * p.col_stride;
    float ss = 0.f;
    for (int r = tid; r < kR; r += nthr) {
      const float v = static_cast<float>(qrow[r]);
      ss = fmaf(v, v, ss);
    }
    const float qn = sqrtf(block_sum(ss));
    const float invn = p.normalize_input ? 1.f / fmaxf(qn, p.eps) : 1.f;
    for (int r = tid; r < kR; r += nthr) vec[r] = static_cast<float>(qrow[r]) * invn;
    __syncthreads();
    float mx = -INFINITY;
    for (int j = tid; j < p.M; j += nthr) {
      float acc = 0.f;
      for (int r = 0; r < kR; ++r) acc = fmaf(vec[r], static_cast<float>(dkt[(size_t)j * kR + r]), acc);
      prob[j] = beta * acc;
      mx = fmaxf(mx, prob[j]);
    }
    mx = block_max(mx);
    if (p.argmax) {
      __syncthreads();
      if (tid == 0) {
        int best = 0;
        for (int j = 0; j < p.M; ++j) if (prob[j] == mx) { best = j; break; }
        p.argmax[idx] = best;
      }
      __syncthreads();
    }
    float sum = 0.f;
    for (int j = tid; j < p.M; j += nthr) {
      prob[j] = expf(prob[j] - mx);
      sum += prob[j];
    }
    sum = block_sum(sum);
    __syncthreads();
    float on = 0.f;
    for (int r = tid; r < kR; r += nthr) {
      float acc = 0.f;
      for (int j = 0; j < p.M; ++j) acc = fmaf(prob[j], static_cast<float>(dv[(size_t)r * p.M + j]), acc);
      vec[r] = acc / sum;
      on = fmaf(vec[r], vec[r], on);
    }
    on = sqrtf(block_sum(on));
    const float factor = p.normalize_output ? 1.f / fmaxf(on, p.eps) : 1.f;
    T* zrow = reinterpret_cast<T*>(p.z) + (size_t)idx * kR;
    for (int r = tid; r < kR; r += nthr) zrow[r] = from_f32<T>(vec[r] * factor);
    if (tid == 0) {
      p.lse[idx] = mx + logf(sum);
      p.out_norm[idx] = on;
    }
    __syncthreads();
  }
}

template <int kR, typename T>
__global__ void __launch_bounds__(192, 1) route_fwd_kernel(const __grid_constant__ CUtensorMap tq,
                                                           const __grid_constant__ CUtensorMap tdk,
                                                           const __grid_constant__ CUtensorMap tdv,
                                                           const FwdParams p) {
  using C = FwdCfg<kR>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ uint64_t q_full, o_full;
  __shared__ uint64_t dk_full[C::kStages], dk_empty[C::kStages], dv_full[C::kStages], dv_empty[C::kStages];
  __shared__ uint64_t s_full[C::kB], p_full[C::kB], p_empty[C::kB];
  __shared__ uint32_t tmem_base;
  __shared__ int abort_flag, is_last;

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const uint32_t rank = cluster_ctarank() & 1u;
  const int pair = blockIdx.x / 2;
  const int tiles_per_group = (p.rows + 127) / 128;
  const int g = pair / tiles_per_group;
  const int row0 = (pair % tiles_per_group) * 128;  // first row of the pair inside the group
  const int NJ = p.M / C::kNA;
  Abort ab{&abort_flag, p.status};
  if (threadIdx.x == 0) trace_time(p.trace, 0);
  // fine post-mortem timeline of the first pair: 1024 ints per CTA after the 8-int slots
  int* ft = (p.trace && blockIdx.x < 2) ? p.trace + 8 * gridDim.x + blockIdx.x * 1024 : nullptr;

  if (threadIdx.x == 0) {
    abort_flag = 0;
    mbar_init(&q_full, 1);
    mbar_init(&o_full, 1);
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(&dk_full[s], 1);
      mbar_init(&dk_empty[s], 1);
      mbar_init(&dv_full[s], 1);
      mbar_init(&dv_empty[s], 1);
    }
    for (int b = 0; b < C::kB; ++b) {
      mbar_init(&s_full[b], 1);
      mbar_init(&p_full[b], 2);  // one arrival per CTA of the pair
      mbar_init(&p_empty[b], 1);
    }
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc<2>(&tmem_base, C::kTmemCols);
    tmem_relinquish<2>();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem = tmem_base;
  if (threadIdx.x == 0) trace_time(p.trace, 1);

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producers (both CTAs)
    // Lane 0 streams q and the key tiles, lane 1 the value tiles; the rings
    // advance independently so scores can run ahead of the P.Dv^T products.
    if (lane == 0) {
      prefetch_tmap(&tq);
      prefetch_tmap(&tdk);
      if (rank == 0) mbar_arrive_expect_tx(&q_full, 2 * C::kQBytes);
      const uint32_t qf = mapa_shared(smem_u32(&q_full), 0);
      const int qcol = g * p.col_stride;
      // Every box must overlap the tensor (a box wholly outside it may not
      // deliver its bytes); rows past the end are never stored.
      const int qrow = min(row0 + 64 * (int)rank, p.rows - 1);
      for (int kb = 0; kb < kR / 64; ++kb)
        tma_load_2d_pair(&tq, qf, smem + C::kOffQ + kb * (C::kRows * 128), qcol + kb * 64, qrow);
      int dk_issued = 0;
      for (int j = 0; j < NJ; ++j) {
        const int s = j % C::kStages;
        const uint32_t ph = (j / C::kStages) & 1u;
        if (!mbar_wait(&dk_empty[s], ph ^ 1u, ab, 11)) break;
        if (rank == 0) mbar_arrive_expect_tx(&dk_full[s], 2 * C::kDkBytes);
        const uint32_t kf = mapa_shared(smem_u32(&dk_full[s]), 0);
        for (int kb = 0; kb < kR / 64; ++kb)
          tma_load_2d_pair(&tdk, kf, smem + C::kOffDk + s * C::kDkBytes + kb * ((C::kNA / 2) * 128), kb * 64,
                           j * C::kNA + (C::kNA / 2) * (int)rank);
        dk_issued = j + 1;
      }
      if (rank == 0) {  // drain: the leader's barriers count both CTAs' bytes
        mbar_wait_drain(&q_full, 0);
        for (int j = (dk_issued > C::kStages ? dk_issued - C::kStages : 0); j < dk_issued; ++j)
          mbar_wait_drain(&dk_full[j % C::kStages], (j / C::kStages) & 1u);
      }
    } else if (lane == 1) {
      prefetch_tmap(&tdv);
      int dv_issued = 0;
      for (int j = 0; j < NJ; ++j) {
        const int s = j % C::kStages;
        const uint32_t ph = (j / C::kStages) & 1u;
        if (!mbar_wait(&dv_empty[s], ph ^ 1u, ab, 12)) break;
        if (rank == 0) mbar_arrive_expect_tx(&dv_full[s], 2 * C::kDvBytes);
        const uint32_t vf = mapa_shared(smem_u32(&dv_full[s]), 0);
        for (int i = 0; i < C::kPV; ++i)
          tma_load_2d_pair(&tdv, vf, smem + C::kOffDv + s * C::kDvBytes + i * ((C::kNc / 2) * 128), j * C::kNA,
                           i * C::kNc + (C::kNc / 2) * (int)rank);
        dv_issued = j + 1;
      }
      if (rank == 0)
        for (int j = (dv_issued > C::kStages ? dv_issued - C::kStages : 0); j < dv_issued; ++j)
          mbar_wait_drain(&dv_full[j % C::kStages], (j / C::kStages) & 1u);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (leader CTA)
    if (rank == 0 && lane == 0) {
      const uint32_t idesc_s = idesc_f16(128, C::kNA, std::is_same<T, __nv_bfloat16>::value, false, false);
      const uint32_t idesc_o = idesc_f16(128, C::kNc, true, false, false);
      bool ok = mbar_wait(&q_full, 0, ab, 21);
      tc_fence_after();
      auto commit_both = [&](uint64_t* bar) {
        mma_commit<2>(smem_u32(bar));
        mma_commit<2>(mapa_shared(smem_u32(bar), 1));
      };
      auto issue_s = [&](int j) -> bool {
        const int sb = j % C::kB, s = j % C::kStages;
        trace_at(ft, 100 + 2 * j);
        if (j >= C::kB && !mbar_wait(&p_full[sb], ((j - C::kB) / C::kB) & 1u, ab, 22)) return false;
        if (!mbar_wait(&dk_full[s], (j / C::kStages) & 1u, ab, 23)) return false;
        tc_fence_after();
        const uint32_t qa = smem_u32(smem + C::kOffQ), ka = smem_u32(smem + C::kOffDk + s * C::kDkBytes);
#pragma unroll 4
        for (int k = 0; k < kR / 16; ++k) {
          const int kb = k >> 2, kin = k & 3;
          const uint64_t ad = sdesc_sw128(qa + kb * (C::kRows * 128) + kin * 32, 16, 1024);
          const uint64_t bd = sdesc_sw128(ka + kb * ((C::kNA / 2) * 128) + kin * 32, 16, 1024);
          mma_f16_ss<2>(tmem + C::kTmemS + (uint32_t)sb * 32, ad, bd, idesc_s, k > 0 ? 1u : 0u);
        }
        commit_both(&s_full[sb]);
        commit_both(&dk_empty[s]);
        trace_at(ft, 101 + 2 * j);
        return true;
      };
      auto issue_pv = [&](int j) -> bool {
        const int pb = j % C::kB, s = j % C::kStages;
        trace_at(ft, 200 + 4 * j);
        if (!mbar_wait(&p_full[pb], (j / C::kB) & 1u, ab, 24)) return false;
        trace_at(ft, 201 + 4 * j);
        if (!mbar_wait(&dv_full[s], (j / C::kStages) & 1u, ab, 25)) return false;
        tc_fence_after();
        const uint32_t pa = smem_u32(smem + C::kOffP + pb * C::kPBytes);
        const uint32_t va = smem_u32(smem + C::kOffDv + s * C::kDvBytes);
#pragma unroll
        for (int i = 0; i < C::kPV; ++i) {
#pragma unroll
          for (int k = 0; k < C::kNA / 16; ++k) {
            const uint64_t ad = sdesc_sw128(pa + k * 32, 16, 1024);
            const uint64_t bd = sdesc_sw128(va + i * ((C::kNc / 2) * 128) + k * 32, 16, 1024);
            mma_f16_ss<2>(tmem + C::kTmemO + i * (C::kNc / 2), ad, bd, idesc_o, (j > 0 || k > 0) ? 1u : 0u);
          }
        }
        commit_both(&p_empty[pb]);
        commit_both(&dv_empty[s]);
        trace_at(ft, 202 + 4 * j);
        return true;
      };
      trace_time(p.trace, 2);
      // Scores run up to kB tiles ahead of the probability products.
      int next_s = 0;
      for (int j = 0; ok && j < NJ; ++j) {
        while (ok && next_s < NJ && next_s < j + C::kB) ok = issue_s(next_s++);
        if (ok) ok = issue_pv(j);
      }
      commit_both(&o_full);
      trace_time(p.trace, 3);
      mbar_wait_drain(&o_full, 0);  // every issued MMA has completed
    }
  } else {
    // ------------------------------------------------------------ softmax + epilogue (warps 2..5)
    const int quad = warp & 3;               // TMEM lane quadrant this warp may access
    const int l = quad * 32 + lane;          // TMEM lane
    const int r = l & 63, half = l >> 6;     // local row, which half of the tile columns
    const int grow = row0 + 64 * (int)rank + r;
    const uint32_t lane_base = (uint32_t)(quad * 32) << 16;
    float* red = reinterpret_cast<float*>(smem + C::kOffRed);
    const uint32_t pf_leader = mapa_shared(smem_u32(&p_full[0]), 0);
    const bool arriver = (warp == 2 && lane == 0);

    // q row norm from the staged q tile (S_0 complete implies q landed).
    bool ok = mbar_wait(&s_full[0], 0, ab, 31);
    if (arriver) trace_time(p.trace, 4);
    float qn2 = 0.f;
    if (ok) {
      const uint32_t qa = smem_u32(smem + C::kOffQ);
      for (int kb = 0; kb < kR / 64; ++kb) {
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const uint4 v = ld_shared_v4(qa + kb * (C::kRows * 128) + sw128_offset(r, c));
          const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 f = unpack2<T>(w[e]);
            qn2 = fmaf(f.x, f.x, fmaf(f.y, f.y, qn2));
          }
        }
      }
    }
    const float beta = *p.beta;
    const float qn = sqrtf(qn2);
    const float invn = p.normalize_input ? 1.f / fmaxf(qn, p.eps) : 1.f;
    const float kLog2e = 1.4426950408889634f;
    const float scale = beta * invn * kLog2e;                     // log2-domain multiplier of S
    const float bound = beta * qn * invn * (*p.dk_max) * kLog2e;  // >= every scaled score
    float sum = 0.f, mx = -INFINITY;
    int amax = 0;
    const bool want_argmax = p.argmax != nullptr;

    // Every thread runs every iteration (named barriers need all 128), even
    // after a failed wait; failed threads just skip the work.
    for (int j = 0; j < NJ; ++j) {
      const int sb = j % C::kB;
      if (arriver) trace_at(ft, 400 + 8 * j);
      if (ok && j > 0) ok = mbar_wait(&s_full[sb], (j / C::kB) & 1u, ab, 32);
      if (arriver) trace_at(ft, 401 + 8 * j);
      if (ok && j >= C::kB) ok = mbar_wait(&p_empty[sb], ((j - C::kB) / C::kB) & 1u, ab, 33);
      // tcgen05.ld is warp-collective: the whole warp loads or none of it.
      ok = __all_sync(0xffffffffu, ok);
      if (ok) {
        tc_fence_after();
        float v[32];
        tmem_ld32(tmem + lane_base + C::kTmemS + (uint32_t)sb * 32, v);
        tmem_wait_ld();
        if (arriver) trace_at(ft, 402 + 8 * j);
        uint32_t packed[16];
#pragma unroll
        for (int i = 0; i < 32; i += 2) {
          const float a = v[i] * scale, b = v[i + 1] * scale;
          if (want_argmax) {
            const int base = j * C::kNA + half * 32 + i;
            if (a > mx) amax = base;
            if (b > fmaxf(mx, a)) amax = base + 1;
          }
          mx = fmaxf(mx, fmaxf(a, b));
          const float ea = ex2(a - bound), eb = ex2(b - bound);
          sum += ea + eb;
          packed[i / 2] = pack_bf16x2(ea, eb);
        }
        const uint32_t pa = smem_u32(smem + C::kOffP + sb * C::kPBytes);
#pragma unroll
        for (int c = 0; c < 4; ++c)
          st_shared_v4(pa + sw128_offset(r, half * 4 + c), packed[4 * c], packed[4 * c + 1], packed[4 * c + 2],
                       packed[4 * c + 3]);
        if (arriver) trace_at(ft, 403 + 8 * j);
        fence_proxy_async();
        if (arriver) trace_at(ft, 404 + 8 * j);
      }
      tc_fence_before();
      named_bar_sync(1, 128);
      if (arriver) {
        trace_at(ft, 405 + 8 * j);
        mbar_arrive_cluster(pf_leader + sb * 8);
        trace_at(ft, 406 + 8 * j);
      }
    }

    if (arriver) trace_time(p.trace, 5);
    // ---- epilogue: combine the two column halves of each row, normalise, store.
    if (ok) ok = mbar_wait(&o_full, 0, ab, 34);
    ok = __all_sync(0xffffffffu, ok);
    if (arriver) trace_time(p.trace, 6);
    red[l] = sum;
    red[128 + l] = mx;
    named_bar_sync(1, 128);
    const float sum_all = sum + red[l ^ 64];
    const float mx_other = red[128 + (l ^ 64)];
    const float mx_all = fmaxf(mx, mx_other);
    named_bar_sync(1, 128);
    // argmax: the half holding the larger maximum wins (ties: lower index = half 0)
    int* ired = reinterpret_cast<int*>(red);
    ired[l] = amax;
    named_bar_sync(1, 128);
    const int amax_other = ired[l ^ 64];
    const int amax_all = (mx > mx_other || (mx == mx_other && half == 0)) ? amax : amax_other;
    named_bar_sync(1, 128);
    tc_fence_after();
    float ss = 0.f;
    if (ok) {
      for (int i = 0; i < C::kPV; ++i) {
        for (int c = 0; c < C::kNc / 2; c += 32) {
          float v[32];
          tmem_ld32(tmem + lane_base + C::kTmemO + i * (C::kNc / 2) + c, v);
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 32; ++e) ss = fmaf(v[e], v[e], ss);
        }
      }
    }
    red[l] = ss;
    named_bar_sync(1, 128);
    const float ss_all = ss + red[l ^ 64];
    const float onorm = sqrtf(ss_all);  // ||o|| where o = sum_all * r
    const float factor = p.normalize_output ? 1.f / fmaxf(onorm, p.eps * sum_all) : 1.f / sum_all;
    const bool live = grow < p.rows;
    if (ok) {  // warp-uniform: every lane loads, only rows that exist are stored
      T* zrow = reinterpret_cast<T*>(p.z) + ((size_t)g * p.rows + (live ? grow : 0)) * kR;
      for (int i = 0; i < C::kPV; ++i) {
        const int col0 = i * C::kNc + half * (C::kNc / 2);
        for (int c = 0; c < C::kNc / 2; c += 32) {
          float v[32];
          tmem_ld32(tmem + lane_base + C::kTmemO + i * (C::kNc / 2) + c, v);
          tmem_wait_ld();
          if (live) {
            uint32_t w[16];
#pragma unroll
            for (int e = 0; e < 16; ++e) w[e] = pack2<T>(v[2 * e] * factor, v[2 * e + 1] * factor);
            uint4* dst = reinterpret_cast<uint4*>(zrow + col0 + c);
#pragma unroll
            for (int e = 0; e < 4; ++e) dst[e] = make_uint4(w[4 * e], w[4 * e + 1], w[4 * e + 2], w[4 * e + 3]);
          }
        }
      }
    }
    if (ok && live) {
      if (half == 0) {
        const size_t idx = (size_t)g * p.rows + grow;
        const float kLn2 = 0.6931471805599453f;
        p.lse[idx] = (bound + log2f(sum_all)) * kLn2;
        p.out_norm[idx] = onorm / sum_all;
        if (want_argmax) p.argmax[idx] = amax_all;
        if (mx_all - bound < -100.f || !(sum_all > 0.f)) {
          const int slot = atomicAdd(&p.work[1], 1);
          if (slot < p.repair_cap) p.work[2 + slot] = (int)idx;
          else atomicOr(p.status, DA_DEV_ROW_OVERFLOW);
        }
      }
    }
  }

  tc_fence_before();
  __threadfence();
  __syncthreads();
  cluster_sync();
  if (warp == 1) tmem_dealloc<2>(tmem, C::kTmemCols);

  // The last CTA to finish repairs the listed rows and resets the counters.
  if (threadIdx.x == 0) is_last = atomicAdd(&p.work[0], 1) == (int)gridDim.x - 1;
  __syncthreads();
  if (is_last) {
    __threadfence();
    repair_listed_rows<kR, T>(p, reinterpret_cast<float*>(smem));
    __syncthreads();
    if (threadIdx.x == 0) {
      p.work[1] = 0;
      p.work[0] = 0;
      __threadfence();
    }
  }
  if (threadIdx.x == 0) trace_time(p.trace, 7);
}

template <int kR, typename T>
int launch_fwd(const RouteFwdArgs& a, cudaStream_t st) {
  using C = FwdCfg<kR>;
  const CUtensorMapDataType qdt = std::is_same<T, __nv_bfloat16>::value ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                                        : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  if ((a.M + kR + 64) * 4 > C::kSmem) return DA_ERR_SHAPE;  // repair scratch must fit
  CUtensorMap tq, tdk, tdv;
  int rc = make_tmap_2d(&tq, a.q, qdt, 2, a.q_cols, a.rows, (uint64_t)a.q_row_stride * 2, 64, 64);
  if (rc) return rc;
  rc = make_tmap_2d(&tdk, a.dk_t, qdt, 2, kR, a.M, (uint64_t)kR * 2, 64, C::kNA / 2);
  if (rc) return rc;
  rc = make_tmap_2d(&tdv, a.dv, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a.M, kR, (uint64_t)a.M * 2, 64, C::kNc / 2);
  if (rc) return rc;
  FwdParams p;
  p.q = a.q;
  p.q_row_stride = a.q_row_stride;
  p.dk_t = a.dk_t;
  p.dv = a.dv;
  p.rows = (int)a.rows;
  p.groups = a.groups;
  p.col_stride = (int)a.group_col_stride;
  p.M = (int)a.M;
  p.beta = a.beta;
  p.dk_max = a.dk_max;
  p.eps = a.eps;
  p.normalize_input = a.normalize_input;
  p.normalize_output = a.normalize_output;
  p.z = a.z;
  p.lse = a.lse;
  p.out_norm = a.out_norm;
  p.argmax = a.argmax;
  p.work = a.work;
  p.repair_cap = a.repair_cap;
  p.status = a.status;
  p.trace = debug_trace();
  auto kern = route_fwd_kernel<kR, T>;
  const int smem = C::kSmem + 1024;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
    return record_cuda_error();
  const long pairs = (long)a.groups * ((a.rows + 127) / 128);
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  cfg.gridDim = dim3((unsigned)(2 * pairs), 1, 1);
  cfg.blockDim = dim3(C::kThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, kern, tq, tdk, tdv, p) != cudaSuccess) return record_cuda_error();
  note_launch();
  return DA_OK;
}

int route_fwd(const RouteFwdArgs& a, cudaStream_t st) {
  const bool bf16 = a.dtype == DA_BF16;
  switch (a.R) {
    case 64: return bf16 ? launch_fwd<64, __nv_bfloat16>(a, st) : launch_fwd<64, __half>(a, st);
    case 128: return bf16 ? launch_fwd<128, __nv_bfloat16>(a, st) : launch_fwd<128, __half>(a, st);
    case 256: return bf16 ? launch_fwd<256, __nv_bfloat16>(a, st) : launch_fwd<256, __half>(a, st);
    case 512: return bf16 ? launch_fwd<512, __nv_bfloat16>(a, st) : launch_fwd<512, __half>(a, st);
    default: return DA_ERR_UNSUPPORTED;
  }
}

}  // namespace route
}  // namespace da

extern "C" int da_route_fwd(const void* q, int64_t rows, int64_t q_cols, int64_t q_row_stride, int groups,
                            int64_t group_col_stride, int64_t R, int64_t M, int dtype, const void* dict_key_t,
                            const void* dict_value, const float* beta, const float* dk_max, float eps,
                            int normalize_input, int normalize_output, void* z, float* lse, float* out_norm,
                            int* argmax, int* work, int repair_cap, int* status, void* stream) {
  using namespace da;
  if (!q || !dict_key_t || !dict_value || !beta || !dk_max || !z || !lse || !out_norm || !work || !status)
    return DA_ERR_NULL;
  if (int rc = bind_device(q)) return rc;
  if (dtype != DA_BF16 && dtype != DA_F16) return DA_ERR_DTYPE;
  if (rows <= 0 || groups <= 0 || M <= 0 || M % 64 || rows > (1ll << 30)) return DA_ERR_SHAPE;
  if (R != 64 && R != 128 && R != 256 && R != 512) return DA_ERR_UNSUPPORTED;
  if ((int64_t)(groups - 1) * group_col_stride + R > q_cols || q_row_stride < q_cols) return DA_ERR_SHAPE;
  if (group_col_stride % 64 || (reinterpret_cast<uintptr_t>(z) & 15)) return DA_ERR_ALIGN;
  if (repair_cap < 0) return DA_ERR_SHAPE;
  route::RouteFwdArgs a{q, rows, q_cols, q_row_stride, groups, group_col_stride, R, M, dtype, dict_key_t,
                        dict_value, beta, dk_max, eps, normalize_input, normalize_output, z, lse, out_norm,
                        argmax, work, repair_cap, status};
  return route::route_fwd(a, static_cast<cudaStream_t>(stream));
}
