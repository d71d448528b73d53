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
  int compact;          // wide kernel: the two-CTAs-per-SM layout (see wide_layout)
  int coarse;           // wide kernel: tile plan for more pairs than SMs (see wide_layout)
};

// Exact fp32 recomputation of `count` listed rows (global indices g * rows + row) by one CTA (rare path).
template <int kR, typename T>
__device__ void repair_rows(const FwdParams& p, const int* list, int count, float* buf) {
  const int nthr = blockDim.x, tid = threadIdx.x;
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
    const int idx = list[it];
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
  // Pairs start at different atom tiles (and wrap around), so the CTAs of a
  // wave do not all read the same dictionary lines from L2 at once.
  const int rot = pair % NJ;
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
  grid_dependency_wait();  // predecessors' outputs are visible from here on
  grid_launch_dependents();
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
        trace_at(ft, 700 + j);
        if (rank == 0) mbar_arrive_expect_tx(&dk_full[s], 2 * C::kDkBytes);
        const uint32_t kf = mapa_shared(smem_u32(&dk_full[s]), 0);
        for (int kb = 0; kb < kR / 64; ++kb)
          tma_load_2d_pair(&tdk, kf, smem + C::kOffDk + s * C::kDkBytes + kb * ((C::kNA / 2) * 128), kb * 64,
                           ((j + rot) % NJ) * C::kNA + (C::kNA / 2) * (int)rank);
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
          tma_load_2d_pair(&tdv, vf, smem + C::kOffDv + s * C::kDvBytes + i * ((C::kNc / 2) * 128), ((j + rot) % NJ) * C::kNA,
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
      auto commit_both = [&](uint64_t* bar) { mma_commit_pair(smem_u32(bar)); };
      auto issue_s = [&](int j) -> bool {
        const int sb = j % C::kB, s = j % C::kStages;
        trace_at(ft, 100 + 2 * j);
        if (j >= C::kB && !mbar_wait(&p_full[sb], ((j - C::kB) / C::kB) & 1u, ab, 22)) return false;
        if (!mbar_wait(&dk_full[s], (j / C::kStages) & 1u, ab, 23)) return false;
        trace_at(ft, 600 + j);
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
            // first index of the maximum, whatever order the tiles were visited in
            const int base = ((j + rot) % NJ) * C::kNA + half * 32 + i;
            if (a > mx || (a == mx && base < amax)) amax = base;
            const float ma = fmaxf(mx, a);
            if (b > ma || (b == ma && base + 1 < amax)) amax = base + 1;
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
        mbar_arrive_remote(pf_leader + sb * 8);
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
    // argmax: the half holding the larger maximum wins (ties: the lower index)
    int* ired = reinterpret_cast<int*>(red);
    ired[l] = amax;
    named_bar_sync(1, 128);
    const int amax_other = ired[l ^ 64];
    const int amax_all = mx > mx_other ? amax : (mx < mx_other ? amax_other : min(amax, amax_other));
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
    repair_rows<kR, T>(p, p.work + 2, min(p.work[1], p.repair_cap), reinterpret_cast<float*>(smem));
    __syncthreads();
    if (threadIdx.x == 0) {
      p.work[1] = 0;
      p.work[0] = 0;
      __threadfence();
    }
  }
  if (threadIdx.x == 0) trace_time(p.trace, 7);
}

// ============================================================================
// Wide-tile variant (R = 128 / 256 / 512, M a multiple of 128).
//
// The paired MMA only reaches full rate with N = 256 (each instruction costs
// ~46 cycles to issue whatever its N), and the 64-atom tiles above issue 16
// small score instructions per tile.  Here a pair scores 128 or 256 atoms per
// tile (N = nk) with the key rows streamed as 64-column K chunks through one
// ring and the value rows as 64-atom K chunks through another, exactly like
// the outer attention's single-map kernel; the epilogue (statistics, output
// normalisation, exact repair of low-mass rows) is the one above.
struct WideLayout {
  int nk, kchunks, nc, npv;
  int kbb, kslots;  // key chunks per TMA box, ring slots of kbb chunks
  int q_bytes, k_stage, v_stage, p_bytes;
  int nks, nvs, nsb, npb;
  int off_q, off_k, off_v, off_p, off_red, smem;
  int tmem_s, s_cols, tmem_cols;
};

constexpr int kWideMaxK = 8, kWideMaxV = 4, kWideMaxSB = 4, kWideMaxPB = 2;
// warp0 keys, warp1 score MMAs, warps2-5 softmax/epilogue, warp6 values, warp7 P.Dv^T MMAs, and in
// the one-CTA-per-SM layout warps 8 and 9 as second key and value producers.  The two products have
// their own issuing threads, so a P.Dv^T product never waits behind the key chunks of a score tile
// further ahead (and the reverse).  One warp's TMA stages complete one after another (about 1 us
// per stage for paired loads, nearly whatever the stage's size), so stages are as large as the
// rings allow and, where registers permit, each stream has two producers taking alternate stages.
constexpr int kValueWarp = 6;
constexpr int kPvWarp = 7;
constexpr int kKeyWarp2 = 8, kValueWarp2 = 9;
// kLat: the latency layout for fewer pairs than SMs (one producer per stream, one interleaved MMA
// issuer, probabilities stored chunk by chunk), warps 0-6 only.
template <int kMinBlocks, bool kLat>
constexpr int wide_threads() { return kLat ? 224 : (kMinBlocks == 2 ? 256 : 320); }

// compact: a layout two CTAs of which fit one SM (<= 256 TMEM columns, ~108 KB of shared memory),
// so that one pair's serial chain (setup, scores, softmax, epilogue) overlaps another's when there
// are more pairs than SMs; 128-atom tiles and shorter rings.
// coarse: more pairs than SMs (throughput-bound): key boxes of up to 32 KB; with fewer pairs every
// pair has few atom tiles and 16 KB boxes let the first products start sooner.
__host__ __device__ inline WideLayout wide_layout(int R, int M, bool compact = false, bool coarse = true) {
  WideLayout L;
  L.kchunks = R / 64;
  L.nc = R < 256 ? R : 256;
  L.npv = R / L.nc;
  L.q_bytes = 64 * R * 2;
  L.v_stage = (R / 2) * 128;  // this CTA's R/2 value rows x 64 atoms
  const int red = 2 * 128 * 4;
  const int avail = compact ? 108 * 1024 : 225 * 1024;
  L.nk = 0;
  for (int nk = (M % 256 == 0 && !compact) ? 256 : 128; nk >= 128 && L.nk == 0; nk -= 128) {
    if (M % nk) continue;
    for (int npb = 2; npb >= 1 && L.nk == 0; --npb) {
      const int k_stage = (nk / 2) * 128, p_bytes = 64 * nk * 2;
      const int rest = avail - L.q_bytes - npb * p_bytes - 2 * L.v_stage - red;
      if (rest >= 3 * k_stage) {
        L.nk = nk;
        L.k_stage = k_stage;
        L.p_bytes = p_bytes;
        L.npb = npb;
        L.nvs = 2;
        L.nks = rest / k_stage > kWideMaxK ? kWideMaxK : rest / k_stage;
      }
    }
  }
  if (L.nk == 0) {
    L.nk = 0;  // caller falls back to the 64-atom kernel
    L.nks = 0;
    L.smem = 0;
    return L;
  }
  // several 64-column key chunks of the same atoms per box (<= 32 KB), keeping at least two slots
  L.kbb = 1;
  for (int b = 4; b >= 2; b /= 2)
    if (L.kchunks % b == 0 && L.nks / b >= 2 && b * L.k_stage <= (coarse ? 32768 : 16384)) {
      L.kbb = b;
      break;
    }
  L.kslots = L.nks / L.kbb;
  L.nks = L.kslots * L.kbb;
  L.s_cols = L.nk / 2;
  L.tmem_s = R / 2;
  const int nsb = ((compact ? 256 : 512) - R / 2) / L.s_cols;
  L.nsb = nsb > kWideMaxSB ? kWideMaxSB : nsb;
  L.off_q = 0;
  L.off_k = L.off_q + L.q_bytes;
  L.off_v = L.off_k + L.nks * L.k_stage;
  L.off_p = L.off_v + L.nvs * L.v_stage;
  L.off_red = L.off_p + L.npb * L.p_bytes;
  const int used = L.off_red + red;
  L.smem = (used < 120 * 1024 && !compact) ? 120 * 1024 : used;  // one CTA per SM unless compact
  const int cols = R / 2 + L.nsb * L.s_cols;
  L.tmem_cols = cols <= 128 ? 128 : (cols <= 256 ? 256 : 512);
  return L;
}

template <int kR, typename T, int kMinBlocks, bool kLat>
__global__ void __launch_bounds__(wide_threads<kMinBlocks, kLat>(), kMinBlocks) route_fwd_wide_kernel(const __grid_constant__ CUtensorMap tq,
                                                                const __grid_constant__ CUtensorMap tdk,
                                                                const __grid_constant__ CUtensorMap tdv,
                                                                const FwdParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ uint64_t q_full, o_full;
  __shared__ uint64_t k_full[kWideMaxK], k_empty[kWideMaxK], v_full[kWideMaxV], v_empty[kWideMaxV];
  __shared__ uint64_t s_full[kWideMaxSB], p_full[kWideMaxSB], p_empty[kWideMaxPB];
  __shared__ uint32_t tmem_base;
  __shared__ int abort_flag, n_listed;
  __shared__ int listed[64];  // this CTA's rows whose mass fell below the fixed offset's range

  const WideLayout L = wide_layout(kR, p.M, p.compact != 0, p.coarse != 0);
  constexpr int kRows = 64;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const uint32_t rank = cluster_ctarank() & 1u;
  const int pair = blockIdx.x / 2;
  const int tiles_per_group = (p.rows + 127) / 128;
  const int g = pair / tiles_per_group;
  const int row0 = (pair % tiles_per_group) * 128;
  const int nk = L.nk;
  const int NJ = p.M / nk;
  const int rot = pair % NJ;  // pairs start at different atom tiles
  Abort ab{&abort_flag, p.status};
  if (threadIdx.x == 0) trace_time(p.trace, 0);
  // post-mortem per-tile timeline of the first pair (debug trace only): 4096 ints per CTA after the 8-int slots
  int* ft = (p.trace && blockIdx.x < 2) ? p.trace + 8 * gridDim.x + blockIdx.x * 4096 : nullptr;

  if (threadIdx.x == 0) {
    abort_flag = 0;
    n_listed = 0;
    mbar_init(&q_full, 1);
    mbar_init(&o_full, 1);
    for (int i = 0; i < kWideMaxK; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
    }
    for (int i = 0; i < kWideMaxV; ++i) {
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
    }
    for (int i = 0; i < kWideMaxSB; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 2);
    }
    for (int i = 0; i < kWideMaxPB; ++i) mbar_init(&p_empty[i], 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc<2>(&tmem_base, L.tmem_cols);
    tmem_relinquish<2>();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();
  tc_fence_after();
  grid_dependency_wait();  // predecessors' outputs are visible from here on
  grid_launch_dependents();
  const uint32_t tmem = tmem_base;
  if (threadIdx.x == 0) trace_time(p.trace, 1);

  constexpr int kProducers = (kMinBlocks == 2 || kLat) ? 1 : 2;  // per stream
  if (warp == 0 || (kProducers == 2 && warp == kKeyWarp2)) {
    // ---------------------------------------------------------------- key producers (both CTAs): warp 0
    // loads q and the even key boxes, warp 8 (if present) the odd ones
    if (lane == 0) {
      const int pi = warp == 0 ? 0 : 1;
      prefetch_tmap(&tdk);
      if (pi == 0) {
        prefetch_tmap(&tq);
        if (rank == 0) mbar_arrive_expect_tx(&q_full, 2 * L.q_bytes);
        const uint32_t qf = mapa_shared(smem_u32(&q_full), 0);
        const int qrow = min(row0 + 64 * (int)rank, p.rows - 1);  // boxes never start outside the matrix
        for (int kb = 0; kb < kR / 64; ++kb)
          tma_load_2d_pair(&tq, qf, smem + L.off_q + kb * (kRows * 128), g * p.col_stride + kb * 64, qrow);
      }
      const int box_bytes = L.kbb * L.k_stage;
      int kx = 0;  // key boxes of all producers
      bool ok = true;
      for (int j = 0; ok && j < NJ; ++j) {
        const int jj = (j + rot) % NJ;
        for (int c = 0; c < L.kchunks; c += L.kbb, ++kx) {
          if (kx % kProducers != pi) continue;
          const int st = kx % L.kslots;
          if (!mbar_wait(&k_empty[st], ((kx / L.kslots) & 1u) ^ 1u, ab, 11)) { ok = false; break; }
          if (rank == 0) mbar_arrive_expect_tx(&k_full[st], 2 * box_bytes);
          tma_load_3d_pair(&tdk, mapa_shared(smem_u32(&k_full[st]), 0), smem + L.off_k + st * box_bytes, 0,
                           jj * nk + (int)rank * (nk / 2), c);
        }
      }
      if (rank == 0) {  // drain: none of this producer's loads may be in flight at teardown
        if (pi == 0) mbar_wait_drain(&q_full, 0);
        for (int c = (kx > L.kslots ? kx - L.kslots : 0); c < kx; ++c)
          if (c % kProducers == pi) mbar_wait_drain(&k_full[c % L.kslots], (c / L.kslots) & 1u);
      }
    }
  } else if (warp == kValueWarp || (kProducers == 2 && warp == kValueWarp2)) {
    // ---------------------------------------------------------------- value producers: this CTA's R/2
    // value rows of every N block, 64 atoms per stage, one box per stage
    if (lane == 0) {
      const int pi = warp == kValueWarp ? 0 : 1;
      prefetch_tmap(&tdv);
      int vc = 0;
      bool ok = true;
      for (int j = 0; ok && j < NJ; ++j) {
        const int jj = (j + rot) % NJ;
        for (int c = 0; c < nk / 64; ++c, ++vc) {
          if (vc % kProducers != pi) continue;
          const int st = vc % L.nvs;
          if (!mbar_wait(&v_empty[st], ((vc / L.nvs) & 1u) ^ 1u, ab, 12)) { ok = false; break; }
          if (rank == 0) mbar_arrive_expect_tx(&v_full[st], 2 * L.v_stage);
          tma_load_3d_pair(&tdv, mapa_shared(smem_u32(&v_full[st]), 0), smem + L.off_v + st * L.v_stage,
                           jj * nk + c * 64, (int)rank * (L.nc / 2), 0);
        }
      }
      if (rank == 0)
        for (int c = (vc > L.nvs ? vc - L.nvs : 0); c < vc; ++c)
          if (c % kProducers == pi) mbar_wait_drain(&v_full[c % L.nvs], (c / L.nvs) & 1u);
    }
  } else if (warp == 1 || warp == kPvWarp) {
    // ---------------------------------------------------------------- MMA issuers (leader): scores on
    // warp 1, probability products on warp 7
    if (rank == 0 && lane == 0) {
      const uint32_t idesc_s = idesc_f16(128, nk, std::is_same<T, __nv_bfloat16>::value, false, false);
      const uint32_t idesc_o = idesc_f16(128, L.nc, true, false, false);  // Dv rows are K-major (atoms contiguous)
      auto commit_both = [&](uint64_t* bar) { mma_commit_pair(smem_u32(bar)); };
      const uint32_t qa = smem_u32(smem + L.off_q);
      int kx = 0, kst = 0, vc = 0;  // key boxes consumed and current key slot; value stages consumed
      auto issue_s = [&](int j) -> bool {  // S_j = q . Dk_j into score buffer j % nsb
        const int sb = j % L.nsb;
        if (j < 256) trace_at(ft, 1024 + 4 * j);
        if (j >= L.nsb && !mbar_wait(&p_full[sb], ((j - L.nsb) / L.nsb) & 1u, ab, 22)) return false;
        if (j < 256) trace_at(ft, 1025 + 4 * j);
        const uint32_t d = tmem + L.tmem_s + (uint32_t)(sb * L.s_cols);
        for (int c = 0; c < L.kchunks; ++c) {
          const int cib = c % L.kbb;  // chunk inside the current box
          if (cib == 0) {
            kst = kx % L.kslots;
            if (!mbar_wait(&k_full[kst], (kx / L.kslots) & 1u, ab, 23)) return false;
            tc_fence_after();
          }
          const uint64_t ad0 = sdesc_sw128(qa + c * (kRows * 128), 16, 1024);
          const uint64_t bd0 = sdesc_sw128(smem_u32(smem + L.off_k + (kst * L.kbb + cib) * L.k_stage), 16, 1024);
#pragma unroll
          for (int kin = 0; kin < 4; ++kin)  // +32 B per K step of 16 = +2 in the encoded address
            mma_f16_ss<2>(d, ad0 + 2 * kin, bd0 + 2 * kin, idesc_s, (c | kin) ? 1u : 0u);
          if (cib == L.kbb - 1) {
            commit_both(&k_empty[kst]);
            ++kx;
          }
        }
        commit_both(&s_full[sb]);
        if (j < 256) trace_at(ft, 1026 + 4 * j);
        return true;
      };
      // P_j . Dv_j^T once probability tile j and its value rows are in shared memory.  The wait on
      // p_full[j % nsb] cannot alias a later phase: tile j + nsb's probabilities need P buffer
      // (j + nsb) % npb back, i.e. the product of tile j + nsb - npb >= j (nsb >= npb).
      auto issue_pv = [&](int j) -> bool {
        const int pb = j % L.npb;
        if (j < 256) trace_at(ft, 2048 + 4 * j);
        if (!mbar_wait(&p_full[j % L.nsb], (j / L.nsb) & 1u, ab, 24)) return false;
        if (j < 256) trace_at(ft, 2049 + 4 * j);
        const uint32_t pa = smem_u32(smem + L.off_p + pb * L.p_bytes);
        for (int c = 0; c < nk / 64; ++c, ++vc) {
          const int st = vc % L.nvs;
          if (!mbar_wait(&v_full[st], (vc / L.nvs) & 1u, ab, 25)) return false;
          tc_fence_after();
          const uint32_t va = smem_u32(smem + L.off_v + st * L.v_stage);
          const uint64_t ad0 = sdesc_sw128(pa + c * (kRows * 128), 16, 1024);
          for (int i = 0; i < L.npv; ++i) {
            const uint64_t bd0 = sdesc_sw128(va + i * ((L.nc / 2) * 128), 16, 1024);
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
              mma_f16_ss<2>(tmem + (uint32_t)(i * (L.nc / 2)), ad0 + 2 * kk, bd0 + 2 * kk, idesc_o,
                            (j | c | kk) ? 1u : 0u);
          }
          commit_both(&v_empty[st]);
        }
        commit_both(&p_empty[pb]);
        if (j < 256) trace_at(ft, 2050 + 4 * j);
        return true;
      };
      bool ok = mbar_wait(&q_full, 0, ab, 21);
      if (warp == 1) trace_time(p.trace, 2);
      tc_fence_after();
      if (!kLat) {
        // many pairs per SM: the two products from their own threads, so neither waits behind the
        // other's operand stream
        if (warp == 1) {
          for (int j = 0; ok && j < NJ; ++j) ok = issue_s(j);
          trace_time(p.trace, 3);
        } else {
          for (int j = 0; ok && j < NJ; ++j) ok = issue_pv(j);
          commit_both(&o_full);
          mbar_wait_drain(&o_full, 0);  // every probability product (and so every score product) has completed
        }
      } else if (warp == 1) {
        // a few atom tiles per pair: one thread, scores up to nsb tiles ahead of the products
        int next_s = 0;
        for (int j = 0; ok && j < NJ; ++j) {
          while (ok && next_s < NJ && next_s < j + L.nsb) ok = issue_s(next_s++);
          if (ok) ok = issue_pv(j);
        }
        commit_both(&o_full);
        trace_time(p.trace, 3);
        mbar_wait_drain(&o_full, 0);
      }
    }
  } else {
    // ---------------------------------------------------------------- softmax + epilogue (warps 2..5)
    const int quad = warp & 3;
    const int l = quad * 32 + lane;
    const int r = l & 63, half = l >> 6;
    const int grow = row0 + 64 * (int)rank + r;
    const uint32_t lane_base = (uint32_t)(quad * 32) << 16;
    float* red = reinterpret_cast<float*>(smem + L.off_red);
    const uint32_t pf_leader = mapa_shared(smem_u32(&p_full[0]), 0);
    const bool arriver = (warp == 2 && lane == 0);
    const int hc = nk / 2;  // atoms of a tile per thread

    bool ok = mbar_wait(&s_full[0], 0, ab, 31);  // S_0 complete: the q tile has landed
    if (arriver) trace_time(p.trace, 4);
    float qn2 = 0.f;
    if (ok) {
      const uint32_t qa = smem_u32(smem + L.off_q);
      for (int kb = 0; kb < kR / 64; ++kb)
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const uint4 v = ld_shared_v4(qa + kb * (kRows * 128) + sw128_offset(r, c));
          const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 f = unpack2<T>(w[e]);
            qn2 = fmaf(f.x, f.x, fmaf(f.y, f.y, qn2));
          }
        }
    }
    const float beta = *p.beta;
    const float qn = sqrtf(qn2);
    const float invn = p.normalize_input ? 1.f / fmaxf(qn, p.eps) : 1.f;
    const float kLog2e = 1.4426950408889634f;
    const float scale = beta * invn * kLog2e;
    const float bound = beta * qn * invn * (*p.dk_max) * kLog2e;
    float sum = 0.f, mx = -INFINITY;
    int amax = 0;
    const bool want_argmax = p.argmax != nullptr;

    // A tile's probabilities are formed in registers first and stored once the P buffer is free, so
    // with a single P buffer the softmax of tile j + 1 overlaps the product of tile j.
    constexpr int kMaxCh = kMinBlocks == 2 ? 2 : 4;  // 32-atom chunks per thread per tile (compact: nk = 128)
    const int nch = hc / 32;
    for (int j = 0; j < NJ; ++j) {
      const int sb = j % L.nsb, pb = j % L.npb;
      const int jj = (j + rot) % NJ;
      if (arriver && j < 256) trace_at(ft, 3072 + 4 * j);
      if (ok && j > 0) ok = mbar_wait(&s_full[sb], (j / L.nsb) & 1u, ab, 32);
      if (arriver && j < 256) trace_at(ft, 3073 + 4 * j);
      if (kLat && ok && j >= L.npb) ok = mbar_wait(&p_empty[pb], ((j - L.npb) / L.npb) & 1u, ab, 33);
      ok = __all_sync(0xffffffffu, ok);  // tcgen05.ld is warp-collective
      if constexpr (kLat) {  // P buffer already free: each 32-atom chunk is stored as soon as it is formed
        if (ok) {
          tc_fence_after();
          const uint32_t pa = smem_u32(smem + L.off_p + pb * L.p_bytes);
          for (int ch = 0; ch < nch; ++ch) {
            float v[32];
            tmem_ld32(tmem + lane_base + L.tmem_s + (uint32_t)(sb * L.s_cols + ch * 32), v);
            tmem_wait_ld();
            const int kc = half * hc + ch * 32;
            uint32_t pk[16];
#pragma unroll
            for (int i = 0; i < 32; i += 2) {
              const float a = v[i] * scale, b = v[i + 1] * scale;
              if (want_argmax) {
                const int base = jj * nk + kc + i;
                if (a > mx || (a == mx && base < amax)) amax = base;
                const float ma = fmaxf(mx, a);
                if (b > ma || (b == ma && base + 1 < amax)) amax = base + 1;
              }
              mx = fmaxf(mx, fmaxf(a, b));
              const float ea = ex2(a - bound), eb = ex2(b - bound);
              sum += ea + eb;
              pk[i / 2] = pack_bf16x2(ea, eb);
            }
            const uint32_t box = pa + (kc >> 6) * (kRows * 128);
            const int cb = (kc & 63) >> 3;
#pragma unroll
            for (int e = 0; e < 4; ++e)
              st_shared_v4(box + sw128_offset(r, cb + e), pk[4 * e], pk[4 * e + 1], pk[4 * e + 2], pk[4 * e + 3]);
          }
          fence_proxy_async();
        }
        tc_fence_before();
        named_bar_sync(1, 128);
        if (arriver) mbar_arrive_remote(pf_leader + sb * 8);
        continue;
      }
      uint32_t packed[kMaxCh][16];
      if (ok) {
        tc_fence_after();
#pragma unroll
        for (int ch = 0; ch < kMaxCh; ++ch) {
          if (ch < nch) {
            float v[32];
            tmem_ld32(tmem + lane_base + L.tmem_s + (uint32_t)(sb * L.s_cols + ch * 32), v);
            tmem_wait_ld();
            const int kc = half * hc + ch * 32;  // atom column inside the tile
#pragma unroll
            for (int i = 0; i < 32; i += 2) {
              const float a = v[i] * scale, b = v[i + 1] * scale;
              if (want_argmax) {  // first index of the maximum, whatever the visiting order
                const int base = jj * nk + kc + i;
                if (a > mx || (a == mx && base < amax)) amax = base;
                const float ma = fmaxf(mx, a);
                if (b > ma || (b == ma && base + 1 < amax)) amax = base + 1;
              }
              mx = fmaxf(mx, fmaxf(a, b));
              const float ea = ex2(a - bound), eb = ex2(b - bound);
              sum += ea + eb;
              packed[ch][i / 2] = pack_bf16x2(ea, eb);
            }
          }
        }
      }
      if (ok && j >= L.npb) ok = mbar_wait(&p_empty[pb], ((j - L.npb) / L.npb) & 1u, ab, 33);
      if (arriver && j < 256) trace_at(ft, 3074 + 4 * j);
      ok = __all_sync(0xffffffffu, ok);
      if (ok) {
        const uint32_t pa = smem_u32(smem + L.off_p + pb * L.p_bytes);
#pragma unroll
        for (int ch = 0; ch < kMaxCh; ++ch) {
          if (ch < nch) {
            const int kc = half * hc + ch * 32;
            const uint32_t box = pa + (kc >> 6) * (kRows * 128);
            const int cb = (kc & 63) >> 3;
#pragma unroll
            for (int e = 0; e < 4; ++e)
              st_shared_v4(box + sw128_offset(r, cb + e), packed[ch][4 * e], packed[ch][4 * e + 1],
                           packed[ch][4 * e + 2], packed[ch][4 * e + 3]);
          }
        }
        fence_proxy_async();
      }
      tc_fence_before();
      named_bar_sync(1, 128);
      if (arriver) mbar_arrive_remote(pf_leader + sb * 8);
      if (arriver && j < 256) trace_at(ft, 3075 + 4 * j);
    }

    // ---- epilogue: combine the two column halves of each row, normalise, store.
    if (arriver) trace_time(p.trace, 5);
    if (ok) ok = mbar_wait(&o_full, 0, ab, 34);
    if (arriver) trace_time(p.trace, 6);
    ok = __all_sync(0xffffffffu, ok);
    red[l] = sum;
    red[128 + l] = mx;
    named_bar_sync(1, 128);
    const float sum_all = sum + red[l ^ 64];
    const float mx_other = red[128 + (l ^ 64)];
    const float mx_all = fmaxf(mx, mx_other);
    named_bar_sync(1, 128);
    int* ired = reinterpret_cast<int*>(red);
    ired[l] = amax;
    named_bar_sync(1, 128);
    const int amax_other = ired[l ^ 64];
    const int amax_all = mx > mx_other ? amax : (mx < mx_other ? amax_other : min(amax, amax_other));
    named_bar_sync(1, 128);
    tc_fence_after();
    float ss = 0.f;
    if (ok) {
      for (int i = 0; i < L.npv; ++i)
        for (int c = 0; c < L.nc / 2; c += 32) {
          float v[32];
          tmem_ld32(tmem + lane_base + (uint32_t)(i * (L.nc / 2) + c), v);
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 32; ++e) ss = fmaf(v[e], v[e], ss);
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
      for (int i = 0; i < L.npv; ++i) {
        const int col0 = i * L.nc + half * (L.nc / 2);
        for (int c = 0; c < L.nc / 2; c += 32) {
          float v[32];
          tmem_ld32(tmem + lane_base + (uint32_t)(i * (L.nc / 2) + c), v);
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
    if (ok && live && half == 0) {
      const size_t idx = (size_t)g * p.rows + grow;
      const float kLn2 = 0.6931471805599453f;
      p.lse[idx] = (bound + log2f(sum_all)) * kLn2;
      p.out_norm[idx] = onorm / sum_all;
      if (want_argmax) p.argmax[idx] = amax_all;
      if (mx_all - bound < -100.f || !(sum_all > 0.f)) listed[atomicAdd(&n_listed, 1)] = (int)idx;
    }
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync();
  if (warp == 1) tmem_dealloc<2>(tmem, L.tmem_cols);

  // This CTA recomputes its own listed rows exactly (rare); the pipeline's shared memory is free now.
  if (n_listed > 0) repair_rows<kR, T>(p, listed, n_listed, reinterpret_cast<float*>(smem));
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
  const long pairs = (long)a.groups * ((a.rows + 127) / 128);
  // two CTAs per SM when every SM gets several pairs and the compact layout exists for this shape
  const WideLayout Wc = wide_layout(kR, (int)a.M, true);
  // (the compact kernel holds a tile's probabilities for nk = 128 in registers; both layouts need
  // nsb >= npb, see the probability-product issuer)
  const bool compact = kR >= 128 && kR <= 256 && pairs >= sm_count() && Wc.nk == 128 && Wc.nks >= 3 && Wc.nsb >= 2 &&
                       Wc.nsb >= Wc.npb && Wc.tmem_cols <= 256;
  p.compact = compact ? 1 : 0;
  const bool coarse = pairs >= sm_count();
  p.coarse = coarse ? 1 : 0;
  const WideLayout W = compact ? wide_layout(kR, (int)a.M, true, coarse) : wide_layout(kR, (int)a.M, false, coarse);
  const bool wide = kR >= 128 && W.nk != 0 && W.nks >= 3 && W.nsb >= 2 && W.nsb >= W.npb;
  if (wide) {  // re-encode the key / value maps with the wide tile's boxes
    {  // keys Dk^T [M, R]: (64-column block, atom, block index); a box is nk/2 atoms x kbb blocks
      const uint64_t dims[3] = {64, (uint64_t)a.M, (uint64_t)kR / 64};
      const uint64_t strides[2] = {(uint64_t)kR * 2, 128};
      const uint32_t box[3] = {64, (uint32_t)(W.nk / 2), (uint32_t)W.kbb};
      rc = make_tmap_blocks(&tdk, a.dk_t, qdt, 2, 3, dims, strides, box);
      if (rc) return rc;
    }
    {  // values Dv [R, M]: (64 atoms, row inside an nc-row group, group); a box is 64 atoms x this
       // CTA's nc/2 rows of each of the npv groups
      const uint64_t dims[3] = {(uint64_t)a.M, (uint64_t)W.nc, (uint64_t)kR / W.nc};
      const uint64_t strides[2] = {(uint64_t)a.M * 2, (uint64_t)W.nc * a.M * 2};
      const uint32_t box[3] = {64, (uint32_t)(W.nc / 2), (uint32_t)W.npv};
      rc = make_tmap_blocks(&tdv, a.dv, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, 3, dims, strides, box);
      if (rc) return rc;
    }
    if ((a.M + kR + 64) * 4 > W.smem) return DA_ERR_SHAPE;  // repair scratch must fit
  }
  const bool lat = !compact && !coarse;
  auto kern = !wide ? route_fwd_kernel<kR, T>
                    : (compact ? route_fwd_wide_kernel<kR, T, 2, false>
                               : (lat ? route_fwd_wide_kernel<kR, T, 1, true> : route_fwd_wide_kernel<kR, T, 1, false>));
  const int smem = (wide ? W.smem : C::kSmem) + 1024;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
    return record_cuda_error();
  const int threads = !wide ? C::kThreads
                            : (compact ? wide_threads<2, false>() : (lat ? wide_threads<1, true>() : wide_threads<1, false>()));
  return launch_kernel(kern, dim3((unsigned)(2 * pairs), 1, 1), dim3(threads, 1, 1), smem, st, true, tq, tdk, tdv, p);
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
