// Dictionary route, backward: the dictionary gradients and the temperature gradient.
//
// Reference: the two dictionary-gradient GEMMs of _DictionaryRouteFunction.backward
// (triton_kernels.py:1706-1707 in the fused path, :1938-1961 in the multi-kernel
// path: grad_reconstructed^T @ weights and normalized^T @ grad_logits) and its
// per-row beta gradient (:1447-1501), with the math of ops.py:16-62.  Per route
// row (q_hat = invn q, P = softmax(beta q_hat.Dk), g = d r, delta = <P, dP>):
//   dDv  = sum_rows g (x) P
//   dDk  = sum_rows q (x) dL',   dL' = invn beta P (dP - delta),   dP = g.Dv
//   dbeta = sum_rows sum_atoms (q_hat.dk) P (dP - delta)
// The reference materialises P and the logit gradient as [rows, M] tensors and
// multiplies them on cuBLAS.  Here nothing of size [rows, M] reaches memory:
//
// One CTA pair (2-CTA cluster, cta_group::2 MMAs) owns one tile of 128 atoms
// (64 per CTA) and a contiguous chunk of route-row tiles.  The pair's Dk and
// Dv rows stay resident in shared memory; per row tile it streams q and g
// (the output-normalisation gradient the row-parallel kernel stored) and
//   * recomputes S^T = Dk_tile q^T and dP^T = Dv_tile g^T into TMEM
//     (double-buffered; M = atoms, N = rows);
//   * the softmax warpgroup rebuilds P from the forward's log-sum-exp, forms
//     dL', writes P^T and dL'^T (one row of atoms per thread) to shared memory
//     and accumulates dbeta;
//   * dDv^T += P^T g and dDk^T += dL'^T q accumulate in TMEM over the chunk.
// Each pair then stores its [128 atoms, R] partial sums; a second kernel adds
// the chunks' partials in a fixed order (deterministic) and writes dDk, dDv
// in the [R, M] layout of the dictionaries, and dbeta.
//
// Two TMA rings per CTA: ring A holds the S / dP operands (this CTA's half of
// the tile's rows, all R columns of q and g), ring B the dD operands (all rows
// of the tile, this CTA's half of the R columns).  A cta_group::2 product reads
// the same shared-memory offset in both CTAs, so the rows-half and the
// columns-half layouts cannot share storage; the rings free independently (A
// once S and dP are done, B once the dD products are), so each needs only two
// stages.  Producer warps 0 (ring A) and 6 (ring B) each complete about one
// stage per 0.4 us, so a stage carries a whole row tile (32 KB per CTA).
#include <math.h>

#include "common.cuh"
#include "host_util.h"
#include "route_common.h"

namespace da {
namespace route {
namespace dgrad {

// warp 0 ring-A TMA, 1 MMA, 2-5 and 7-10 softmax (two warpgroups, each thread half of its row range:
// with one softmax warp per SM sub-partition the per-element chain left the latencies exposed and paced
// the kernel at ~2.6 us per row tile), 6 ring-B TMA
constexpr int kThreads = 352;
constexpr int kRingBWarp = 6;
constexpr int kSoftmax2 = 7;  // first warp of the second softmax warpgroup
constexpr int kAtoms = 64;     // atoms per CTA (128 per pair)

template <int kR>
struct Cfg {
  static constexpr int kTR = kR == 128 ? 128 : 64;  // route rows per tile (pair)
  static constexpr int kHalfRows = kTR / 2;          // rows of a tile held per CTA in ring A
  static constexpr int kDictBytes = kAtoms * kR * 2; // Dk (or Dv) rows of this CTA's atoms
  static constexpr int kXBytes = kHalfRows * kR * 2; // ring A: one tensor, this CTA's rows, all columns
  static constexpr int kYBytes = kTR * (kR / 2) * 2; // ring B: one tensor, all rows, this CTA's columns
  static constexpr int kPBytes = kAtoms * kTR * 2;   // P^T (or dL'^T) tile
  static constexpr int kOffDk = 0;
  static constexpr int kOffDv = kOffDk + kDictBytes;
  static constexpr int kOffA = kOffDv + kDictBytes;            // 2 stages x (q, g)
  static constexpr int kStatBytes = kTR * 16;                 // the tile's rows: {lse2, invn, delta, 0}
  static constexpr int kBStage = 2 * kYBytes + kStatBytes;     // ring B stage: q, g, row statistics
  static constexpr int kOffB = kOffA + 2 * 2 * kXBytes;        // 2 stages
  static constexpr int kOffP = kOffB + 2 * kBStage;
  static constexpr int kOffDl = kOffP + kPBytes;               // 2 buffers (P: one, released early)
  static constexpr int kCols = kTR / 4;                        // tile rows (score columns) per softmax thread
  static constexpr int kOffRed = kOffDl + 2 * kPBytes;
  static constexpr int kSmem = kOffRed + 64;
  static_assert(kCols == 32 || kCols == 16, "softmax column split");
  static_assert(kSmem + 1024 <= 232448, "dictionary-gradient tile does not fit in shared memory");
  // TMEM: dDk^T (R/2 folded columns), dDv^T, then 2 x S^T and 2 x dP^T (kTR/2 each)
  static constexpr int kTmemDk = 0;
  static constexpr int kTmemDv = kR / 2;
  static constexpr int kTmemS = kR;
  static constexpr int kTmemP = kR + kTR;
  static constexpr int kTmemCols = 512;
  static_assert(kR + 2 * kTR <= kTmemCols, "TMEM budget");
};

struct Params {
  int64_t rows;            // rows per group
  int groups;
  int64_t col_stride;      // column offset between groups in q
  int M;
  int tiles_per_group;     // ceil(rows / kTR)
  int64_t tiles;           // groups * tiles_per_group
  int chunks;              // row chunks (pairs = chunks * M / 128)
  const float* beta;
  const float* lse;        // [groups, rows]
  const float* row_stats;  // [groups, rows_pad, 4]: lse2, invn, delta, 0 (dead rows: +inf, 0, 0, 0)
  int64_t rows_pad;        // rows rounded up to 128
  float* part;             // [chunks, 2, M, R]: dDk^T then dDv^T partial sums
  float* part_beta;        // [pairs * 2]
  int* status;
  int* trace;              // optional post-mortem timeline of the first pair (debug)
};

template <typename T, int kR>
__global__ void __launch_bounds__(kThreads, 1) dict_grad_kernel(const __grid_constant__ CUtensorMap tqa,
                                                                const __grid_constant__ CUtensorMap tqb,
                                                                const __grid_constant__ CUtensorMap tga,
                                                                const __grid_constant__ CUtensorMap tgb,
                                                                const __grid_constant__ CUtensorMap tdk,
                                                                const __grid_constant__ CUtensorMap tdv,
                                                                const Params p) {
  using C = Cfg<kR>;
  constexpr int kTR = C::kTR;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ uint64_t dict_full, full_a[2], empty_a[2], full_b[2], empty_b[2], s_full[2], p_full[2], p_empty, dl_empty[2],
      stats_full[2], done;
  __shared__ uint32_t tmem_base;
  __shared__ int abort_flag;

  constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const uint32_t rank = cluster_ctarank() & 1u;
  const int nj = p.M / (2 * kAtoms);
  const int pair = blockIdx.x / 2;
  const int jt = pair % nj, chunk = pair / nj;
  const int64_t f0 = (int64_t)chunk * p.tiles / p.chunks, f1 = (int64_t)(chunk + 1) * p.tiles / p.chunks;
  const int nt = (int)(f1 - f0);  // >= 1: the host never makes more chunks than tiles
  Abort ab{&abort_flag, p.status};
  // debug timeline of the first pair: 4096 stamps per CTA, [role * 1024 + 4 * tile + event], after the
  // 2^18 slots the row pass may stamp
  int* ft = (p.trace && blockIdx.x < 2) ? p.trace + (1 << 18) + blockIdx.x * 4096 : nullptr;
  auto stamp = [&](int role, int t, int ev) {
    if (t < 256) trace_at(ft, role * 1024 + 4 * t + ev);
  };

  if (threadIdx.x == 0) {
    abort_flag = 0;
    mbar_init(&dict_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&full_a[i], 1);
      mbar_init(&empty_a[i], 1);
      mbar_init(&full_b[i], 1);
      mbar_init(&empty_b[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 16);  // one arrival per softmax warp of the pair
    }
    mbar_init(&p_empty, 1);
    mbar_init(&stats_full[0], 1);  // this CTA's own copy of the tile's row statistics
    mbar_init(&stats_full[1], 1);
    mbar_init(&dl_empty[0], 1);
    mbar_init(&dl_empty[1], 1);
    mbar_init(&done, 1);
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
  grid_dependency_wait();  // the row-parallel kernel's g and row statistics are visible from here on
  grid_launch_dependents();
  const uint32_t tmem = tmem_base;

  auto tile_of = [&](int t, int& g, int64_t& row0) {
    const int64_t f = f0 + t;
    g = (int)(f / p.tiles_per_group);
    row0 = (f % p.tiles_per_group) * kTR;
  };

  if ((warp == 0 || warp == kRingBWarp) && lane == 0) {
    // ---------------------------------------------------------------- TMA producers
    const bool ring_a = warp == 0;
    uint64_t* full = ring_a ? full_a : full_b;
    uint64_t* empty = ring_a ? empty_a : empty_b;
    const int bytes = ring_a ? 2 * C::kXBytes : 2 * C::kYBytes;  // paired tensor loads (the leader counts both CTAs)
    if (ring_a) {
      prefetch_tmap(&tqa);
      prefetch_tmap(&tga);
      prefetch_tmap(&tdk);
      prefetch_tmap(&tdv);
      // resident dictionary rows of this CTA's 64 atoms (all R columns)
      if (rank == 0) mbar_arrive_expect_tx(&dict_full, 2 * 2 * C::kDictBytes);
      const uint32_t dbar = mapa_shared(smem_u32(&dict_full), 0);
      const int atom0 = jt * 2 * kAtoms + kAtoms * (int)rank;
      tma_load_3d_pair(&tdk, dbar, smem + C::kOffDk, 0, atom0, 0);
      tma_load_3d_pair(&tdv, dbar, smem + C::kOffDv, 0, atom0, 0);
    } else {
      prefetch_tmap(&tqb);
      prefetch_tmap(&tgb);
    }
    bool ok = true;
    for (int t = 0; ok && t < nt; ++t) {
      const int s = t & 1;
      stamp(ring_a ? 0 : 1, t, 0);
      if (!mbar_wait(&empty[s], ((t >> 1) & 1u) ^ 1u, ab, ring_a ? 51 : 52)) { ok = false; break; }
      stamp(ring_a ? 0 : 1, t, 1);
      if (rank == 0) mbar_arrive_expect_tx(&full[s], 2 * bytes);
      const uint32_t bar = mapa_shared(smem_u32(&full[s]), 0);
      int g;
      int64_t row0;
      tile_of(t, g, row0);
      if (ring_a) {  // this CTA's half of the tile's rows, every column of q and g
        uint8_t* dst = smem + C::kOffA + s * 2 * C::kXBytes;
        const int r = (int)(row0 + (int64_t)rank * C::kHalfRows);
        tma_load_3d_pair(&tqa, bar, dst, 0, r, (int)(g * p.col_stride / 64));
        tma_load_3d_pair(&tga, bar, dst + C::kXBytes, 0, (int)(g * p.rows + r), 0);
      } else {  // every row of the tile, this CTA's half of the columns, and the rows' statistics
        uint8_t* dst = smem + C::kOffB + s * C::kBStage;
        const int cb = (int)rank * (kR / 128);
        tma_load_3d_pair(&tqb, bar, dst, 0, (int)row0, (int)(g * p.col_stride / 64) + cb);
        tma_load_3d_pair(&tgb, bar, dst + C::kYBytes, 0, (int)(g * p.rows + row0), cb);
        mbar_arrive_expect_tx(&stats_full[s], C::kStatBytes);
        bulk_load(dst + 2 * C::kYBytes, p.row_stats + 4 * ((int64_t)g * p.rows_pad + row0), C::kStatBytes,
                  &stats_full[s]);
      }
    }
    if (rank == 0) {  // drain: the leader's barriers count both CTAs' bytes
      if (ring_a) mbar_wait_drain(&dict_full, 0);
      for (int t = (nt > 2 ? nt - 2 : 0); t < nt; ++t) mbar_wait_drain(&full[t & 1], (t >> 1) & 1u);
    }
    if (!ring_a)  // each CTA's own statistics copies
      for (int t = (nt > 2 ? nt - 2 : 0); t < nt; ++t) mbar_wait_drain(&stats_full[t & 1], (t >> 1) & 1u);
  } else if (warp == 1 && lane == 0 && rank == 0) {
    // ---------------------------------------------------------------- MMA issuer (pair leader)
    const uint32_t idesc_s = idesc_f16(128, kTR, kBf16, false, false);
    const uint32_t idesc_p = idesc_f16(128, kTR, true, false, false);   // Dv and g are bf16
    const uint32_t idesc_v = idesc_f16(128, kR, true, false, true);     // P^T . g, g MN-major
    const uint32_t idesc_k = idesc_f16(128, kR, kBf16, false, true);    // dL'^T . q, q MN-major
    auto commit_both = [&](uint64_t* bar) { mma_commit_pair(smem_u32(bar)); };
    const uint32_t dk_a = smem_u32(smem + C::kOffDk), dv_a = smem_u32(smem + C::kOffDv);
    const uint32_t p_a = smem_u32(smem + C::kOffP), dl_a = smem_u32(smem + C::kOffDl);
    auto issue_sdp = [&](int t) -> bool {
      const int b = t & 1;
      stamp(2, t, 0);
      if (t >= 2 && !mbar_wait(&p_full[b], ((t - 2) >> 1) & 1u, ab, 53)) return false;
      if (!mbar_wait(&full_a[b], (t >> 1) & 1u, ab, 54)) return false;
      stamp(2, t, 1);
      tc_fence_after();
      const uint32_t qx = smem_u32(smem + C::kOffA + b * 2 * C::kXBytes), gx = qx + C::kXBytes;
      const uint32_t ds = tmem + C::kTmemS + b * (kTR / 2), dp = tmem + C::kTmemP + b * (kTR / 2);
#pragma unroll
      for (int k = 0; k < kR / 16; ++k) {  // S^T = Dk_tile . q^T  (K = R)
        const uint32_t ka = (k >> 2) * (kAtoms * 128) + (k & 3) * 32, kb = (k >> 2) * (C::kHalfRows * 128) + (k & 3) * 32;
        mma_f16_ss<2>(ds, sdesc_sw128(dk_a + ka, 16, 1024), sdesc_sw128(qx + kb, 16, 1024), idesc_s, k ? 1u : 0u);
      }
#pragma unroll
      for (int k = 0; k < kR / 16; ++k) {  // dP^T = Dv_tile . g^T
        const uint32_t ka = (k >> 2) * (kAtoms * 128) + (k & 3) * 32, kb = (k >> 2) * (C::kHalfRows * 128) + (k & 3) * 32;
        mma_f16_ss<2>(dp, sdesc_sw128(dv_a + ka, 16, 1024), sdesc_sw128(gx + kb, 16, 1024), idesc_p, k ? 1u : 0u);
      }
      commit_both(&s_full[b]);
      commit_both(&empty_a[b]);
      return true;
    };
    auto issue_dd = [&](int t) -> bool {
      const int b = t & 1;
      stamp(2, t, 2);
      if (!mbar_wait(&p_full[b], (t >> 1) & 1u, ab, 55)) return false;
      tc_fence_after();
      if (!mbar_wait(&full_b[b], (t >> 1) & 1u, ab, 56)) return false;
      stamp(2, t, 3);
      tc_fence_after();
      const uint32_t qy = smem_u32(smem + C::kOffB + b * C::kBStage), gy = qy + C::kYBytes;
#pragma unroll
      for (int kk = 0; kk < kTR / 16; ++kk) {  // dDv^T += P^T . g   (K = rows of the tile)
        const uint32_t ka = (kk >> 2) * (kAtoms * 128) + (kk & 3) * 32;
        mma_f16_ss<2>(tmem + C::kTmemDv, sdesc_sw128(p_a + ka, 16, 1024),
                      sdesc_sw128(gy + kk * 16 * 128, kTR * 128, 1024), idesc_v, (t | kk) ? 1u : 0u);
      }
      commit_both(&p_empty);  // the P tile is free for the next row tile while dDk runs
      const uint32_t dlb = dl_a + b * C::kPBytes;
#pragma unroll
      for (int kk = 0; kk < kTR / 16; ++kk) {  // dDk^T += dL'^T . q
        const uint32_t ka = (kk >> 2) * (kAtoms * 128) + (kk & 3) * 32;
        mma_f16_ss<2>(tmem + C::kTmemDk, sdesc_sw128(dlb + ka, 16, 1024),
                      sdesc_sw128(qy + kk * 16 * 128, kTR * 128, 1024), idesc_k, (t | kk) ? 1u : 0u);
      }
      commit_both(&dl_empty[b]);
      commit_both(&empty_b[b]);
      return true;
    };
    bool ok = mbar_wait(&dict_full, 0, ab, 57);
    tc_fence_after();
    if (ok) ok = issue_sdp(0);
    for (int t = 0; ok && t < nt; ++t) {
      if (t + 1 < nt) ok = issue_sdp(t + 1);
      if (ok) ok = issue_dd(t);
    }
    commit_both(&done);
    mbar_wait_drain(&done, 0);
  } else if ((warp >= 2 && warp <= 5) || warp >= kSoftmax2) {
    // ---------------------------------------------------------------- softmax (thread = atom x kCols tile rows)
    // TMEM lane l holds atom l % 64 and tile rows (l / 64) * kTR/2 + [0, kTR/2); warpgroup wg takes kCols of
    // them.  The warps issue no global loads (a proxy fence waits for a thread's outstanding loads, which
    // put ~1 us into every tile): each tile's row statistics arrive in ring B's stage by a bulk copy.  Each
    // warp arrives on the pair leader's barrier itself, so no named barrier runs per tile.
    constexpr int kCols = C::kCols;
    const int wg = warp >= kSoftmax2 ? 1 : 0;
    const int quad = warp & 3;
    const int l = quad * 32 + lane;
    const int a = l & 63, h = l >> 6;
    const int wslot = wg * 4 + quad;
    const int rr0 = h * (kTR / 2) + wg * kCols;  // first tile row of this thread
    const uint32_t lane_base = (uint32_t)(quad * 32) << 16;
    const float kLog2e = 1.4426950408889634f;
    const float beta = *p.beta;
    const uint32_t p_a = smem_u32(smem + C::kOffP), dl_a = smem_u32(smem + C::kOffDl);
    const uint32_t pf_leader = mapa_shared(smem_u32(&p_full[0]), 0);
    float dbeta = 0.f;
    bool ok = true;
    const bool tracer = warp == 2 && lane == 0;
    for (int t = 0; t < nt; ++t) {
      const int b = t & 1;
      // this thread's rows' {lse2, invn, delta}, copied into ring B's stage by its producer
      const float4* st4 = reinterpret_cast<const float4*>(smem + C::kOffB + b * C::kBStage + 2 * C::kYBytes) + rr0;
      if (tracer) stamp(3, t, 0);
      if (ok) ok = mbar_wait(&s_full[b], (t >> 1) & 1u, ab, 58);
      if (ok) ok = mbar_wait(&stats_full[b], (t >> 1) & 1u, ab, 62);
      ok = __all_sync(0xffffffffu, ok);
      if (tracer) stamp(3, t, 1);
      if (ok) {
        tc_fence_after();
        float sv[kCols], dpv[kCols];
        const uint32_t col = b * (kTR / 2) + wg * kCols;
        if constexpr (kCols == 32) {
          tmem_ld32(tmem + lane_base + C::kTmemS + col, sv);
          tmem_ld32(tmem + lane_base + C::kTmemP + col, dpv);
        } else {
          tmem_ld16(tmem + lane_base + C::kTmemS + col, sv);
          tmem_ld16(tmem + lane_base + C::kTmemP + col, dpv);
        }
        tmem_wait_ld();
        tc_fence_before();
        uint32_t pk[kCols / 2], dk[kCols / 2];
#pragma unroll
        for (int i = 0; i < kCols; i += 2) {
          float pr[2], dl[2];
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const float4 rs = st4[i + e];  // lse2, invn, delta
            const float invn = rs.y;
            pr[e] = ex2(sv[i + e] * (beta * invn * kLog2e) - rs.x);
            const float dls = pr[e] * (dpv[i + e] - rs.z);
            dbeta = fmaf(sv[i + e] * invn, dls, dbeta);
            dl[e] = dls * invn * beta;
          }
          pk[i / 2] = pack_bf16x2(pr[0], pr[1]);
          dk[i / 2] = pack2<T>(dl[0], dl[1]);
        }
        {  // the previous tile's dDv product has read P; the one before the previous tile's dDk, dL' buffer b
          bool w = true;
          if (t > 0) w = mbar_wait(&p_empty, (t - 1) & 1u, ab, 59);
          if (w && t > 1) w = mbar_wait(&dl_empty[b], ((t - 2) >> 1) & 1u, ab, 61);
          ok = ok && __all_sync(0xffffffffu, w);
        }
        if (tracer) stamp(3, t, 2);
        if (ok) {
          const uint32_t kb = (uint32_t)(rr0 >> 6) * (kAtoms * 128);
          const uint32_t c0 = (uint32_t)(rr0 & 63) >> 3;
#pragma unroll
          for (int e = 0; e < kCols / 8; ++e) {
            st_shared_v4(p_a + kb + sw128_offset(a, c0 + e), pk[4 * e], pk[4 * e + 1], pk[4 * e + 2], pk[4 * e + 3]);
            st_shared_v4(dl_a + b * C::kPBytes + kb + sw128_offset(a, c0 + e), dk[4 * e], dk[4 * e + 1],
                         dk[4 * e + 2], dk[4 * e + 3]);
          }
          fence_proxy_async();  // this thread's P / dL' stores, visible to the tensor core
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive_remote(pf_leader + b * 8);  // this warp: TMEM read, tiles written
      if (tracer) stamp(3, t, 3);
    }

    // ---- epilogue: this CTA's [64 atoms, R] partial sums (warpgroup wg stores the kind wg), then dbeta
    if (ok) ok = mbar_wait(&done, 0, ab, 60);
    ok = __all_sync(0xffffffffu, ok);
    tc_fence_after();
    if (ok) {
      const int atom = jt * 2 * kAtoms + kAtoms * (int)rank + a;
      const int kind = wg;
      float* dst = p.part + (((size_t)chunk * 2 + kind) * p.M + atom) * kR + h * (kR / 2);
      const uint32_t col0 = kind == 0 ? C::kTmemDk : C::kTmemDv;
#pragma unroll
      for (int c = 0; c < kR / 2; c += 32) {
        float v[32];
        tmem_ld32(tmem + lane_base + col0 + c, v);
        tmem_wait_ld();
#pragma unroll
        for (int e = 0; e < 8; ++e)
          reinterpret_cast<float4*>(dst + c)[e] = make_float4(v[4 * e], v[4 * e + 1], v[4 * e + 2], v[4 * e + 3]);
      }
    }
    for (int o = 16; o; o >>= 1) dbeta += __shfl_xor_sync(0xffffffffu, dbeta, o);
    float* red = reinterpret_cast<float*>(smem + C::kOffRed);
    if (lane == 0) red[wslot] = dbeta;
    named_bar_sync(1, 256);
    if (wg == 0 && l == 0) {
      float sum = 0.f;
      for (int i = 0; i < 8; ++i) sum += red[i];
      p.part_beta[2 * pair + rank] = ok ? sum : 0.f;
    }
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();
  if (warp == 1) tmem_dealloc<2>(tmem, C::kTmemCols);
}

// d_key[r, m] = sum_c part[c, 0, m, r], d_value likewise from part[c, 1]: chunks added in index order
// (32 x 32 tiles transposed through shared memory); block (0, 0, 0) also adds the dbeta partials in
// index order.
__global__ void __launch_bounds__(256) dict_grad_reduce_kernel(const float* part, int chunks, int M, int R,
                                                               float* d_key, float* d_value, const float* part_beta,
                                                               int n_beta, float* dbeta) {
  __shared__ float tile[32][33];
  grid_dependency_wait();
  grid_launch_dependents();
  const int kind = blockIdx.z;
  const int a0 = blockIdx.x * 32, r0 = blockIdx.y * 32;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;  // 32 x 8
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  for (int c = 0; c < chunks; ++c) {
    const float* src = part + ((size_t)c * 2 + kind) * M * R;
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[i] += src[(size_t)(a0 + ty + 8 * i) * R + r0 + tx];
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) tile[ty + 8 * i][tx] = acc[i];
  __syncthreads();
  float* out = kind == 0 ? d_key : d_value;
  if (out) {
#pragma unroll
    for (int i = 0; i < 4; ++i) out[(size_t)(r0 + ty + 8 * i) * M + a0 + tx] = tile[tx][ty + 8 * i];
  }
  if (dbeta && blockIdx.x == 0 && blockIdx.y == 0 && kind == 0 && threadIdx.x == 0) {
    float s = 0.f;
    for (int i = 0; i < n_beta; ++i) s += part_beta[i];
    *dbeta = s;
  }
}

// Row chunks per atom tile: one CTA pair per two SMs in total (about 200 KB of shared memory each),
// never more chunks than row tiles.
inline int chunks_for(int64_t tiles, int nj) {
  int c = (sm_count() / 2) / nj;
  if (c < 1) c = 1;
  if (c > tiles) c = (int)tiles;
  return c;
}

inline size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

struct WorkLayout {
  size_t off_g, off_stats, off_part, off_beta, bytes;
  int chunks, pairs, tr;
};

inline WorkLayout work_layout(int64_t rows, int groups, int64_t R, int64_t M) {
  WorkLayout W;
  W.tr = R == 128 ? 128 : 64;
  const int64_t tiles = (int64_t)groups * ((rows + W.tr - 1) / W.tr);
  const int nj = (int)(M / 128);
  W.chunks = chunks_for(tiles, nj);
  W.pairs = W.chunks * nj;
  W.off_g = 0;
  W.off_stats = align256(W.off_g + (size_t)groups * rows * R * 2);
  W.off_part = align256(W.off_stats + (size_t)groups * ((rows + 127) / 128 * 128) * 4 * 4);
  W.off_beta = align256(W.off_part + (size_t)W.chunks * 2 * M * R * 4);
  W.bytes = align256(W.off_beta + (size_t)W.pairs * 2 * 4);
  return W;
}

template <typename T, int kR>
int launch(const RouteBwdArgs& a, const WorkLayout& W, uint8_t* ws, float* d_key, float* d_value, float* dbeta,
           cudaStream_t st) {
  using C = Cfg<kR>;
  constexpr int kTR = C::kTR;
  const CUtensorMapDataType qdt =
      std::is_same<T, __nv_bfloat16>::value ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  const CUtensorMapDataType bdt = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  const __nv_bfloat16* g = reinterpret_cast<const __nv_bfloat16*>(ws + W.off_g);
  CUtensorMap tqa, tqb, tga, tgb, tdk, tdv;
  {  // q: (64-column block, row, block index) over [rows, q_cols]
    const uint64_t dims[3] = {64, (uint64_t)a.rows, (uint64_t)a.q_cols / 64};
    const uint64_t strides[2] = {(uint64_t)a.q_row_stride * 2, 128};
    const uint32_t box_a[3] = {64, (uint32_t)C::kHalfRows, (uint32_t)(kR / 64)};
    const uint32_t box_b[3] = {64, (uint32_t)kTR, (uint32_t)(kR / 128)};
    if (int rc = make_tmap_blocks(&tqa, a.q, qdt, 2, 3, dims, strides, box_a)) return rc;
    if (int rc = make_tmap_blocks(&tqb, a.q, qdt, 2, 3, dims, strides, box_b)) return rc;
  }
  {  // g: [groups * rows, R] bf16
    const uint64_t dims[3] = {64, (uint64_t)a.groups * a.rows, (uint64_t)kR / 64};
    const uint64_t strides[2] = {(uint64_t)kR * 2, 128};
    const uint32_t box_a[3] = {64, (uint32_t)C::kHalfRows, (uint32_t)(kR / 64)};
    const uint32_t box_b[3] = {64, (uint32_t)kTR, (uint32_t)(kR / 128)};
    if (int rc = make_tmap_blocks(&tga, g, bdt, 2, 3, dims, strides, box_a)) return rc;
    if (int rc = make_tmap_blocks(&tgb, g, bdt, 2, 3, dims, strides, box_b)) return rc;
  }
  {  // Dk^T [M, R] (dtype), Dv^T [M, R] bf16: 64 atoms x all R columns per box
    const uint64_t dims[3] = {64, (uint64_t)a.M, (uint64_t)kR / 64};
    const uint64_t strides[2] = {(uint64_t)kR * 2, 128};
    const uint32_t box[3] = {64, 64, (uint32_t)(kR / 64)};
    if (int rc = make_tmap_blocks(&tdk, a.dk_t, qdt, 2, 3, dims, strides, box)) return rc;
    if (int rc = make_tmap_blocks(&tdv, a.dv_t, bdt, 2, 3, dims, strides, box)) return rc;
  }
  Params p;
  p.rows = a.rows;
  p.groups = a.groups;
  p.col_stride = a.group_col_stride;
  p.M = (int)a.M;
  p.tiles_per_group = (int)((a.rows + kTR - 1) / kTR);
  p.tiles = (int64_t)a.groups * p.tiles_per_group;
  p.chunks = W.chunks;
  p.beta = a.beta;
  p.lse = a.lse;
  p.row_stats = reinterpret_cast<const float*>(ws + W.off_stats);
  p.rows_pad = (a.rows + 127) / 128 * 128;
  p.part = reinterpret_cast<float*>(ws + W.off_part);
  p.part_beta = reinterpret_cast<float*>(ws + W.off_beta);
  p.status = a.status;
  p.trace = debug_trace();
  auto kern = dict_grad_kernel<T, kR>;
  const int smem = C::kSmem + 1024;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
    return record_cuda_error();
  if (int rc = launch_kernel(kern, dim3((unsigned)(2 * W.pairs), 1, 1), dim3(kThreads, 1, 1), smem, st, true, tqa,
                             tqb, tga, tgb, tdk, tdv, p))
    return rc;
  const dim3 rgrid((unsigned)(a.M / 32), (unsigned)(kR / 32), 2);
  return launch_kernel(dict_grad_reduce_kernel, rgrid, dim3(256, 1, 1), 0, st, false, (const float*)p.part,
                       W.chunks, (int)a.M, kR, d_key, d_value, (const float*)p.part_beta, 2 * W.pairs, dbeta);
}

}  // namespace dgrad

bool route_bwd_fused_supported(const RouteBwdArgs& a) {
  if (a.R != 128 && a.R != 256) return false;
  if (a.M % 128 || a.q_cols % 64 || a.group_col_stride % 64 || a.q_row_stride % 8) return false;
  const int tr = a.R == 128 ? 128 : 64;
  if (a.rows < tr) return false;  // every TMA box lies inside the tensors
  return true;
}

int64_t route_bwd_workspace_bytes(int64_t rows, int groups, int64_t R, int64_t M) {
  return (int64_t)dgrad::work_layout(rows, groups, R, M).bytes;
}

int route_bwd_fused(RouteBwdArgs a, void* workspace, int64_t workspace_bytes, float* d_key, float* d_value,
                    float* dbeta, cudaStream_t st) {
  const dgrad::WorkLayout W = dgrad::work_layout(a.rows, a.groups, a.R, a.M);
  if (!workspace || workspace_bytes < (int64_t)W.bytes) return DA_ERR_WORKSPACE;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  // row-parallel pass: dq, g and the per-row statistics, no [rows, M] outputs, no dbeta atomics
  a.p_out = nullptr;
  a.dl_out = nullptr;
  a.g_out = ws + W.off_g;
  a.row_stats = reinterpret_cast<float*>(ws + W.off_stats);
  a.dbeta = nullptr;
  if (int rc = route_bwd(a, st)) return rc;
  const bool bf16 = a.dtype == DA_BF16;
  if (a.R == 128)
    return bf16 ? dgrad::launch<__nv_bfloat16, 128>(a, W, ws, d_key, d_value, dbeta, st)
                : dgrad::launch<__half, 128>(a, W, ws, d_key, d_value, dbeta, st);
  return bf16 ? dgrad::launch<__nv_bfloat16, 256>(a, W, ws, d_key, d_value, dbeta, st)
              : dgrad::launch<__half, 256>(a, W, ws, d_key, d_value, dbeta, st);
}

}  // namespace route
}  // namespace da

extern "C" int64_t da_route_bwd_workspace_size(int64_t rows, int groups, int64_t R, int64_t M) {
  if (rows <= 0 || groups <= 0 || (R != 128 && R != 256) || M <= 0 || M % 128) return -1;
  return da::route::route_bwd_workspace_bytes(rows, groups, R, M);
}

extern "C" int da_route_bwd_fused(const void* q, int64_t rows, int64_t q_cols, int64_t q_row_stride, int groups,
                                  int64_t group_col_stride, int64_t R, int64_t M, int dtype, const void* dict_key_t,
                                  const void* dict_value_t, const float* beta, float eps, int normalize_input,
                                  int normalize_output, const void* z, const void* dz, const float* lse,
                                  const float* out_norm, void* dq, float* d_key, float* d_value, float* dbeta,
                                  void* workspace, int64_t workspace_bytes, int* status, void* stream) {
  using namespace da;
  if (!q || !dict_key_t || !dict_value_t || !beta || !z || !dz || !lse || !out_norm || !dq || !status || !workspace)
    return DA_ERR_NULL;
  if (int rc = bind_device(q)) return rc;
  if (dtype != DA_BF16 && dtype != DA_F16) return DA_ERR_DTYPE;
  if (rows <= 0 || groups <= 0 || M <= 0 || rows > (1ll << 30)) return DA_ERR_SHAPE;
  if ((int64_t)(groups - 1) * group_col_stride + R > q_cols || q_row_stride < q_cols) return DA_ERR_SHAPE;
  const uintptr_t any = reinterpret_cast<uintptr_t>(z) | reinterpret_cast<uintptr_t>(dz) |
                        reinterpret_cast<uintptr_t>(dq) | reinterpret_cast<uintptr_t>(q) |
                        reinterpret_cast<uintptr_t>(workspace) | reinterpret_cast<uintptr_t>(d_key) |
                        reinterpret_cast<uintptr_t>(d_value);
  if (any & 15) return DA_ERR_ALIGN;
  route::RouteBwdArgs a{q,      rows,      q_cols,           q_row_stride,     groups,  group_col_stride,
                        R,      M,         dtype,            dict_key_t,       dict_value_t, beta,
                        eps,    normalize_input, normalize_output, z,          dz,      lse,
                        out_norm, dq,      nullptr,          nullptr,          nullptr, nullptr,
                        status};
  if (!route::route_bwd_fused_supported(a)) return DA_ERR_UNSUPPORTED;
  return route::route_bwd_fused(a, workspace, workspace_bytes, d_key, d_value, dbeta,
                                static_cast<cudaStream_t>(stream));
}
