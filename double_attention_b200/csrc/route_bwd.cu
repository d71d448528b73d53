// Dictionary route, backward (identity logits, softmax assignment).
//
// Reference: _DictionaryRouteFunction.backward (triton_kernels.py:1873-1981)
// with _row_l2_normalize_backward (:1410-1444) and
// _row_scaled_softmax_backward (:1447-1501); math of ops.py:16-62.  Per route
// row, with q_hat = q * invn (invn = 1 / max(||q||, eps) when normalize_input),
// P = softmax(beta * q_hat . Dk), r = P . Dv^T, z = r / max(||r||, eps):
//   g     = d r  = (dz - z <z, dz>) / ||r||        (||r|| > eps; dz / eps else;
//                                                   dz without normalize_output)
//   dP    = g . Dv                                  (one value per atom)
//   delta = <P, dP> = <r, g>                        (closed form from z, dz)
//   dLs   = P * (dP - delta)                        (gradient of beta * logits)
//   dbeta = sum_rows sum_atoms (q_hat . dk) * dLs
//   dq_hat = beta * dLs . Dk^T,  dq = input-normalisation backward of dq_hat
//   dDv   = sum_rows g (x) P,   dDk = sum_rows q_hat (x) beta * dLs.
//
// One CTA pair (2-CTA cluster, cta_group::2 MMAs) owns 128 rows of one group
// and walks the dictionary in tiles of 128 atoms:
//   * the softmax warpgroup first forms g (bf16) in shared memory from z and
//     dz (and stores it for the dictionary-gradient GEMM);
//   * S = q . Dk_j and dP = g . Dv_j land in TMEM (double-buffered);
//   * the softmax warpgroup recomputes P from the forward's log-sum-exp,
//     forms dL' = invn * beta * dLs, writes it to shared memory (operand of
//     the next MMA) and stores P and dL' rows for the dictionary gradients;
//   * u += dL'_j . Dk_j^T accumulates invn * dq_hat in TMEM (folded).
// The epilogue applies the input-normalisation backward,
//   dq = u - q_hat <q_hat, u>  (u = invn * dq_hat),
// and writes dq in the layout of q.  The dictionary gradients are two
// split-K GEMMs over the stored rows (dDv = G^T P, dDk = sum_groups q^T dL').
// Operands stream through one ring of 16 KB stages in the order the MMA warp
// consumes them.
#include <math.h>

#include "common.cuh"
#include "host_util.h"
#include "route_common.h"

namespace da {
namespace route {
namespace bwd {

constexpr int kThreads = 192;
constexpr int kRows = 64;        // rows per CTA
constexpr int kNA = 128;         // atoms per tile (per pair)
constexpr int kStage = 16384;
constexpr int kMaxStages = 8;

struct Params {
  int64_t rows;            // rows per group
  int64_t q_row_stride;
  int64_t col_stride;      // column offset between groups inside q / dq
  int R, M, groups;
  const float* beta;
  float eps;
  int normalize_input, normalize_output;
  const void* z;           // [groups, rows, R] dtype
  const void* dz;          // [groups, rows, R] dtype
  const float* lse;        // [groups, rows]
  const float* out_norm;   // [groups, rows]
  void* dq;                // layout of q (dtype), written
  __nv_bfloat16* p_out;    // [groups, rows, M]
  void* dl_out;            // [groups, rows, M] dtype: invn * beta * dLs
  __nv_bfloat16* g_out;    // [groups, rows, R]
  float* dbeta;            // accumulated (may be null)
  float* row_stats;        // [groups, rows_pad, 4]: lse2, invn, delta, 0 (may be null)
  float* dbeta_part;       // [2 * pairs * 4]: per-(CTA, warp) dbeta partials summed in order (null: atomics)
  int* status;
  int* trace;              // optional progress stamps (debug)
  int compact;             // the two-CTAs-per-SM layout (make_layout)
};

struct Layout {
  int rchunks, ncol, nins, nst, smem;
  int nb;  // score / dP / dL' tile buffers (2; 1 in the compact layout)
  int off_q, off_g, off_dl, off_red, off_ring;
  int tmem_u, tmem_s, tmem_p, tmem_cols;
};

// compact: single-buffered tiles so that two CTAs fit one SM (<= 256 TMEM columns, ~100 KB of shared
// memory, R <= 128); the other CTA's work then overlaps what double buffering used to.
__host__ __device__ inline Layout make_layout(int R, bool compact = false) {
  Layout L;
  L.nb = compact ? 1 : 2;
  L.rchunks = (R + 127) / 128;     // 128-column K chunks of the score / dP products
  L.ncol = R < 256 ? R : 256;      // N of one u instruction
  L.nins = R / L.ncol;
  L.off_q = 0;
  L.off_g = L.off_q + kRows * R * 2;
  L.off_dl = L.off_g + kRows * R * 2;
  L.off_red = L.off_dl + L.nb * kRows * kNA * 2;
  L.off_ring = L.off_red + 2048;
  const int avail = (compact ? 108 * 1024 : 225 * 1024) - L.off_ring;
  L.nst = avail / kStage > kMaxStages ? kMaxStages : avail / kStage;
  L.smem = L.off_ring + L.nst * kStage;
  L.tmem_u = 0;
  L.tmem_s = R / 2;
  L.tmem_p = L.tmem_s + L.nb * (kNA / 2);
  const int cols = L.tmem_p + L.nb * (kNA / 2);
  L.tmem_cols = cols <= 256 ? 256 : 512;
  return L;
}

template <typename T, int kMinBlocks>
__global__ void __launch_bounds__(kThreads, kMinBlocks) route_bwd_kernel(const __grid_constant__ CUtensorMap tq,
                                                                const __grid_constant__ CUtensorMap tdk,
                                                                const __grid_constant__ CUtensorMap tdv,
                                                                const __grid_constant__ CUtensorMap tz,
                                                                const __grid_constant__ CUtensorMap tdz,
                                                                const Params p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ uint64_t in_full, g_full, o_full, zd_full, r_full[kMaxStages], r_empty[kMaxStages];
  __shared__ uint64_t s_full[2], p_full[2], dl_empty[2];
  __shared__ uint32_t tmem_base;
  __shared__ int abort_flag;

  constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
  const int R = p.R;
  const Layout L = make_layout(R, p.compact != 0);
  const int nb = L.nb;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const uint32_t rank = cluster_ctarank() & 1u;
  const int tiles_per_group = (int)((p.rows + 127) / 128);
  const int pair = blockIdx.x / 2;
  const int grp = pair / tiles_per_group;
  const int row0 = (pair % tiles_per_group) * 128;
  const int NJ = p.M / kNA;
  // R <= 256: this CTA's z rows land in the (not yet used) dL' buffer and its dz rows in the g
  // buffer by TMA, so the output-normalisation backward reads both from shared memory once
  const bool zd_tma = R <= 128 * L.nb;  // z fills the dL' buffers
  Abort ab{&abort_flag, p.status};
  // debug trace: 8 phase stamps per CTA, then per-tile stamps of the first pair
  int* ft = (p.trace && blockIdx.x < 2) ? p.trace + gridDim.x * 8 + blockIdx.x * 256 : nullptr;
  if (threadIdx.x == 0) trace_time(p.trace, 0);

  if (threadIdx.x == 0) {
    abort_flag = 0;
    mbar_init(&in_full, 1);
    mbar_init(&g_full, 2);  // one arrival per CTA of the pair
    mbar_init(&o_full, 1);
    mbar_init(&zd_full, 1);
    for (int i = 0; i < kMaxStages; ++i) {
      mbar_init(&r_full[i], 1);
      mbar_init(&r_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 8);  // one arrival per row-math warp of the pair
      mbar_init(&dl_empty[i], 1);
    }
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

  if (warp == 0 && lane == 0) {
    // ---------------------------------------------------------------- TMA producer
    prefetch_tmap(&tq);
    prefetch_tmap(&tdk);
    prefetch_tmap(&tdv);
    const uint32_t inf = mapa_shared(smem_u32(&in_full), 0);
    if (rank == 0) mbar_arrive_expect_tx(&in_full, 2 * kRows * R * 2);
    // every box must overlap the tensor; rows past the end are never stored
    const int qrow = (int)min((int64_t)row0 + 64 * (int)rank, p.rows - 1);
    const int qcol = (int)(grp * p.col_stride);
    for (int cb = 0; cb < R / 64; ++cb)
      tma_load_2d_pair(&tq, inf, smem + L.off_q + cb * (kRows * 128), qcol + cb * 64, qrow);
    if (zd_tma) {  // this CTA's own rows of z and dz, on its own barrier
      prefetch_tmap(&tz);
      prefetch_tmap(&tdz);
      mbar_arrive_expect_tx(&zd_full, 2 * kRows * R * 2);
      const int zrow = (int)((int64_t)grp * p.rows + qrow);
      for (int cb = 0; cb < R / 64; ++cb) {
        tma_load_2d(&tz, &zd_full, smem + L.off_dl + cb * (kRows * 128), cb * 64, zrow);
        tma_load_2d(&tdz, &zd_full, smem + L.off_g + cb * (kRows * 128), cb * 64, zrow);
      }
    }
    int it = 0;
    bool ok = true;
    auto stage = [&](int bytes) -> uint8_t* {
      const int s = it % L.nst;
      if (!mbar_wait(&r_empty[s], ((it / L.nst) & 1u) ^ 1u, ab, 11)) { ok = false; return nullptr; }
      if (rank == 0) mbar_arrive_expect_tx(&r_full[s], 2 * bytes);
      return smem + L.off_ring + s * kStage;
    };
    auto stage_bar = [&]() { return mapa_shared(smem_u32(&r_full[it % L.nst]), 0); };
    auto items_sdp = [&](int j) {  // key and value rows of this CTA's 64 atoms, K-major, 128 columns per stage
      const int arow = j * kNA + 64 * (int)rank;
      for (int pass = 0; pass < 2; ++pass)
        for (int cc = 0; ok && cc < L.rchunks; ++cc, ++it) {
          const int nb = (R - cc * 128) >= 128 ? 2 : 1;
          uint8_t* dst = stage(nb * 64 * 128);
          if (!ok) return;
          const uint32_t bar = stage_bar();
          for (int bx = 0; bx < nb; ++bx)
            tma_load_2d_pair(pass == 0 ? &tdk : &tdv, bar, dst + bx * (64 * 128), cc * 128 + bx * 64, arow);
        }
    };
    auto items_u = [&](int j) {  // key rows of all 128 atoms, MN-major: this CTA's half of each N block
      const int per = (L.ncol / 2) / 64;
      for (int kc = 0; ok && kc < kNA / 64; ++kc)
        for (int ins = 0; ok && ins < L.nins; ++ins, ++it) {
          uint8_t* dst = stage(per * 64 * 128);
          if (!ok) return;
          const uint32_t bar = stage_bar();
          for (int bx = 0; bx < per; ++bx)
            tma_load_2d_pair(&tdk, bar, dst + bx * (64 * 128), ins * L.ncol + (int)rank * (L.ncol / 2) + bx * 64,
                             j * kNA + kc * 64);
        }
    };
    items_sdp(0);
    for (int j = 0; ok && j < NJ; ++j) {
      if (j + 1 < NJ) items_sdp(j + 1);
      items_u(j);
    }
    if (zd_tma) mbar_wait_drain(&zd_full, 0);
    if (rank == 0) {
      mbar_wait_drain(&in_full, 0);
      for (int i = (it > L.nst ? it - L.nst : 0); i < it; ++i) mbar_wait_drain(&r_full[i % L.nst], (i / L.nst) & 1u);
    }
  } else if (warp == 1 && lane == 0 && rank == 0) {
    // ---------------------------------------------------------------- MMA issuer (leader)
    const uint32_t idesc_s = idesc_f16(128, kNA, kBf16, false, false);
    const uint32_t idesc_p = idesc_f16(128, kNA, true, false, false);      // g and Dv are bf16
    const uint32_t idesc_u = idesc_f16(128, L.ncol, kBf16, false, true);   // B = Dk rows, MN-major
    auto commit_both = [&](uint64_t* bar) { mma_commit_pair(smem_u32(bar)); };
    int it = 0;
    auto take = [&](uint32_t* addr) -> bool {
      const int s = it % L.nst;
      if (!mbar_wait(&r_full[s], (it / L.nst) & 1u, ab, 23)) return false;
      tc_fence_after();
      *addr = smem_u32(smem + L.off_ring + s * kStage);
      return true;
    };
    auto give = [&]() { commit_both(&r_empty[it % L.nst]); ++it; };
    const uint32_t qa = smem_u32(smem + L.off_q), ga = smem_u32(smem + L.off_g);
    bool g_ready = false;
    auto issue_sdp = [&](int j) -> bool {
      const int sb = j % nb;
      trace_at(ft, 16 + 4 * j);
      if (j >= nb && !mbar_wait(&p_full[sb], ((j - nb) / nb) & 1u, ab, 22)) return false;
      trace_at(ft, 17 + 4 * j);
      for (int pass = 0; pass < 2; ++pass) {
        if (pass == 1 && !g_ready) {
          if (!mbar_wait(&g_full, 0, ab, 26)) return false;
          tc_fence_after();
          g_ready = true;
        }
        const uint32_t a0 = pass == 0 ? qa : ga;
        const uint32_t d = tmem + (pass == 0 ? L.tmem_s : L.tmem_p) + sb * (kNA / 2);
        const uint32_t idesc = pass == 0 ? idesc_s : idesc_p;
        for (int cc = 0; cc < L.rchunks; ++cc) {
          uint32_t st;
          if (!take(&st)) return false;
          const int nk16 = ((R - cc * 128) >= 128 ? 128 : R - cc * 128) / 16;
          for (int k = 0; k < nk16; ++k) {
            const uint64_t ad = sdesc_sw128(a0 + (cc * 2 + (k >> 2)) * (kRows * 128) + (k & 3) * 32, 16, 1024);
            const uint64_t bd = sdesc_sw128(st + (k >> 2) * (64 * 128) + (k & 3) * 32, 16, 1024);
            mma_f16_ss<2>(d, ad, bd, idesc, (cc | k) ? 1u : 0u);
          }
          give();
        }
      }
      commit_both(&s_full[sb]);
      trace_at(ft, 18 + 4 * j);
      return true;
    };
    auto issue_u = [&](int j) -> bool {
      const int sb = j % nb;
      if (!mbar_wait(&p_full[sb], (j / nb) & 1u, ab, 24)) return false;
      trace_at(ft, 19 + 4 * j);
      tc_fence_after();
      const uint32_t dla = smem_u32(smem + L.off_dl + sb * (kRows * kNA * 2));
      for (int kc = 0; kc < kNA / 64; ++kc)
        for (int ins = 0; ins < L.nins; ++ins) {
          uint32_t st;
          if (!take(&st)) return false;
          for (int kk = 0; kk < 4; ++kk) {
            const uint64_t ad = sdesc_sw128(dla + kc * (kRows * 128) + kk * 32, 16, 1024);
            const uint64_t bd = sdesc_sw128(st + kk * 16 * 128, 64 * 128, 1024);
            mma_f16_ss<2>(tmem + L.tmem_u + ins * (L.ncol / 2), ad, bd, idesc_u, (j | kc | kk) ? 1u : 0u);
          }
          give();
        }
      commit_both(&dl_empty[sb]);
      return true;
    };
    bool ok = mbar_wait(&in_full, 0, ab, 21);
    tc_fence_after();
    if (ok) ok = issue_sdp(0);
    for (int j = 0; ok && j < NJ; ++j) {
      if (j + 1 < NJ) ok = issue_sdp(j + 1);
      if (ok) ok = issue_u(j);
    }
    commit_both(&o_full);
    mbar_wait_drain(&o_full, 0);
  } else if (warp >= 2) {
    // ---------------------------------------------------------------- row math (4 warps, thread = row x half)
    const int quad = warp & 3;
    const int l = quad * 32 + lane;
    const int r = l & 63, half = l >> 6;
    const int64_t grow = row0 + 64 * (int)rank + r;
    const bool live = grow < p.rows;
    const int64_t idx = (int64_t)grp * p.rows + (live ? grow : 0);
    const uint32_t lane_base = (uint32_t)(quad * 32) << 16;
    const bool arriver = (warp == 2 && lane == 0);
    float* red = reinterpret_cast<float*>(smem + L.off_red);
    const float kLog2e = 1.4426950408889634f;
    const float beta = *p.beta;
    const int hw = R / 2;  // columns of this thread's half of the row

    // ---- g = d r from z and dz (this thread: columns half*hw .. +hw), 8 x 16-byte loads in flight
    const uint4* zrow = reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(p.z) + idx * R + half * hw);
    const uint4* dzrow = reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(p.dz) + idx * R + half * hw);
    const float on = live ? __ldg(p.out_norm + idx) : 1.f;
    float zd = 0.f, zz = 0.f;
    const uint32_t zsm = smem_u32(smem + L.off_dl), dzsm = smem_u32(smem + L.off_g);
    auto zd_addr = [&](int col) { return (uint32_t)((col >> 6) * (kRows * 128)) + sw128_offset(r, (col & 63) >> 3); };
    bool zd_ok = true;
    if (zd_tma) {
      zd_ok = __all_sync(0xffffffffu, mbar_wait(&zd_full, 0, ab, 36));
      if (zd_ok)
        for (int c = 0; c < hw / 8; ++c) {
          const uint32_t o = zd_addr(half * hw + c * 8);
          const uint4 a = ld_shared_v4(zsm + o), d = ld_shared_v4(dzsm + o);
          const uint32_t wa[4] = {a.x, a.y, a.z, a.w}, wd[4] = {d.x, d.y, d.z, d.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 fa = unpack2<T>(wa[e]), fd = unpack2<T>(wd[e]);
            zd = fmaf(fa.x, fd.x, fmaf(fa.y, fd.y, zd));
            zz = fmaf(fa.x, fa.x, fmaf(fa.y, fa.y, zz));
          }
        }
      if (!live) zd = zz = 0.f;
    }
    for (int c0 = 0; !zd_tma && c0 < hw / 8; c0 += 8) {
      uint4 a[8], d[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        a[i] = live ? __ldg(zrow + c0 + i) : make_uint4(0u, 0u, 0u, 0u);
        d[i] = live ? __ldg(dzrow + c0 + i) : make_uint4(0u, 0u, 0u, 0u);
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const uint32_t wa[4] = {a[i].x, a[i].y, a[i].z, a[i].w}, wd[4] = {d[i].x, d[i].y, d[i].z, d[i].w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 fa = unpack2<T>(wa[e]), fd = unpack2<T>(wd[e]);
          zd = fmaf(fa.x, fd.x, fmaf(fa.y, fd.y, zd));
          zz = fmaf(fa.x, fa.x, fmaf(fa.y, fa.y, zz));
        }
      }
    }
    red[l] = zd;
    red[128 + l] = zz;
    named_bar_sync(1, 128);
    zd += red[l ^ 64];
    zz += red[128 + (l ^ 64)];
    named_bar_sync(1, 128);
    // g = ca * dz - cb * z;  delta = <r, g> with r = z * max(on, eps) (normalised) or z
    float ca = 1.f, cb = 0.f, delta = zd;
    if (p.normalize_output) {
      if (on > p.eps) {
        ca = 1.f / on;
        cb = zd / on;
        delta = zd * (1.f - zz);
      } else {
        ca = 1.f / p.eps;
        delta = zd;
      }
    }
    if (zd_tma) {  // g in place of dz (each thread rewrites only what it read)
      uint4* grow_out = reinterpret_cast<uint4*>(p.g_out + idx * R + half * hw);
      if (zd_ok)
        for (int c = 0; c < hw / 8; ++c) {
          const uint32_t o = zd_addr(half * hw + c * 8);
          const uint4 a = ld_shared_v4(zsm + o), d = ld_shared_v4(dzsm + o);
          const uint32_t wa[4] = {a.x, a.y, a.z, a.w}, wd[4] = {d.x, d.y, d.z, d.w};
          uint32_t w[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 fa = unpack2<T>(wa[e]), fd = unpack2<T>(wd[e]);
            w[e] = live ? pack_bf16x2(ca * fd.x - cb * fa.x, ca * fd.y - cb * fa.y) : 0u;
          }
          if (live) grow_out[c] = make_uint4(w[0], w[1], w[2], w[3]);
          st_shared_v4(dzsm + o, w[0], w[1], w[2], w[3]);
        }
      fence_proxy_async();
    } else {
      const uint32_t gsm = smem_u32(smem + L.off_g);
      uint4* grow_out = reinterpret_cast<uint4*>(p.g_out + idx * R + half * hw);
      for (int c0 = 0; c0 < hw / 8; c0 += 8) {
        uint4 a[8], d[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          a[i] = live ? __ldg(zrow + c0 + i) : make_uint4(0u, 0u, 0u, 0u);
          d[i] = live ? __ldg(dzrow + c0 + i) : make_uint4(0u, 0u, 0u, 0u);
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const uint32_t wa[4] = {a[i].x, a[i].y, a[i].z, a[i].w}, wd[4] = {d[i].x, d[i].y, d[i].z, d[i].w};
          uint32_t w[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 fa = unpack2<T>(wa[e]), fd = unpack2<T>(wd[e]);
            w[e] = live ? pack_bf16x2(ca * fd.x - cb * fa.x, ca * fd.y - cb * fa.y) : 0u;
          }
          if (live) grow_out[c0 + i] = make_uint4(w[0], w[1], w[2], w[3]);
          const int col = half * hw + (c0 + i) * 8;
          st_shared_v4(gsm + (col >> 6) * (kRows * 128) + sw128_offset(r, (col & 63) >> 3), w[0], w[1], w[2], w[3]);
        }
      }
      fence_proxy_async();
    }
    named_bar_sync(1, 128);
    if (arriver) mbar_arrive_remote(mapa_shared(smem_u32(&g_full), 0));
    if (arriver) trace_time(p.trace, 2);

    // ---- per atom tile: P, dL' (shared memory + rows for the dictionary gradients), dbeta
    const float lse2 = live ? p.lse[idx] * kLog2e : 0.f;
    float invn = 1.f, qn = 0.f;
    float dbeta = 0.f;
    bool ok = true;
    const uint32_t pf_leader = mapa_shared(smem_u32(&p_full[0]), 0);
    T* dl_row = reinterpret_cast<T*>(p.dl_out) + idx * p.M;
    __nv_bfloat16* p_row = p.p_out + idx * p.M;
    for (int j = 0; j < NJ; ++j) {
      const int sb = j % nb;
      if (arriver) trace_at(ft, 128 + 4 * j);
      if (ok) ok = mbar_wait(&s_full[sb], (j / nb) & 1u, ab, 32);
      if (arriver) trace_at(ft, 129 + 4 * j);
      if (j == 0 && ok) {  // S_0 complete: the q tile has landed in both CTAs
        const uint32_t qa = smem_u32(smem + L.off_q);
        float qn2 = 0.f;
        for (int cb = 0; cb < R / 64; ++cb)
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            const uint4 v = ld_shared_v4(qa + cb * (kRows * 128) + sw128_offset(r, c));
            const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float2 f = unpack2<T>(w[e]);
              qn2 = fmaf(f.x, f.x, fmaf(f.y, f.y, qn2));
            }
          }
        qn = sqrtf(qn2);
        invn = p.normalize_input ? 1.f / fmaxf(qn, p.eps) : 1.f;
        if (p.row_stats && half == 0) {  // every row of the tile, dead rows too (no probability mass)
          const int64_t prow = (int64_t)grp * tiles_per_group * 128 + row0 + 64 * (int)rank + r;
          *reinterpret_cast<float4*>(p.row_stats + 4 * prow) =
              live ? make_float4(lse2, invn, delta, 0.f) : make_float4(INFINITY, 0.f, 0.f, 0.f);
        }
      }
      if (ok && j >= nb) ok = mbar_wait(&dl_empty[sb], ((j - nb) / nb) & 1u, ab, 33);
      ok = __all_sync(0xffffffffu, ok);
      if (ok) {
        tc_fence_after();
        const float scale2 = beta * invn * kLog2e;
        const float dl_scale = invn * beta;
        const uint32_t dla = smem_u32(smem + L.off_dl + sb * (kRows * kNA * 2));
        for (int ch = 0; ch < 2; ++ch) {
          float sv[32], dpv[32];
          tmem_ld32(tmem + lane_base + L.tmem_s + sb * (kNA / 2) + ch * 32, sv);
          tmem_ld32(tmem + lane_base + L.tmem_p + sb * (kNA / 2) + ch * 32, dpv);
          tmem_wait_ld();
          uint32_t pk[16], dk[16];
#pragma unroll
          for (int i = 0; i < 32; i += 2) {
            float pr[2], dl[2];
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              pr[h] = live ? ex2(sv[i + h] * scale2 - lse2) : 0.f;
              const float dls = pr[h] * (dpv[i + h] - delta);
              dbeta = fmaf(sv[i + h] * invn, dls, dbeta);
              dl[h] = dls * dl_scale;
            }
            pk[i / 2] = pack_bf16x2(pr[0], pr[1]);
            dk[i / 2] = pack2<T>(dl[0], dl[1]);
          }
          const int a0 = half * 64 + ch * 32;  // atom inside the tile
#pragma unroll
          for (int e = 0; e < 4; ++e)
            st_shared_v4(dla + half * (kRows * 128) + sw128_offset(r, ch * 4 + e), dk[4 * e], dk[4 * e + 1],
                         dk[4 * e + 2], dk[4 * e + 3]);
          if (live && p.p_out) {
            uint4* pd = reinterpret_cast<uint4*>(p_row + j * kNA + a0);
            uint4* dd = reinterpret_cast<uint4*>(dl_row + j * kNA + a0);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              pd[e] = make_uint4(pk[4 * e], pk[4 * e + 1], pk[4 * e + 2], pk[4 * e + 3]);
              dd[e] = make_uint4(dk[4 * e], dk[4 * e + 1], dk[4 * e + 2], dk[4 * e + 3]);
            }
          }
        }
        fence_proxy_async();
      }
      if (arriver) trace_at(ft, 130 + 4 * j);
      tc_fence_before();
      __syncwarp();  // this warp's TMEM reads are done and its dL' stores fenced: it arrives by itself
      if (lane == 0) mbar_arrive_remote(pf_leader + sb * 8);
    }
    if (arriver) trace_time(p.trace, 3);
    if (p.dbeta) {
      for (int o = 16; o; o >>= 1) dbeta += __shfl_xor_sync(0xffffffffu, dbeta, o);
      if (p.dbeta_part) {
        if (lane == 0) p.dbeta_part[blockIdx.x * 4 + quad] = ok ? dbeta : 0.f;
      } else if (lane == 0 && ok) {
        atomicAdd(p.dbeta, dbeta);
      }
    }

    // ---- epilogue: dq = u - q_hat <q_hat, u>   (u = invn * dq_hat, folded TMEM)
    if (ok) ok = mbar_wait(&o_full, 0, ab, 34);
    if (arriver) trace_time(p.trace, 4);
    ok = __all_sync(0xffffffffu, ok);
    tc_fence_after();
    const uint32_t qa = smem_u32(smem + L.off_q);
    float qu = 0.f;
    if (ok) {
      for (int ins = 0; ins < L.nins; ++ins)
        for (int c = 0; c < L.ncol / 2; c += 32) {
          float v[32];
          tmem_ld32(tmem + lane_base + L.tmem_u + ins * (L.ncol / 2) + c, v);
          tmem_wait_ld();
          const int col = ins * L.ncol + half * (L.ncol / 2) + c;
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const uint4 qv = ld_shared_v4(qa + (col >> 6) * (kRows * 128) + sw128_offset(r, ((col & 63) >> 3) + e));
            const uint32_t w[4] = {qv.x, qv.y, qv.z, qv.w};
#pragma unroll
            for (int h = 0; h < 4; ++h) {
              const float2 f = unpack2<T>(w[h]);
              qu = fmaf(f.x, v[8 * e + 2 * h], fmaf(f.y, v[8 * e + 2 * h + 1], qu));
            }
          }
        }
    }
    red[l] = qu;
    named_bar_sync(1, 128);
    qu += red[l ^ 64];
    // dq_c = u_c - invn^2 <q, u> q_c when the input was normalised (and not clamped)
    const float coef = (p.normalize_input && qn > p.eps) ? invn * invn * qu : 0.f;
    if (ok) {
      T* dq_row = reinterpret_cast<T*>(p.dq) + (live ? grow : 0) * p.q_row_stride + grp * p.col_stride;
      for (int ins = 0; ins < L.nins; ++ins)
        for (int c = 0; c < L.ncol / 2; c += 32) {
          float v[32];
          tmem_ld32(tmem + lane_base + L.tmem_u + ins * (L.ncol / 2) + c, v);
          tmem_wait_ld();
          const int col = ins * L.ncol + half * (L.ncol / 2) + c;
          uint32_t w[16];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const uint4 qv = ld_shared_v4(qa + (col >> 6) * (kRows * 128) + sw128_offset(r, ((col & 63) >> 3) + e));
            const uint32_t qw[4] = {qv.x, qv.y, qv.z, qv.w};
#pragma unroll
            for (int h = 0; h < 4; ++h) {
              const float2 f = unpack2<T>(qw[h]);
              w[4 * e + h] = pack2<T>(v[8 * e + 2 * h] - coef * f.x, v[8 * e + 2 * h + 1] - coef * f.y);
            }
          }
          if (live) {
            uint4* dst = reinterpret_cast<uint4*>(dq_row + col);
#pragma unroll
            for (int e = 0; e < 4; ++e) dst[e] = make_uint4(w[4 * e], w[4 * e + 1], w[4 * e + 2], w[4 * e + 3]);
          }
        }
    }
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();
  if (warp == 1) tmem_dealloc<2>(tmem, L.tmem_cols);
  if (threadIdx.x == 0) trace_time(p.trace, 5);
}

// *dbeta += the sum of n partials: strided in index order per thread, then a fixed tree.
__global__ void __launch_bounds__(256) dbeta_sum_kernel(const float* part, int n, float* dbeta) {
  __shared__ float red[256];
  grid_dependency_wait();
  grid_launch_dependents();
  float s = 0.f;
  for (int i = threadIdx.x; i < n; i += 256) s += part[i];
  red[threadIdx.x] = s;
  __syncthreads();
  for (int w = 128; w; w >>= 1) {
    if (threadIdx.x < w) red[threadIdx.x] += red[threadIdx.x + w];
    __syncthreads();
  }
  if (threadIdx.x == 0) *dbeta += red[0];
}

template <typename T>
int launch(const RouteBwdArgs& a, cudaStream_t st) {
  const long pairs = (long)a.groups * ((a.rows + 127) / 128);
  const bool compact = a.R <= 128 && pairs >= sm_count() && make_layout((int)a.R, true).nst >= 3;
  const Layout L = make_layout((int)a.R, compact);
  const CUtensorMapDataType qdt =
      std::is_same<T, __nv_bfloat16>::value ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUtensorMap tq, tdk, tdv;
  int rc = make_tmap_2d(&tq, a.q, qdt, 2, a.q_cols, a.rows, (uint64_t)a.q_row_stride * 2, 64, 64);
  if (rc) return rc;
  rc = make_tmap_2d(&tdk, a.dk_t, qdt, 2, a.R, a.M, (uint64_t)a.R * 2, 64, 64);
  if (rc) return rc;
  rc = make_tmap_2d(&tdv, a.dv_t, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a.R, a.M, (uint64_t)a.R * 2, 64, 64);
  if (rc) return rc;
  CUtensorMap tz = tq, tdz = tq;  // z and dz rows [groups * rows, R] (used for R <= 256)
  if (a.R <= 256) {
    rc = make_tmap_2d(&tz, a.z, qdt, 2, a.R, (uint64_t)a.groups * a.rows, (uint64_t)a.R * 2, 64, 64);
    if (rc) return rc;
    rc = make_tmap_2d(&tdz, a.dz, qdt, 2, a.R, (uint64_t)a.groups * a.rows, (uint64_t)a.R * 2, 64, 64);
    if (rc) return rc;
  }
  Params p;
  p.rows = a.rows;
  p.q_row_stride = a.q_row_stride;
  p.col_stride = a.group_col_stride;
  p.R = (int)a.R;
  p.M = (int)a.M;
  p.groups = a.groups;
  p.beta = a.beta;
  p.eps = a.eps;
  p.normalize_input = a.normalize_input;
  p.normalize_output = a.normalize_output;
  p.z = a.z;
  p.dz = a.dz;
  p.lse = a.lse;
  p.out_norm = a.out_norm;
  p.dq = a.dq;
  p.p_out = static_cast<__nv_bfloat16*>(a.p_out);
  p.dl_out = a.dl_out;
  p.g_out = static_cast<__nv_bfloat16*>(a.g_out);
  p.dbeta = a.dbeta;
  p.row_stats = a.row_stats;
  p.dbeta_part = a.dbeta ? a.dbeta_part : nullptr;
  p.status = a.status;
  p.trace = debug_trace();
  p.compact = compact ? 1 : 0;
  auto kern = compact ? route_bwd_kernel<T, 2> : route_bwd_kernel<T, 1>;
  const int smem = ((L.smem < 120 * 1024 && !compact) ? 120 * 1024 : L.smem) + 1024;  // one CTA per SM unless compact
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
    return record_cuda_error();
  if (int rc = launch_kernel(kern, dim3((unsigned)(2 * pairs), 1, 1), dim3(kThreads, 1, 1), smem, st, true, tq, tdk,
                             tdv, tz, tdz, p))
    return rc;
  if (!p.dbeta_part) return DA_OK;
  return launch_kernel(dbeta_sum_kernel, dim3(1), dim3(256), 0, st, false, (const float*)p.dbeta_part,
                       (int)(8 * pairs), a.dbeta);
}

}  // namespace bwd

int route_bwd(const RouteBwdArgs& a, cudaStream_t st) {
  return a.dtype == DA_BF16 ? bwd::launch<__nv_bfloat16>(a, st) : bwd::launch<__half>(a, st);
}

}  // namespace route
}  // namespace da

extern "C" int da_route_bwd(const void* q, int64_t rows, int64_t q_cols, int64_t q_row_stride, int groups,
                            int64_t group_col_stride, int64_t R, int64_t M, int dtype, const void* dict_key_t,
                            const void* dict_value_t, const float* beta, float eps, int normalize_input,
                            int normalize_output, const void* z, const void* dz, const float* lse,
                            const float* out_norm, void* dq, void* p_out, void* dl_out, void* g_out, float* dbeta,
                            float* dbeta_work, int64_t dbeta_work_elems, int* status, void* stream) {
  using namespace da;
  if (!q || !dict_key_t || !dict_value_t || !beta || !z || !dz || !lse || !out_norm || !dq || !g_out || !status)
    return DA_ERR_NULL;
  if ((p_out == nullptr) != (dl_out == nullptr)) return DA_ERR_NULL;  // both or neither
  if (int rc = bind_device(q)) return rc;
  if (dtype != DA_BF16 && dtype != DA_F16) return DA_ERR_DTYPE;
  if (rows <= 0 || groups <= 0 || M <= 0) return DA_ERR_SHAPE;
  if (R != 128 && R != 256 && R != 512) return DA_ERR_UNSUPPORTED;
  if (M % route::bwd::kNA) return DA_ERR_UNSUPPORTED;
  if ((int64_t)(groups - 1) * group_col_stride + R > q_cols || q_row_stride < q_cols) return DA_ERR_SHAPE;
  if (group_col_stride % 64 || q_row_stride % 8) return DA_ERR_ALIGN;
  {
    const route::bwd::Layout L = route::bwd::make_layout((int)R);
    if (L.nst < 2) return DA_ERR_UNSUPPORTED;
  }
  const uintptr_t any = reinterpret_cast<uintptr_t>(z) | reinterpret_cast<uintptr_t>(dz) |
                        reinterpret_cast<uintptr_t>(dq) | reinterpret_cast<uintptr_t>(p_out) |
                        reinterpret_cast<uintptr_t>(dl_out) | reinterpret_cast<uintptr_t>(g_out);
  if (any & 15) return DA_ERR_ALIGN;
  route::RouteBwdArgs a{q,      rows,      q_cols,           q_row_stride,     groups, group_col_stride,
                        R,      M,         dtype,            dict_key_t,       dict_value_t, beta,
                        eps,    normalize_input, normalize_output, z,          dz,     lse,
                        out_norm, dq,      p_out,            dl_out,           g_out,  dbeta,
                        status};
  if (dbeta && dbeta_work) {
    if (dbeta_work_elems < 8 * (int64_t)groups * ((rows + 127) / 128)) return DA_ERR_WORKSPACE;
    a.dbeta_part = dbeta_work;
  }
  return route::route_bwd(a, static_cast<cudaStream_t>(stream));
}
