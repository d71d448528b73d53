// Outer routed attention, backward (one score map per launch).
//
// Reference: _routed_attention_triton_backward (triton_kernels.py:2093-2263)
// and the autograd of routed_attention_reference (ops.py:65-93).  With
// S = gamma_eff * Q K^T (gamma_eff = gamma / sqrt(group)), P = exp(S - lse)
// (causal), Y_map = P V and the map's output weight alpha:
//   delta = <dY, Y_map> (row sums, Y_map = P V of this map alone),
//   dS  = alpha * P * (dY V^T - delta)         (gradient of the scaled score),
//   dQ  = gamma_eff * dS K,   dK = gamma_eff * dS^T Q,   dV += alpha * P^T dY,
//   dgamma = sum dS * (Q K^T) / sqrt(group)    (gradient of the map's scale),
//   dalpha = sum delta                         (left to the caller).
//
// Two paired-CTA kernels (2-CTA clusters, cta_group::2 MMAs, TMEM folded):
//   * query-parallel: a pair owns 128 query rows and loops over key tiles of
//     128: S and dP land in TMEM (double-buffered), the softmax warpgroup writes
//     dS (bf16) to shared memory, dQ accumulates in TMEM;
//   * key-parallel: a pair owns 128 keys and loops over query tiles of 128:
//     S^T and dP^T land in TMEM, P^T and dS^T go to shared memory, dV (D=512:
//     256 TMEM columns per CTA) and dK accumulate in TMEM.
// Operands stream through one ring of 16 KB stages filled in exactly the
// order the MMA warp consumes them, so the ring never waits on a softmax step
// that itself waits on the ring.  Gradients are accumulated into fp32
// outputs (several maps can share a branch and all maps share V).
#include <math.h>

#include "attn_common.h"
#include "common.cuh"
#include "host_util.h"

namespace da {
namespace attn {
namespace bwd {

constexpr int kThreads = 192;
constexpr int kRows = 64;        // rows (queries or keys) per CTA
constexpr int kTile = 128;       // columns (keys or queries) per tile
constexpr int kStage = 16384;    // ring stage bytes
constexpr int kMaxStages = 8;

struct Params {
  // row maps: row(b, branch, t) = base + b*sb + branch*sbr + t
  int64_t q_rows, q_base, q_sb, q_sbr;
  int64_t k_rows, k_base, k_sb, k_sbr;
  int B, T, R, D, group, branch0, causal;
  const float* scale;       // this map's score scale gamma_s (device scalar)
  const float* weight;      // this map's output weight alpha_s (device scalar), or null for 1
  const float* lse;         // [B, T] natural log, this map
  const float* delta;       // [B, T] <dY, Y_map>
  float* dq;                // fp32 [q_rows, R] (accumulated), or null
  float* dk;                // fp32 [k_rows, R] (accumulated), or null
  float* dv;                // fp32 [B*T, D] (accumulated), or null
  float* dscale;            // fp32 scalar (accumulated d gamma_s), or null
  int* status;
  int do_dv, do_dk;         // key-parallel kernel: which of dV / dK this launch accumulates
};

// Shared plumbing of both kernels.
struct Ring {
  uint64_t* full;
  uint64_t* empty;
  uint8_t* base;
  int n;
};

DA_DEV int64_t qk_row(int64_t base, int64_t sb, int64_t sbr, int b, int branch, int t) {
  return base + (int64_t)b * sb + (int64_t)branch * sbr + t;
}

// =============================================================================== dQ kernel
struct DqLayout {
  int kw, rpb, kw_chunks, d_chunks, nins, ncol;
  int off_q, off_dy, off_ds, off_red, off_ring, nst, smem;
  int tmem_dq, tmem_s, tmem_p, tmem_cols;
};

__host__ __device__ inline DqLayout dq_layout(int group, int R, int D) {
  DqLayout L;
  L.kw = group * R;
  L.rpb = R / 64;
  L.kw_chunks = (L.kw + 127) / 128;   // 128-column K chunks for S
  L.d_chunks = D / 128;               // 128-column V chunks for dP
  L.ncol = L.kw < 256 ? L.kw : 256;   // N of one dQ instruction
  L.nins = L.kw / L.ncol;
  L.off_q = 0;
  L.off_dy = L.off_q + kRows * L.kw * 2;
  L.off_ds = L.off_dy + kRows * D * 2;
  L.off_red = L.off_ds + 2 * kRows * kTile * 2;
  L.off_ring = L.off_red + 4096;
  const int avail = 225 * 1024 - L.off_ring;
  L.nst = avail / kStage > kMaxStages ? kMaxStages : avail / kStage;
  L.smem = L.off_ring + L.nst * kStage;
  L.tmem_dq = 0;
  L.tmem_s = L.kw / 2;
  L.tmem_p = L.tmem_s + 2 * (kTile / 2);
  const int cols = L.tmem_p + 2 * (kTile / 2);
  L.tmem_cols = cols <= 256 ? 256 : 512;
  return L;
}

template <typename T>
__global__ void __launch_bounds__(kThreads, 1) dq_kernel(const __grid_constant__ CUtensorMap tq,
                                                         const __grid_constant__ CUtensorMap tk,
                                                         const __grid_constant__ CUtensorMap tv,
                                                         const __grid_constant__ CUtensorMap tdy, const Params p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ uint64_t in_full, o_full, r_full[kMaxStages], r_empty[kMaxStages];
  __shared__ uint64_t s_full[2], p_full[2], ds_empty[2];
  __shared__ uint32_t tmem_base;
  __shared__ int abort_flag;

  const DqLayout L = dq_layout(p.group, p.R, p.D);
  constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const uint32_t rank = cluster_ctarank() & 1u;
  const int tiles = (p.T + kTile - 1) / kTile;
  const int pair = blockIdx.x / 2;
  const int b = pair / tiles;
  const int t0 = (tiles - 1 - pair % tiles) * kTile;
  const int nj = p.causal ? t0 / kTile + 1 : tiles;  // key tiles (128 keys, aligned with query tiles)
  Abort ab{&abort_flag, p.status};

  if (threadIdx.x == 0) {
    abort_flag = 0;
    mbar_init(&in_full, 1);
    mbar_init(&o_full, 1);
    for (int i = 0; i < kMaxStages; ++i) {
      mbar_init(&r_full[i], 1);
      mbar_init(&r_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 2);
      mbar_init(&ds_empty[i], 1);
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
  const uint32_t tmem = tmem_base;
  const int64_t rowsBT = (int64_t)p.B * p.T;

  if (warp == 0 && lane == 0) {
    // ---------------------------------------------------------------- TMA producer
    prefetch_tmap(&tq);
    prefetch_tmap(&tk);
    prefetch_tmap(&tv);
    prefetch_tmap(&tdy);
    const uint32_t inf = mapa_shared(smem_u32(&in_full), 0);
    if (rank == 0) mbar_arrive_expect_tx(&in_full, 2 * (kRows * L.kw * 2 + kRows * p.D * 2));
    const int tq_row = t0 + 64 * (int)rank;
    for (int cb = 0; cb < L.kw / 64; ++cb) {
      const int gi = cb / L.rpb, x = (cb % L.rpb) * 64;
      const int64_t row = qk_row(p.q_base, p.q_sb, p.q_sbr, b, p.branch0 + gi, tq_row);
      tma_load_2d_pair(&tq, inf, smem + L.off_q + cb * (kRows * 128), x, (int)min(row, p.q_rows - 1));
    }
    const int dy_row = (int)min((int64_t)b * p.T + tq_row, rowsBT - 1);
    for (int cb = 0; cb < p.D / 64; ++cb)
      tma_load_2d_pair(&tdy, inf, smem + L.off_dy + cb * (kRows * 128), cb * 64, dy_row);
    int it = 0;
    bool ok = true;
    auto stage = [&](int bytes) -> uint8_t* {  // acquire the next ring stage
      const int s = it % L.nst;
      if (!mbar_wait(&r_empty[s], ((it / L.nst) & 1u) ^ 1u, ab, 11)) { ok = false; return nullptr; }
      if (rank == 0) mbar_arrive_expect_tx(&r_full[s], 2 * bytes);
      return smem + L.off_ring + s * kStage;
    };
    auto stage_bar = [&]() { return mapa_shared(smem_u32(&r_full[it % L.nst]), 0); };
    auto items_sdp = [&](int j) {
      const int krow0 = j * kTile + 64 * (int)rank;  // this CTA's 64 keys of the tile
      for (int cc = 0; ok && cc < L.kw_chunks; ++cc, ++it) {
        const int nb = (L.kw - cc * 128) >= 128 ? 2 : 1;
        uint8_t* dst = stage(nb * kRows * 128);
        if (!ok) return;
        const uint32_t bar = stage_bar();
        for (int bx = 0; bx < nb; ++bx) {
          const int cb = cc * 2 + bx, gi = cb / L.rpb, x = (cb % L.rpb) * 64;
          const int64_t row = qk_row(p.k_base, p.k_sb, p.k_sbr, b, p.branch0 + gi, krow0);
          tma_load_2d_pair(&tk, bar, dst + bx * (kRows * 128), x, (int)min(row, p.k_rows - 1));
        }
      }
      for (int cc = 0; ok && cc < L.d_chunks; ++cc, ++it) {
        uint8_t* dst = stage(2 * kRows * 128);
        if (!ok) return;
        const uint32_t bar = stage_bar();
        const int y = (int)min((int64_t)b * p.T + krow0, rowsBT - 1);
        for (int bx = 0; bx < 2; ++bx) tma_load_2d_pair(&tv, bar, dst + bx * (kRows * 128), cc * 128 + bx * 64, y);
      }
    };
    auto items_dq = [&](int j) {
      const int per = (L.ncol / 2) / 64;
      for (int kc = 0; ok && kc < kTile / 64; ++kc)
        for (int ins = 0; ok && ins < L.nins; ++ins, ++it) {
          uint8_t* dst = stage(per * 64 * 128);
          if (!ok) return;
          const uint32_t bar = stage_bar();
          for (int bx = 0; bx < per; ++bx) {
            const int col = ins * L.ncol + (int)rank * (L.ncol / 2) + bx * 64;
            const int cb = col / 64, gi = cb / L.rpb, x = (cb % L.rpb) * 64;
            const int64_t row = qk_row(p.k_base, p.k_sb, p.k_sbr, b, p.branch0 + gi, j * kTile + kc * 64);
            tma_load_2d_pair(&tk, bar, dst + bx * (64 * 128), x, (int)min(row, p.k_rows - 1));
          }
        }
    };
    items_sdp(0);
    for (int j = 0; ok && j < nj; ++j) {
      if (j + 1 < nj) items_sdp(j + 1);
      items_dq(j);
    }
    if (rank == 0) {
      mbar_wait_drain(&in_full, 0);
      for (int i = (it > L.nst ? it - L.nst : 0); i < it; ++i) mbar_wait_drain(&r_full[i % L.nst], (i / L.nst) & 1u);
    }
  } else if (warp == 1 && lane == 0 && rank == 0) {
    // ---------------------------------------------------------------- MMA issuer (leader)
    const uint32_t idesc_s = idesc_f16(128, kTile, kBf16, false, false);
    const uint32_t idesc_q = idesc_f16(128, L.ncol, kBf16, false, true);  // B = K, MN-major
    auto commit_both = [&](uint64_t* bar) {
      mma_commit<2>(smem_u32(bar));
      mma_commit<2>(mapa_shared(smem_u32(bar), 1));
    };
    int it = 0;
    auto take = [&](uint32_t* addr) -> bool {
      const int s = it % L.nst;
      if (!mbar_wait(&r_full[s], (it / L.nst) & 1u, ab, 23)) return false;
      tc_fence_after();
      *addr = smem_u32(smem + L.off_ring + s * kStage);
      return true;
    };
    auto give = [&]() { commit_both(&r_empty[it % L.nst]); ++it; };
    const uint32_t qa = smem_u32(smem + L.off_q), dya = smem_u32(smem + L.off_dy);
    auto issue_sdp = [&](int j) -> bool {
      const int sb = j & 1;
      if (j >= 2 && !mbar_wait(&p_full[sb], ((j - 2) >> 1) & 1u, ab, 22)) return false;
      const uint32_t ds = tmem + L.tmem_s + sb * (kTile / 2), dp = tmem + L.tmem_p + sb * (kTile / 2);
      for (int cc = 0; cc < L.kw_chunks; ++cc) {
        uint32_t st;
        if (!take(&st)) return false;
        const int nk16 = ((L.kw - cc * 128) >= 128 ? 128 : L.kw - cc * 128) / 16;
        for (int k = 0; k < nk16; ++k) {
          const uint64_t ad = sdesc_sw128(qa + (cc * 2 + (k >> 2)) * (kRows * 128) + (k & 3) * 32, 16, 1024);
          const uint64_t bd = sdesc_sw128(st + (k >> 2) * (kRows * 128) + (k & 3) * 32, 16, 1024);
          mma_f16_ss<2>(ds, ad, bd, idesc_s, (cc | k) ? 1u : 0u);
        }
        give();
      }
      for (int cc = 0; cc < L.d_chunks; ++cc) {
        uint32_t st;
        if (!take(&st)) return false;
        for (int k = 0; k < 8; ++k) {
          const uint64_t ad = sdesc_sw128(dya + (cc * 2 + (k >> 2)) * (kRows * 128) + (k & 3) * 32, 16, 1024);
          const uint64_t bd = sdesc_sw128(st + (k >> 2) * (kRows * 128) + (k & 3) * 32, 16, 1024);
          mma_f16_ss<2>(dp, ad, bd, idesc_s, (cc | k) ? 1u : 0u);
        }
        give();
      }
      commit_both(&s_full[sb]);
      return true;
    };
    auto issue_dq = [&](int j) -> bool {
      const int sb = j & 1;
      if (!mbar_wait(&p_full[sb], (j >> 1) & 1u, ab, 24)) return false;
      tc_fence_after();
      const uint32_t dsa = smem_u32(smem + L.off_ds + sb * (kRows * kTile * 2));
      for (int kc = 0; kc < kTile / 64; ++kc)
        for (int ins = 0; ins < L.nins; ++ins) {
          uint32_t st;
          if (!take(&st)) return false;
          for (int kk = 0; kk < 4; ++kk) {
            const uint64_t ad = sdesc_sw128(dsa + kc * (kRows * 128) + kk * 32, 16, 1024);
            const uint64_t bd = sdesc_sw128(st + kk * 16 * 128, 64 * 128, 1024);  // MN-major K
            mma_f16_ss<2>(tmem + L.tmem_dq + ins * (L.ncol / 2), ad, bd, idesc_q, (j | kc | kk) ? 1u : 0u);
          }
          give();
        }
      commit_both(&ds_empty[sb]);
      return true;
    };
    bool ok = mbar_wait(&in_full, 0, ab, 21);
    tc_fence_after();
    if (ok) ok = issue_sdp(0);
    for (int j = 0; ok && j < nj; ++j) {
      if (j + 1 < nj) ok = issue_sdp(j + 1);
      if (ok) ok = issue_dq(j);
    }
    commit_both(&o_full);
    mbar_wait_drain(&o_full, 0);
  } else if (warp >= 2) {
    // ---------------------------------------------------------------- softmax + epilogue
    const int quad = warp & 3;
    const int l = quad * 32 + lane;
    const int r = l & 63, half = l >> 6;
    const int t = t0 + 64 * (int)rank + r;
    const bool live = t < p.T;
    const uint32_t lane_base = (uint32_t)(quad * 32) << 16;
    const uint32_t pf_leader = mapa_shared(smem_u32(&p_full[0]), 0);
    const bool arriver = (warp == 2 && lane == 0);
    const float kLog2e = 1.4426950408889634f;
    const float gsc = rsqrtf((float)p.group);
    const float gamma = *p.scale * gsc;
    const float alpha = p.weight ? *p.weight : 1.f;
    const float scale2 = gamma * kLog2e;
    const float lse2 = live ? p.lse[(int64_t)b * p.T + t] * kLog2e : 0.f;
    const float delta = live ? p.delta[(int64_t)b * p.T + t] : 0.f;
    // d gamma from this row's own sums: with A = sum P dP S, B = sum P S,
    // C = sum P dP (the exact delta), sum_k dS_k S_k = alpha (A - C B); this
    // does not inherit the rounding of the delta taken from the stored output.
    float sA = 0.f, sB = 0.f, sC = 0.f;
    bool ok = true;
    for (int j = 0; j < nj; ++j) {
      const int sb = j & 1;
      if (ok) ok = mbar_wait(&s_full[sb], (j >> 1) & 1u, ab, 32);
      if (ok && j >= 2) ok = mbar_wait(&ds_empty[sb], ((j - 2) >> 1) & 1u, ab, 33);
      ok = __all_sync(0xffffffffu, ok);
      if (ok) {
        tc_fence_after();
        const uint32_t dsa = smem_u32(smem + L.off_ds + sb * (kRows * kTile * 2));
        for (int ch = 0; ch < 2; ++ch) {
          float sv[32], pv[32];
          tmem_ld32(tmem + lane_base + L.tmem_s + sb * (kTile / 2) + ch * 32, sv);
          tmem_ld32(tmem + lane_base + L.tmem_p + sb * (kTile / 2) + ch * 32, pv);
          tmem_wait_ld();
          const int k0 = j * kTile + half * 64 + ch * 32;
          int lim = p.T - k0;
          if (p.causal) lim = min(lim, t - k0 + 1);
          if (!live) lim = 0;
          uint32_t packed[16];
#pragma unroll
          for (int i = 0; i < 32; i += 2) {
            float d0 = 0.f, d1 = 0.f;
            if (i < lim) {
              const float pr = ex2(sv[i] * scale2 - lse2);
              d0 = alpha * pr * (pv[i] - delta);
              const float pp = pr * pv[i];
              sA = fmaf(pp, sv[i], sA);
              sB = fmaf(pr, sv[i], sB);
              sC += pp;
            }
            if (i + 1 < lim) {
              const float pr = ex2(sv[i + 1] * scale2 - lse2);
              d1 = alpha * pr * (pv[i + 1] - delta);
              const float pp = pr * pv[i + 1];
              sA = fmaf(pp, sv[i + 1], sA);
              sB = fmaf(pr, sv[i + 1], sB);
              sC += pp;
            }
            packed[i / 2] = pack2<T>(d0, d1);
          }
          // dS tile: box `half` (keys half*64 .. +64), 16-byte chunks ch*4 .. ch*4+3
#pragma unroll
          for (int e = 0; e < 4; ++e)
            st_shared_v4(dsa + half * (kRows * 128) + sw128_offset(r, ch * 4 + e), packed[4 * e], packed[4 * e + 1],
                         packed[4 * e + 2], packed[4 * e + 3]);
        }
        fence_proxy_async();
      }
      tc_fence_before();
      named_bar_sync(1, 128);
      if (arriver) mbar_arrive_cluster(pf_leader + sb * 8);
    }
    if (p.dscale) {  // combine the two halves of each row (every softmax thread takes part)
      float* red = reinterpret_cast<float*>(smem + L.off_red);
      red[l] = sA;
      red[128 + l] = sB;
      red[256 + l] = sC;
      named_bar_sync(1, 128);
      float dg = 0.f;
      if (half == 0 && live && ok)
        dg = alpha * ((sA + red[l ^ 64]) - (sC + red[256 + (l ^ 64)]) * (sB + red[128 + (l ^ 64)]));
      for (int o = 16; o; o >>= 1) dg += __shfl_xor_sync(0xffffffffu, dg, o);
      if (lane == 0 && dg != 0.f) atomicAdd(p.dscale, dg * gsc);
    }
    if (ok) ok = mbar_wait(&o_full, 0, ab, 34);
    ok = __all_sync(0xffffffffu, ok);
    tc_fence_after();
    if (ok) {
      for (int ins = 0; ins < L.nins; ++ins)
        for (int c = 0; c < L.ncol / 2; c += 32) {
          float v[32];
          tmem_ld32(tmem + lane_base + L.tmem_dq + ins * (L.ncol / 2) + c, v);
          tmem_wait_ld();
          if (live && p.dq) {
            const int col = ins * L.ncol + half * (L.ncol / 2) + c;  // 32 columns inside one branch
            const int gi = col / p.R;
            const int64_t row = qk_row(p.q_base, p.q_sb, p.q_sbr, b, p.branch0 + gi, t);
            float* dst = p.dq + row * p.R + (col % p.R);
#pragma unroll
            for (int e = 0; e < 32; e += 4) {
              float4 o = *reinterpret_cast<float4*>(dst + e);
              o.x += gamma * v[e];
              o.y += gamma * v[e + 1];
              o.z += gamma * v[e + 2];
              o.w += gamma * v[e + 3];
              *reinterpret_cast<float4*>(dst + e) = o;
            }
          }
        }
    }
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();
  if (warp == 1) tmem_dealloc<2>(tmem, L.tmem_cols);
}

// =============================================================================== dK/dV kernel
struct KvLayout {
  int kw, rpb, kw_chunks, d_chunks, nins, ncol, dins;
  int off_k, off_v, off_p, off_ds, off_red, off_ring, nst, smem;
  int tmem_dv, tmem_dk, tmem_s, tmem_p, tmem_cols;
};

// dV and dK accumulate side by side in TMEM when they fit (D/2 + group*R/2
// columns next to S^T and dP^T); otherwise the host runs a dV launch and a dK
// launch, each holding one accumulator.
__host__ __device__ inline KvLayout kv_layout(int group, int R, int D, bool do_dv, bool do_dk) {
  KvLayout L;
  L.kw = group * R;
  L.rpb = R / 64;
  L.kw_chunks = (L.kw + 127) / 128;
  L.d_chunks = D / 128;
  L.ncol = L.kw < 256 ? L.kw : 256;
  L.nins = L.kw / L.ncol;
  L.dins = D / 256 > 0 ? D / 256 : 1;  // dV instructions (N = min(D, 256))
  L.off_k = 0;
  L.off_v = L.off_k + kRows * L.kw * 2;
  L.off_p = L.off_v + kRows * D * 2;
  L.off_ds = L.off_p + kRows * kTile * 2;
  L.off_red = L.off_ds + kRows * kTile * 2;
  L.off_ring = L.off_red + 2048;
  const int avail = 225 * 1024 - L.off_ring;
  L.nst = avail / kStage > kMaxStages ? kMaxStages : avail / kStage;
  L.smem = L.off_ring + L.nst * kStage;
  L.tmem_dv = 0;
  L.tmem_dk = do_dv ? D / 2 : 0;
  L.tmem_s = L.tmem_dk + (do_dk ? L.kw / 2 : 0);
  L.tmem_p = L.tmem_s + kTile / 2;
  const int cols = L.tmem_p + (do_dk ? kTile / 2 : 0);
  L.tmem_cols = cols <= 256 ? 256 : (cols <= 512 ? 512 : 1024);  // 1024: does not fit
  return L;
}

template <typename T>
__global__ void __launch_bounds__(kThreads, 1) dkv_kernel(const __grid_constant__ CUtensorMap tq,
                                                          const __grid_constant__ CUtensorMap tk,
                                                          const __grid_constant__ CUtensorMap tv,
                                                          const __grid_constant__ CUtensorMap tdy, const Params p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ uint64_t in_full, o_full, r_full[kMaxStages], r_empty[kMaxStages];
  __shared__ uint64_t s_full, p_full, pd_empty;
  __shared__ uint32_t tmem_base;
  __shared__ int abort_flag;

  const bool do_dv = p.do_dv != 0, do_dk = p.do_dk != 0;
  const KvLayout L = kv_layout(p.group, p.R, p.D, do_dv, do_dk);
  constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const uint32_t rank = cluster_ctarank() & 1u;
  const int tiles = (p.T + kTile - 1) / kTile;
  const int pair = blockIdx.x / 2;
  const int b = pair / tiles;
  const int k0 = (pair % tiles) * kTile;           // first key of this pair (early keys have most queries)
  const int i0 = p.causal ? k0 / kTile : 0;        // first query tile
  const int ni = tiles - i0;
  const int dn = p.D < 256 ? p.D : 256;            // N of one dV instruction
  Abort ab{&abort_flag, p.status};

  if (threadIdx.x == 0) {
    abort_flag = 0;
    mbar_init(&in_full, 1);
    mbar_init(&o_full, 1);
    for (int i = 0; i < kMaxStages; ++i) {
      mbar_init(&r_full[i], 1);
      mbar_init(&r_empty[i], 1);
    }
    mbar_init(&s_full, 1);
    mbar_init(&p_full, 2);
    mbar_init(&pd_empty, 1);
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
  const uint32_t tmem = tmem_base;
  const int64_t rowsBT = (int64_t)p.B * p.T;

  if (warp == 0 && lane == 0) {
    // ---------------------------------------------------------------- TMA producer
    prefetch_tmap(&tq);
    prefetch_tmap(&tk);
    prefetch_tmap(&tv);
    prefetch_tmap(&tdy);
    const uint32_t inf = mapa_shared(smem_u32(&in_full), 0);
    if (rank == 0) mbar_arrive_expect_tx(&in_full, 2 * (kRows * L.kw * 2 + (do_dk ? kRows * p.D * 2 : 0)));
    const int krow = k0 + 64 * (int)rank;
    for (int cb = 0; cb < L.kw / 64; ++cb) {
      const int gi = cb / L.rpb, x = (cb % L.rpb) * 64;
      const int64_t row = qk_row(p.k_base, p.k_sb, p.k_sbr, b, p.branch0 + gi, krow);
      tma_load_2d_pair(&tk, inf, smem + L.off_k + cb * (kRows * 128), x, (int)min(row, p.k_rows - 1));
    }
    const int vy = (int)min((int64_t)b * p.T + krow, rowsBT - 1);
    if (do_dk)  // V rows feed dP^T, needed only for dS
      for (int cb = 0; cb < p.D / 64; ++cb)
        tma_load_2d_pair(&tv, inf, smem + L.off_v + cb * (kRows * 128), cb * 64, vy);
    int it = 0;
    bool ok = true;
    auto stage = [&](int bytes) -> uint8_t* {
      const int s = it % L.nst;
      if (!mbar_wait(&r_empty[s], ((it / L.nst) & 1u) ^ 1u, ab, 11)) { ok = false; return nullptr; }
      if (rank == 0) mbar_arrive_expect_tx(&r_full[s], 2 * bytes);
      return smem + L.off_ring + s * kStage;
    };
    auto stage_bar = [&]() { return mapa_shared(smem_u32(&r_full[it % L.nst]), 0); };
    auto items_sdp = [&](int i) {  // Q chunks (K-major) then dY chunks (K-major), this CTA's 64 queries
      const int q = i * kTile + 64 * (int)rank;
      for (int cc = 0; ok && cc < L.kw_chunks; ++cc, ++it) {
        const int nb = (L.kw - cc * 128) >= 128 ? 2 : 1;
        uint8_t* dst = stage(nb * kRows * 128);
        if (!ok) return;
        const uint32_t bar = stage_bar();
        for (int bx = 0; bx < nb; ++bx) {
          const int cb = cc * 2 + bx, gi = cb / L.rpb, x = (cb % L.rpb) * 64;
          const int64_t row = qk_row(p.q_base, p.q_sb, p.q_sbr, b, p.branch0 + gi, q);
          tma_load_2d_pair(&tq, bar, dst + bx * (kRows * 128), x, (int)min(row, p.q_rows - 1));
        }
      }
      const int y = (int)min((int64_t)b * p.T + q, rowsBT - 1);
      for (int cc = 0; ok && do_dk && cc < L.d_chunks; ++cc, ++it) {
        uint8_t* dst = stage(2 * kRows * 128);
        if (!ok) return;
        const uint32_t bar = stage_bar();
        for (int bx = 0; bx < 2; ++bx) tma_load_2d_pair(&tdy, bar, dst + bx * (kRows * 128), cc * 128 + bx * 64, y);
      }
    };
    auto items_dkv = [&](int i) {  // dY (MN-major) for dV, then Q (MN-major) for dK: all 128 queries
      const int dper = (dn / 2) / 64;
      for (int qc = 0; ok && do_dv && qc < kTile / 64; ++qc) {
        const int q = i * kTile + qc * 64;
        const int y = (int)min((int64_t)b * p.T + q, rowsBT - 1);
        for (int ins = 0; ok && ins < L.dins; ++ins, ++it) {
          uint8_t* dst = stage(dper * 64 * 128);
          if (!ok) return;
          const uint32_t bar = stage_bar();
          for (int bx = 0; bx < dper; ++bx)
            tma_load_2d_pair(&tdy, bar, dst + bx * (64 * 128), ins * dn + (int)rank * (dn / 2) + bx * 64, y);
        }
      }
      const int per = (L.ncol / 2) / 64;
      for (int qc = 0; ok && do_dk && qc < kTile / 64; ++qc)
        for (int ins = 0; ok && ins < L.nins; ++ins, ++it) {
          uint8_t* dst = stage(per * 64 * 128);
          if (!ok) return;
          const uint32_t bar = stage_bar();
          for (int bx = 0; bx < per; ++bx) {
            const int col = ins * L.ncol + (int)rank * (L.ncol / 2) + bx * 64;
            const int cb = col / 64, gi = cb / L.rpb, x = (cb % L.rpb) * 64;
            const int64_t row = qk_row(p.q_base, p.q_sb, p.q_sbr, b, p.branch0 + gi, i * kTile + qc * 64);
            tma_load_2d_pair(&tq, bar, dst + bx * (64 * 128), x, (int)min(row, p.q_rows - 1));
          }
        }
    };
    for (int i = 0; ok && i < ni; ++i) {
      items_sdp(i0 + i);
      items_dkv(i0 + i);
    }
    if (rank == 0) {
      mbar_wait_drain(&in_full, 0);
      for (int k = (it > L.nst ? it - L.nst : 0); k < it; ++k) mbar_wait_drain(&r_full[k % L.nst], (k / L.nst) & 1u);
    }
  } else if (warp == 1 && lane == 0 && rank == 0) {
    // ---------------------------------------------------------------- MMA issuer (leader)
    const uint32_t idesc_s = idesc_f16(128, kTile, kBf16, false, false);
    const uint32_t idesc_v = idesc_f16(128, dn, kBf16, false, true);      // B = dY, MN-major
    const uint32_t idesc_k = idesc_f16(128, L.ncol, kBf16, false, true);  // B = Q, MN-major
    auto commit_both = [&](uint64_t* bar) {
      mma_commit<2>(smem_u32(bar));
      mma_commit<2>(mapa_shared(smem_u32(bar), 1));
    };
    int it = 0;
    auto take = [&](uint32_t* addr) -> bool {
      const int s = it % L.nst;
      if (!mbar_wait(&r_full[s], (it / L.nst) & 1u, ab, 23)) return false;
      tc_fence_after();
      *addr = smem_u32(smem + L.off_ring + s * kStage);
      return true;
    };
    auto give = [&]() { commit_both(&r_empty[it % L.nst]); ++it; };
    const uint32_t ka = smem_u32(smem + L.off_k), va = smem_u32(smem + L.off_v);
    const uint32_t pa = smem_u32(smem + L.off_p), dsa = smem_u32(smem + L.off_ds);
    bool ok = mbar_wait(&in_full, 0, ab, 21);
    tc_fence_after();
    for (int i = 0; ok && i < ni; ++i) {
      // S^T and dP^T need the previous tile's softmax to have read them
      if (i >= 1 && !(ok = mbar_wait(&p_full, (i - 1) & 1u, ab, 22))) break;
      for (int cc = 0; ok && cc < L.kw_chunks; ++cc) {
        uint32_t st;
        if (!(ok = take(&st))) break;
        const int nk16 = ((L.kw - cc * 128) >= 128 ? 128 : L.kw - cc * 128) / 16;
        for (int k = 0; k < nk16; ++k) {
          const uint64_t ad = sdesc_sw128(ka + (cc * 2 + (k >> 2)) * (kRows * 128) + (k & 3) * 32, 16, 1024);
          const uint64_t bd = sdesc_sw128(st + (k >> 2) * (kRows * 128) + (k & 3) * 32, 16, 1024);
          mma_f16_ss<2>(tmem + L.tmem_s, ad, bd, idesc_s, (cc | k) ? 1u : 0u);
        }
        give();
      }
      for (int cc = 0; ok && do_dk && cc < L.d_chunks; ++cc) {
        uint32_t st;
        if (!(ok = take(&st))) break;
        for (int k = 0; k < 8; ++k) {
          const uint64_t ad = sdesc_sw128(va + (cc * 2 + (k >> 2)) * (kRows * 128) + (k & 3) * 32, 16, 1024);
          const uint64_t bd = sdesc_sw128(st + (k >> 2) * (kRows * 128) + (k & 3) * 32, 16, 1024);
          mma_f16_ss<2>(tmem + L.tmem_p, ad, bd, idesc_s, (cc | k) ? 1u : 0u);
        }
        give();
      }
      if (!ok) break;
      commit_both(&s_full);
      // dV += P^T dY and dK += dS^T Q once the softmax wrote this tile's P^T / dS^T
      if (!(ok = mbar_wait(&p_full, i & 1u, ab, 24))) break;
      tc_fence_after();
      for (int qc = 0; ok && do_dv && qc < kTile / 64; ++qc)
        for (int ins = 0; ok && ins < L.dins; ++ins) {
          uint32_t st;
          if (!(ok = take(&st))) break;
          for (int kk = 0; kk < 4; ++kk) {
            const uint64_t ad = sdesc_sw128(pa + qc * (kRows * 128) + kk * 32, 16, 1024);
            const uint64_t bd = sdesc_sw128(st + kk * 16 * 128, 64 * 128, 1024);
            mma_f16_ss<2>(tmem + L.tmem_dv + ins * (dn / 2), ad, bd, idesc_v, (i | qc | kk) ? 1u : 0u);
          }
          give();
        }
      for (int qc = 0; ok && do_dk && qc < kTile / 64; ++qc)
        for (int ins = 0; ok && ins < L.nins; ++ins) {
          uint32_t st;
          if (!(ok = take(&st))) break;
          for (int kk = 0; kk < 4; ++kk) {
            const uint64_t ad = sdesc_sw128(dsa + qc * (kRows * 128) + kk * 32, 16, 1024);
            const uint64_t bd = sdesc_sw128(st + kk * 16 * 128, 64 * 128, 1024);
            mma_f16_ss<2>(tmem + L.tmem_dk + ins * (L.ncol / 2), ad, bd, idesc_k, (i | qc | kk) ? 1u : 0u);
          }
          give();
        }
      if (ok) commit_both(&pd_empty);
    }
    commit_both(&o_full);
    mbar_wait_drain(&o_full, 0);
  } else if (warp >= 2) {
    // ---------------------------------------------------------------- softmax + epilogue
    const int quad = warp & 3;
    const int l = quad * 32 + lane;
    const int r = l & 63, half = l >> 6;
    const int key = k0 + 64 * (int)rank + r;
    const bool live = key < p.T;
    const uint32_t lane_base = (uint32_t)(quad * 32) << 16;
    const uint32_t pf_leader = mapa_shared(smem_u32(&p_full), 0);
    const bool arriver = (warp == 2 && lane == 0);
    const float kLog2e = 1.4426950408889634f;
    const float gamma = *p.scale * rsqrtf((float)p.group);
    const float alpha = p.weight ? *p.weight : 1.f;
    const float scale2 = gamma * kLog2e;
    float* red = reinterpret_cast<float*>(smem + L.off_red);  // [0,128) lse2, [128,256) delta of the tile
    bool ok = true;
    for (int i = 0; i < ni; ++i) {
      const int qt = (i0 + i) * kTile;
      // stage this query tile's log-sum-exp and delta (128 each) in shared memory
      {
        const int tid = l;  // 0..127
        const int q = qt + tid;
        red[tid] = q < p.T ? p.lse[(int64_t)b * p.T + q] * kLog2e : 0.f;
        red[128 + tid] = q < p.T ? p.delta[(int64_t)b * p.T + q] : 0.f;
      }
      if (ok) ok = mbar_wait(&s_full, i & 1u, ab, 32);
      if (ok && i >= 1) ok = mbar_wait(&pd_empty, (i - 1) & 1u, ab, 33);
      named_bar_sync(1, 128);  // red[] visible
      ok = __all_sync(0xffffffffu, ok);
      if (ok) {
        tc_fence_after();
        for (int ch = 0; ch < 2; ++ch) {
          float sv[32], dpv[32];
          tmem_ld32(tmem + lane_base + L.tmem_s + ch * 32, sv);
          if (do_dk) {
            tmem_ld32(tmem + lane_base + L.tmem_p + ch * 32, dpv);
          } else {
#pragma unroll
            for (int e = 0; e < 32; ++e) dpv[e] = 0.f;
          }
          tmem_wait_ld();
          const int qc0 = half * 64 + ch * 32;  // query column inside the tile
          uint32_t pk[16], dk[16];
#pragma unroll
          for (int e = 0; e < 32; e += 2) {
            float pv2[2] = {0.f, 0.f}, dv2[2] = {0.f, 0.f};
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              const int q = qt + qc0 + e + h;
              const bool valid = live && q < p.T && (!p.causal || q >= key);
              if (valid) {
                const float pr = ex2(sv[e + h] * scale2 - red[qc0 + e + h]);
                pv2[h] = pr * alpha;
                dv2[h] = pv2[h] * (dpv[e + h] - red[128 + qc0 + e + h]);
              }
            }
            pk[e / 2] = pack2<T>(pv2[0], pv2[1]);
            dk[e / 2] = pack2<T>(dv2[0], dv2[1]);
          }
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            st_shared_v4(smem_u32(smem + L.off_p) + half * (kRows * 128) + sw128_offset(r, ch * 4 + e), pk[4 * e],
                         pk[4 * e + 1], pk[4 * e + 2], pk[4 * e + 3]);
            st_shared_v4(smem_u32(smem + L.off_ds) + half * (kRows * 128) + sw128_offset(r, ch * 4 + e), dk[4 * e],
                         dk[4 * e + 1], dk[4 * e + 2], dk[4 * e + 3]);
          }
        }
        fence_proxy_async();
      }
      tc_fence_before();
      named_bar_sync(1, 128);
      if (arriver) mbar_arrive_cluster(pf_leader);
    }
    if (ok) ok = mbar_wait(&o_full, 0, ab, 34);
    ok = __all_sync(0xffffffffu, ok);
    tc_fence_after();
    if (ok) {
      for (int ins = 0; do_dv && ins < L.dins; ++ins)
        for (int c = 0; c < dn / 2; c += 32) {
          float v[32];
          tmem_ld32(tmem + lane_base + L.tmem_dv + ins * (dn / 2) + c, v);
          tmem_wait_ld();
          if (live && p.dv) {
            float* dst = p.dv + ((int64_t)b * p.T + key) * p.D + ins * dn + half * (dn / 2) + c;
#pragma unroll
            for (int e = 0; e < 32; e += 4) {
              float4 o = *reinterpret_cast<float4*>(dst + e);
              o.x += v[e];
              o.y += v[e + 1];
              o.z += v[e + 2];
              o.w += v[e + 3];
              *reinterpret_cast<float4*>(dst + e) = o;
            }
          }
        }
      for (int ins = 0; do_dk && ins < L.nins; ++ins)
        for (int c = 0; c < L.ncol / 2; c += 32) {
          float v[32];
          tmem_ld32(tmem + lane_base + L.tmem_dk + ins * (L.ncol / 2) + c, v);
          tmem_wait_ld();
          if (live && p.dk) {
            const int col = ins * L.ncol + half * (L.ncol / 2) + c;
            const int gi = col / p.R;
            const int64_t row = qk_row(p.k_base, p.k_sb, p.k_sbr, b, p.branch0 + gi, key);
            float* dst = p.dk + row * p.R + (col % p.R);
#pragma unroll
            for (int e = 0; e < 32; e += 4) {
              float4 o = *reinterpret_cast<float4*>(dst + e);
              o.x += gamma * v[e];
              o.y += gamma * v[e + 1];
              o.z += gamma * v[e + 2];
              o.w += gamma * v[e + 3];
              *reinterpret_cast<float4*>(dst + e) = o;
            }
          }
        }
    }
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();
  if (warp == 1) tmem_dealloc<2>(tmem, L.tmem_cols);
}

// =============================================================================== delta
// delta[b, t] = <dY[b, t, :], Y[b, t, :]>  (one warp per row)
template <typename T>
__global__ void delta_kernel(const T* __restrict__ dy, const T* __restrict__ y, int64_t rows, int D,
                             float* __restrict__ delta) {
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (row >= rows) return;
  float acc = 0.f;
  for (int c = lane * 8; c < D; c += 256) {
    const uint4 a = *reinterpret_cast<const uint4*>(dy + row * D + c);
    const uint4 bq = *reinterpret_cast<const uint4*>(y + row * D + c);
    const uint32_t wa[4] = {a.x, a.y, a.z, a.w}, wb[4] = {bq.x, bq.y, bq.z, bq.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 fa = unpack2<T>(wa[e]), fb = unpack2<T>(wb[e]);
      acc = fmaf(fa.x, fb.x, fmaf(fa.y, fb.y, acc));
    }
  }
  for (int o = 16; o; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if (lane == 0) delta[row] = acc;
}

template <typename Kern, typename Layout>
int launch_pair(Kern kern, const Layout& L, int pairs, const CUtensorMap& tq, const CUtensorMap& tk,
                const CUtensorMap& tv, const CUtensorMap& tdy, const Params& p, cudaStream_t st) {
  const int smem = (L.smem < 120 * 1024 ? 120 * 1024 : L.smem) + 1024;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
    return record_cuda_error();
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  cfg.gridDim = dim3((unsigned)(2 * pairs), 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, kern, tq, tk, tv, tdy, p) != cudaSuccess) return record_cuda_error();
  note_launch();
  return DA_OK;
}

}  // namespace bwd
}  // namespace attn
}  // namespace da

extern "C" int da_attn_bwd_delta(const void* dy, const void* y, int64_t rows, int D, int dtype, float* delta,
                                 void* stream) {
  using namespace da;
  if (!dy || !y || !delta) return DA_ERR_NULL;
  if (dtype != DA_BF16 && dtype != DA_F16) return DA_ERR_DTYPE;
  if (int rc = bind_device(dy)) return rc;
  if (rows <= 0 || D <= 0 || D % 256) return DA_ERR_SHAPE;
  if ((reinterpret_cast<uintptr_t>(dy) | reinterpret_cast<uintptr_t>(y)) & 15) return DA_ERR_ALIGN;
  const int per_block = 8;
  const unsigned grid = (unsigned)((rows + per_block - 1) / per_block);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (dtype == DA_BF16)
    attn::bwd::delta_kernel<__nv_bfloat16><<<grid, 32 * per_block, 0, st>>>(
        static_cast<const __nv_bfloat16*>(dy), static_cast<const __nv_bfloat16*>(y), rows, D, delta);
  else
    attn::bwd::delta_kernel<__half><<<grid, 32 * per_block, 0, st>>>(
        static_cast<const __half*>(dy), static_cast<const __half*>(y), rows, D, delta);
  if (cudaPeekAtLastError() != cudaSuccess) return record_cuda_error();
  note_launch();
  return DA_OK;
}

extern "C" int da_attn_bwd(const void* q, int64_t q_rows, int64_t q_base, int64_t q_sb, int64_t q_sbr, const void* k,
                           int64_t k_rows, int64_t k_base, int64_t k_sb, int64_t k_sbr, const void* v, const void* dy,
                           int B, int T, int R, int D, int group, int branch0, int causal, int dtype, const float* scale,
                           const float* weight, const float* lse, const float* delta, float* dq, float* dk, float* dv,
                           float* dscale, int* status, void* stream) {
  using namespace da;
  using namespace da::attn::bwd;
  if (!q || !k || !v || !dy || !scale || !lse || !delta || !status) return DA_ERR_NULL;
  if (dtype != DA_BF16 && dtype != DA_F16) return DA_ERR_DTYPE;
  if (int rc = bind_device(q)) return rc;
  if (B <= 0 || T <= 0 || group < 1 || R <= 0 || R % 64 || branch0 < 0) return DA_ERR_SHAPE;
  if (D != 256 && D != 512) return DA_ERR_UNSUPPORTED;
  const int kw = group * R;
  if (kw != 128 && kw != 256 && kw != 512) return DA_ERR_UNSUPPORTED;
  const DqLayout LQ = dq_layout(group, R, D);
  // one key-parallel launch for dV and dK when both accumulators fit in TMEM, else one each
  const bool split = kv_layout(group, R, D, true, true).tmem_cols > 512;
  if (LQ.nst < 2 || LQ.tmem_p + 2 * (kTile / 2) > 512) return DA_ERR_UNSUPPORTED;
  if (kv_layout(group, R, D, true, false).tmem_cols > 512 || kv_layout(group, R, D, false, true).tmem_cols > 512 ||
      kv_layout(group, R, D, true, true).nst < 2)
    return DA_ERR_UNSUPPORTED;
  if ((reinterpret_cast<uintptr_t>(dq) | reinterpret_cast<uintptr_t>(dk) | reinterpret_cast<uintptr_t>(dv)) & 15)
    return DA_ERR_ALIGN;
  // every row a launch can address lies inside the row maps
  const int64_t tiles = (T + kTile - 1) / kTile;
  const int64_t q_last = q_base + (int64_t)(B - 1) * q_sb + (int64_t)(branch0 + group - 1) * q_sbr + (T - 1);
  const int64_t k_last = k_base + (int64_t)(B - 1) * k_sb + (int64_t)(branch0 + group - 1) * k_sbr + (T - 1);
  if (q_base < 0 || k_base < 0 || q_last >= q_rows || k_last >= k_rows) return DA_ERR_SHAPE;
  const CUtensorMapDataType tdt = dtype == DA_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUtensorMap tq, tk, tv, tdy;
  int rc = make_tmap_2d(&tq, q, tdt, 2, R, q_rows, (uint64_t)R * 2, 64, 64);
  if (rc) return rc;
  rc = make_tmap_2d(&tk, k, tdt, 2, R, k_rows, (uint64_t)R * 2, 64, 64);
  if (rc) return rc;
  rc = make_tmap_2d(&tv, v, tdt, 2, D, (uint64_t)B * T, (uint64_t)D * 2, 64, 64);
  if (rc) return rc;
  rc = make_tmap_2d(&tdy, dy, tdt, 2, D, (uint64_t)B * T, (uint64_t)D * 2, 64, 64);
  if (rc) return rc;
  Params p;
  p.q_rows = q_rows; p.q_base = q_base; p.q_sb = q_sb; p.q_sbr = q_sbr;
  p.k_rows = k_rows; p.k_base = k_base; p.k_sb = k_sb; p.k_sbr = k_sbr;
  p.B = B; p.T = T; p.R = R; p.D = D; p.group = group; p.branch0 = branch0; p.causal = causal;
  p.scale = scale; p.weight = weight; p.lse = lse; p.delta = delta;
  p.dq = dq; p.dk = dk; p.dv = dv; p.dscale = dscale; p.status = status;
  p.do_dv = dv != nullptr;
  p.do_dk = dk != nullptr;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int pairs = (int)(B * tiles);
  const bool bf16 = dtype == DA_BF16;
  if (dq || dscale) {
    rc = bf16 ? launch_pair(dq_kernel<__nv_bfloat16>, LQ, pairs, tq, tk, tv, tdy, p, st)
              : launch_pair(dq_kernel<__half>, LQ, pairs, tq, tk, tv, tdy, p, st);
    if (rc) return rc;
  }
  auto launch_kv = [&](bool with_dv, bool with_dk) -> int {
    Params pk = p;
    pk.do_dv = with_dv;
    pk.do_dk = with_dk;
    const KvLayout LK = kv_layout(group, R, D, with_dv, with_dk);
    return bf16 ? launch_pair(dkv_kernel<__nv_bfloat16>, LK, pairs, tq, tk, tv, tdy, pk, st)
                : launch_pair(dkv_kernel<__half>, LK, pairs, tq, tk, tv, tdy, pk, st);
  };
  if (dv && dk && split) {
    rc = launch_kv(true, false);
    if (rc) return rc;
    rc = launch_kv(false, true);
  } else if (dv || dk) {
    rc = launch_kv(dv != nullptr, dk != nullptr);
  }
  return rc;
}
