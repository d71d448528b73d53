// Outer routed attention with the alpha map mix fused, forward.
//
// Reference: routed_attention_reference (src/double_attention/ops.py:65-93),
// the map mix of SharedDictionaryAttention.forward (modules.py:265-272) and
// the Triton kernel it replaces (triton_kernels.py:674-811, :2022-2090):
//
//   A_s = softmax_causal(gamma_s Q_s K_s^T),   Y = sum_s alpha_s A_s V,
//
// with Q_s/K_s the routed vectors of map s (a group of concatenated branches
// scaled by group^-1/4 each, ops.py:113-131, i.e. gamma_s / sqrt(group) on
// the dot product) and V [B, T, D] the dense value shared by every map.
//
// One CTA pair (2-CTA cluster, cta_group::2 MMAs) owns 128 query rows of one
// sequence, 64 per CTA.  Per key tile of 64:
//   * S_s = Q_s K_s^T for every map lands folded in TMEM (32 columns each);
//   * the softmax warpgroup forms one probability tile P (bf16, shared mem);
//   * O += P V with V read straight from [B, T, D] as an MN-major operand;
//     D = 512 costs 256 TMEM columns per CTA thanks to the folded layout,
//     so the whole dense value is accumulated without splitting D.
// Scores are bounded by gamma_s ||q|| max||k||, which serves as a fixed
// softmax offset: no running-max rescaling of O.  With one map the row sum
// normalises O at the end.  With several maps a first sweep over the keys
// (Q K^T only) produces each map's exact log-sum-exp, and the second sweep
// builds the already-normalised mixture P = sum_s alpha_s exp(S_s - lse_s),
// so Y = P V needs a single P.V product for all maps.
#include <math.h>

#include "attn_common.h"
#include "common.cuh"
#include "host_util.h"

namespace da {
namespace attn {

// warps 0 and 8 keys (TMA), warp 1 score MMAs, warps 2-5 softmax/epilogue, warps 6 and 9 values
// (TMA), warp 7 P.V MMAs.  One warp's TMA stages complete one after another (about 1 us per stage
// for paired loads, nearly whatever the stage's size), so each stream has two producer warps
// taking alternate stages, and stages are made as large as the ring allows; the score and P.V
// products have their own issuing threads, so a P.V product never queues behind the key chunks
// of a score tile further ahead (and the reverse).
constexpr int kThreads = 320;
// kLat (fewer query tiles than SMs): one producer per stream, warps 0-7 only
template <bool kLat>
constexpr int fwd_threads() { return kLat ? 256 : kThreads; }
constexpr int kValueWarp = 6;
constexpr int kPvWarp = 7;
constexpr int kKeyWarp2 = 8, kValueWarp2 = 9;  // the second producer of each stream
constexpr int kRows = 64;       // query rows per CTA
constexpr int kMaxK = 8, kMaxV = 4, kMaxSB = 4, kMaxPB = 2;

// Tile plan.  The paired MMA reaches full rate only with N = 256 (its issue
// cost is ~46 cycles regardless of N), so a single map scores 256 keys per
// tile; mixed maps use 128-key tiles processed map by map through rotating
// TMEM score buffers.  Keys and values stream as 64-wide chunks through
// independent stage rings; everything is sized to fit 225 KB of shared
// memory and 512 TMEM columns.
struct Layout {
  int kw, nk, kchunks, rpb;
  int kbb, kslots;  // key chunks per TMA box (one issue), ring slots of kbb chunks
  int nc, npv, per;
  int q_bytes, k_stage, v_stage, p_bytes;
  int nks, nvs, nsb, npb;
  int off_q, off_k, off_v, off_p, off_red, smem;
  int tmem_s, s_cols, tmem_cols;
};

// coarse: many query tiles per SM (throughput-bound), so key boxes of up to 32 KB; otherwise every
// pair has only a few key tiles and 16 KB boxes let the first products start sooner.
__host__ __device__ inline Layout make_layout(int maps, int group, int R, int D, bool mix, bool coarse = true) {
  Layout L;
  L.kw = maps * group * R;
  L.rpb = R / 64;
  L.kchunks = group * L.rpb;
  L.nc = D < 256 ? D : 256;
  L.npv = D / L.nc;
  L.per = (L.nc / 2) / 64;
  L.q_bytes = kRows * L.kw * 2;
  L.v_stage = 64 * D;  // 64 keys x D/2 columns (bf16) per CTA
  // the 4 KB reduction buffer aliases P buffer 0: it is used only while no P.V product reads P
  const int red = 0;
  const int avail = 225 * 1024;
  L.nk = 0;
  for (int nk = mix ? 128 : 256; nk >= 128 && L.nk == 0; nk -= 128) {
    const int k_stage = (nk / 2) * 128, p_bytes = kRows * nk * 2;
    const int rest = avail - L.q_bytes - 2 * p_bytes - 2 * L.v_stage - red;
    if (rest >= (nk == 256 ? 4 : 2) * k_stage) {  // 256-key tiles only with two 32 KB key boxes
      L.nk = nk;
      L.k_stage = k_stage;
      L.p_bytes = p_bytes;
      L.npb = 2;
      L.nvs = 2;
      L.nks = rest / k_stage > kMaxK ? kMaxK : rest / k_stage;
    }
  }
  if (L.nk == 0) {  // last resort: single-buffered probabilities
    L.nk = 128;
    L.k_stage = 64 * 128;
    L.p_bytes = kRows * 128 * 2;
    L.npb = 1;
    L.nvs = 2;
    const int rest = avail - L.q_bytes - L.p_bytes - 2 * L.v_stage - red;
    L.nks = rest / L.k_stage > kMaxK ? kMaxK : rest / L.k_stage;
  }
  // The value ring feeds P.V, which waits for a whole softmax tile: stages
  // moved from the key ring (while it still holds a full score tile of keys)
  // let the values of the next tile land during that softmax.
  {
    const int ring = avail - L.q_bytes - L.npb * L.p_bytes - red;  // bytes of both rings
    while (L.nvs < kMaxV) {
      const int nks = (ring - (L.nvs + 1) * L.v_stage) / L.k_stage;
      if (nks < L.kchunks * (mix ? maps : 1) || nks < 2) break;  // keep a key tile of every map
      ++L.nvs;
      L.nks = nks > kMaxK ? kMaxK : nks;
    }
  }
  // A stage costs about the same whatever its size, so key chunks of the same rows are fetched
  // several column blocks per box (up to 32 KB) while the ring keeps two boxes, one per producer.
  L.kbb = 1;
  for (int b = 4; b >= 2; b /= 2)
    if (L.rpb % b == 0 && L.nks / b >= 2 && b * L.k_stage <= (coarse ? 32768 : 16384)) {
      L.kbb = b;
      break;
    }
  L.kslots = L.nks / L.kbb;
  L.nks = L.kslots * L.kbb;
  L.s_cols = L.nk / 2;
  L.tmem_s = D / 2;
  const int nsb = (512 - D / 2) / L.s_cols;
  L.nsb = nsb > kMaxSB ? kMaxSB : nsb;
  L.off_q = 0;
  L.off_k = L.off_q + L.q_bytes;
  L.off_v = L.off_k + L.nks * L.k_stage;
  L.off_p = L.off_v + L.nvs * L.v_stage;
  L.off_red = L.off_p;  // aliases P buffer 0 (p_bytes >= 16 KB > 4 KB)
  const int used = L.off_p + L.npb * L.p_bytes;
  L.smem = used < 120 * 1024 ? 120 * 1024 : used;  // one CTA per SM
  const int cols = D / 2 + L.nsb * L.s_cols;
  L.tmem_cols = cols <= 32 ? 32 : cols <= 64 ? 64 : cols <= 128 ? 128 : cols <= 256 ? 256 : 512;
  return L;
}

struct FwdParams {
  int64_t q_rows, q_base, q_sb, q_sbr;
  int64_t k_rows, k_base, k_sb, k_sbr;
  int B, T, R, D, maps, group, causal;
  int dsplit, Dp;  // value columns split over dsplit pairs of Dp columns each
  int coarse;      // tile plan for many query tiles per SM (make_layout)
  // Key-range split of the mixed path (few query tiles): ksplit pairs per query tile, each over its share
  // of the key tiles.  phase 0: both sweeps in one launch (ksplit 1); 1: the first sweep only, writing
  // each row's partial sums and maxima of every map to part_sum [ksplit][2][B][maps][T]; 2: the second
  // sweep from the combined partials, writing the partial outputs to part_o [ksplit][B][T][D] (fp32).
  int ksplit, phase;
  float* part_sum;
  float* part_o;
  int branch0[kMaxMaps];
  const float* scales;
  const float* weights;
  const float* key_norm_max;
  float key_norm_bound;
  void* y;
  float* lse;
  int* status;
  int* trace;
};

template <typename T, bool kMix, bool kLat>
__global__ void __launch_bounds__(fwd_threads<kLat>(), 1) attn_fwd_kernel(const __grid_constant__ CUtensorMap tq,
                                                               const __grid_constant__ CUtensorMap tk,
                                                               const __grid_constant__ CUtensorMap tv,
                                                               const FwdParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ uint64_t q_full, o_full;
  __shared__ uint64_t k_full[kMaxK], k_empty[kMaxK], v_full[kMaxV], v_empty[kMaxV];
  __shared__ uint64_t s_full[kMaxSB], p_full[kMaxSB], p_empty[kMaxPB], pv_full[kMaxPB];
  __shared__ uint32_t tmem_base;
  __shared__ int abort_flag;

  const Layout L = make_layout(p.maps, p.group, p.R, p.Dp, kMix, p.coarse != 0);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const uint32_t rank = cluster_ctarank() & 1u;
  const int tiles = (p.T + 127) / 128;
  const int dslice = (blockIdx.x / 2) % p.dsplit;  // the slices of one query tile run side by side
  const int dcol0 = dslice * p.Dp;
  const int khalf = (blockIdx.x / (2 * p.dsplit)) % p.ksplit;  // this pair's share of the key tiles
  const int pair = blockIdx.x / (2 * p.dsplit * p.ksplit);
  // heaviest (latest) query tiles of every sequence first, then the next heaviest: causal work per pair
  // varies with the tile, and this order (longest first across the whole grid) keeps the last wave short
  const int b = pair % p.B;
  const int t0 = (tiles - 1 - pair / p.B) * 128;
  const int nk = L.nk;
  const int nk_all = (p.T + nk - 1) / nk;
  const int nj_all = p.causal ? min(nk_all, (t0 + 127) / nk + 1) : nk_all;
  // key tiles [jb, jb + nj) of this pair's share (ksplit 1: all of them; the last share may be empty)
  const int jspan = (nj_all + p.ksplit - 1) / p.ksplit;
  const int jb = khalf * jspan;
  const int nj = max(0, min(nj_all, jb + jspan) - jb);
  const int maps = kMix ? p.maps : 1;
  // Key tiles are visited from a per-pair starting tile (any order gives the same sums: the softmax
  // offset is fixed), so the pairs of one sequence that run side by side read different key and
  // value lines instead of all requesting the same ones at once.
  const int rot = nj > 0 ? (blockIdx.x / 2) % nj : 0;
  auto ktile = [&](int j) { return jb + (j + rot) % nj; };  // key tile of the j-th visit
  const bool sweep1 = kMix && p.phase != 2;                // the log-sum-exp sweep runs here
  const bool sweep2 = !kMix || p.phase != 1;               // the probability sweep and P.V run here
  const int sweep_units = nj * maps;
  const int U = (sweep1 ? sweep_units : 0) + (sweep2 ? sweep_units : 0);  // S units: (sweep, key tile, map)
  const int u2 = sweep1 ? sweep_units : 0;                 // first unit of the P.V sweep
  const int nv = sweep2 ? nj : 0;                          // P.V key tiles
  Abort ab{&abort_flag, p.status};
  // post-mortem per-unit timeline of the first pair (debug trace only)
  int* ft = (p.trace && blockIdx.x < 2) ? p.trace + blockIdx.x * 4096 : nullptr;

  if (threadIdx.x == 0) {
    abort_flag = 0;
    mbar_init(&q_full, 1);
    mbar_init(&o_full, 1);
    for (int i = 0; i < kMaxK; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
    }
    for (int i = 0; i < kMaxV; ++i) {
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
    }
    for (int i = 0; i < kMaxSB; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 2);
    }
    for (int i = 0; i < kMaxPB; ++i) {
      mbar_init(&p_empty[i], 1);
      mbar_init(&pv_full[i], 2);  // a probability tile is complete in both CTAs
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

  constexpr int kProd = kLat ? 1 : 2;  // producers per stream
  if (warp == 0 || (!kLat && warp == kKeyWarp2)) {
    // ---------------------------------------------------------------- key producers (both CTAs): warp 0
    // takes the even key boxes (and loads q), warp 8 the odd ones
    if (lane == 0) {
      const int pi = warp == 0 ? 0 : 1;
      prefetch_tmap(&tk);
      if (pi == 0) {
        prefetch_tmap(&tq);
        if (rank == 0) mbar_arrive_expect_tx(&q_full, 2 * L.q_bytes);
        const uint32_t qf = mapa_shared(smem_u32(&q_full), 0);
        for (int s = 0; s < maps; ++s)
          for (int gi = 0; gi < p.group; ++gi) {
            const int64_t row = p.q_base + b * p.q_sb + (p.branch0[s] + gi) * p.q_sbr + t0 + 64 * (int)rank;
            const int y = (int)min(row, p.q_rows - 1);  // boxes never start outside the matrix
            for (int kb = 0; kb < L.rpb; ++kb)
              tma_load_2d_pair(&tq, qf, smem + L.off_q + ((s * p.group + gi) * L.rpb + kb) * (kRows * 128), kb * 64, y);
          }
      }
      int kx = 0;  // key boxes of both producers
      const int box_bytes = L.kbb * L.k_stage;
      for (int u = 0; u < U; ++u) {
        const int rem = u % sweep_units, j = rem / maps, s = rem % maps;
        bool ok = true;
        for (int c = 0; c < L.kchunks; c += L.kbb, ++kx) {
          if (kx % kProd != pi) continue;
          const int st = kx % L.kslots;
          if (!mbar_wait(&k_empty[st], ((kx / L.kslots) & 1u) ^ 1u, ab, 11)) { ok = false; break; }
          if (rank == 0) mbar_arrive_expect_tx(&k_full[st], 2 * box_bytes);
          const int gi = c / L.rpb, kb = c % L.rpb;  // kbb divides rpb: a box never spans two branches
          const int64_t row = p.k_base + b * p.k_sb + (p.branch0[s] + gi) * p.k_sbr + ktile(j) * nk + (int)rank * (nk / 2);
          tma_load_3d_pair(&tk, mapa_shared(smem_u32(&k_full[st]), 0), smem + L.off_k + st * box_bytes, 0,
                           (int)min(row, p.k_rows - 1), kb);
        }
        if (!ok) break;
      }
      if (rank == 0) {  // drain: none of this producer's loads may be in flight at teardown
        if (pi == 0) mbar_wait_drain(&q_full, 0);
        for (int c = (kx > L.kslots ? kx - L.kslots : 0); c < kx; ++c)
          if (c % kProd == pi) mbar_wait_drain(&k_full[c % L.kslots], (c / L.kslots) & 1u);
      }
    }
  } else if (warp == kValueWarp || (!kLat && warp == kValueWarp2)) {
    // ---------------------------------------------------------------- value producers: warp 6 even
    // stages, warp 9 odd ones
    if (lane == 0) {
      const int pi = warp == kValueWarp ? 0 : 1;
      prefetch_tmap(&tv);
      int vc = 0;
      const int64_t vrows = (int64_t)p.B * p.T;
      for (int v = 0; v < nv; ++v) {
        bool ok = true;
        for (int c = 0; c < nk / 64; ++c, ++vc) {
          if (vc % kProd != pi) continue;
          const int st = vc % L.nvs;
          if (!mbar_wait(&v_empty[st], ((vc / L.nvs) & 1u) ^ 1u, ab, 12)) { ok = false; break; }
          if (rank == 0) mbar_arrive_expect_tx(&v_full[st], 2 * L.v_stage);
          const uint32_t vf = mapa_shared(smem_u32(&v_full[st]), 0);
          const int y = (int)min((int64_t)b * p.T + ktile(v) * nk + c * 64, vrows - 1);
          // one box: 64 keys x this CTA's per column blocks of each of the npv value groups
          tma_load_4d_pair(&tv, vf, smem + L.off_v + st * L.v_stage, 0, y, (int)rank * L.per, dcol0 / L.nc);
        }
        if (!ok) break;
      }
      if (rank == 0)
        for (int c = (vc > L.nvs ? vc - L.nvs : 0); c < vc; ++c)
          if (c % kProd == pi) mbar_wait_drain(&v_full[c % L.nvs], (c / L.nvs) & 1u);
    }
  } else if (warp == 1 || warp == kPvWarp) {
    // ---------------------------------------------------------------- MMA issuers (leader): scores on warp 1,
    // P.V on warp 7
    if (rank == 0 && lane == 0) {
      const uint32_t idesc_s = idesc_f16(128, nk, std::is_same<T, __nv_bfloat16>::value, false, false);
      const uint32_t idesc_o = idesc_f16(128, L.nc, true, false, true);  // B = V, MN-major
      auto commit_both = [&](uint64_t* bar) { mma_commit_pair(smem_u32(bar)); };
      const uint32_t qa = smem_u32(smem + L.off_q);
      if (warp == 1) trace_at(ft, 0);
      bool ok = mbar_wait(&q_full, 0, ab, 21);
      if (warp == 1) trace_at(ft, 1);
      tc_fence_after();
      if (warp == 1) {
        // S units in order; a score buffer is reused once the softmax has consumed its previous unit.
        int kx = 0, st = 0;  // key boxes consumed, current slot
        for (int u = 0; ok && u < U; ++u) {
          const int sb = u % L.nsb;
          const int s = (u % sweep_units) % maps;
          if (u < 256) trace_at(ft, 1024 + 4 * u);
          if (u >= L.nsb && !mbar_wait(&p_full[sb], ((u - L.nsb) / L.nsb) & 1u, ab, 22)) { ok = false; break; }
          if (u < 256) trace_at(ft, 1025 + 4 * u);
          const uint32_t d = tmem + L.tmem_s + (uint32_t)(sb * L.s_cols);
          for (int c = 0; ok && c < L.kchunks; ++c) {
            const int cib = c % L.kbb;  // chunk inside the current box
            if (cib == 0) {
              st = kx % L.kslots;
              if (!mbar_wait(&k_full[st], (kx / L.kslots) & 1u, ab, 23)) { ok = false; break; }
              tc_fence_after();
            }
            const uint64_t ad0 = sdesc_sw128(qa + (s * L.kchunks + c) * (kRows * 128), 16, 1024);
            const uint64_t bd0 =
                sdesc_sw128(smem_u32(smem + L.off_k + (st * L.kbb + cib) * L.k_stage), 16, 1024);
#pragma unroll
            for (int kin = 0; kin < 4; ++kin)  // +32 B per K step of 16 = +2 in the encoded address
              mma_f16_ss<2>(d, ad0 + 2 * kin, bd0 + 2 * kin, idesc_s, (c | kin) ? 1u : 0u);
            if (cib == L.kbb - 1) {
              commit_both(&k_empty[st]);
              ++kx;
            }
          }
          if (!ok) break;
          commit_both(&s_full[sb]);
          if (u < 256) trace_at(ft, 1026 + 4 * u);
        }
      } else {
        // P.V per key tile, as soon as its probability tile and value rows are in shared memory.
        int vc = 0;
        for (int v = 0; ok && v < nv; ++v) {
          const int pb = v % L.npb;
          if (v < 256) trace_at(ft, 2048 + 4 * v);
          if (!mbar_wait(&pv_full[pb], (v / L.npb) & 1u, ab, 24)) { ok = false; break; }
          if (v < 256) trace_at(ft, 2049 + 4 * v);
          const uint32_t pa = smem_u32(smem + L.off_p + pb * L.p_bytes);
          for (int c = 0; ok && c < nk / 64; ++c, ++vc) {
            const int st = vc % L.nvs;
            if (!mbar_wait(&v_full[st], (vc / L.nvs) & 1u, ab, 25)) { ok = false; break; }
            tc_fence_after();
            const uint32_t va = smem_u32(smem + L.off_v + st * L.v_stage);
            for (int i = 0; i < L.npv; ++i) {
              // MN-major V: rows are keys (K), 128 B = 64 value columns (N);
              // LBO = distance between 64-column boxes, SBO = 8 key rows.
              const uint64_t bd0 = sdesc_sw128(va + i * L.per * (64 * 128), 64 * 128, 1024);
              const uint64_t ad0 = sdesc_sw128(pa + c * (kRows * 128), 16, 1024);
#pragma unroll
              for (int kk = 0; kk < 4; ++kk)  // K step of 16 keys: A +32 B (+2), B +16 rows x 128 B (+128)
                mma_f16_ss<2>(tmem + (uint32_t)(i * (L.nc / 2)), ad0 + 2 * kk, bd0 + 128 * kk, idesc_o,
                              (v | c | kk) ? 1u : 0u);
            }
            commit_both(&v_empty[st]);
          }
          if (!ok) break;
          commit_both(&p_empty[pb]);
          if (v < 256) trace_at(ft, 2050 + 4 * v);
        }
        commit_both(&o_full);
        mbar_wait_drain(&o_full, 0);  // every P.V product (and so every score product) has completed
      }
    }
  } else {
    // ---------------------------------------------------------------- softmax + epilogue
    const int quad = warp & 3;
    const int l = quad * 32 + lane;
    const int r = l & 63, half = l >> 6;
    const int t = t0 + 64 * (int)rank + r;  // query position of this thread's row
    const uint32_t lane_base = (uint32_t)(quad * 32) << 16;
    float* red = reinterpret_cast<float*>(smem + L.off_red);
    const uint32_t pf_leader = mapa_shared(smem_u32(&p_full[0]), 0);
    const bool arriver = (warp == 2 && lane == 0);
    const float kLog2e = 1.4426950408889634f;
    const int hc = nk / 2;  // key columns per thread per tile

    // (a pair with an empty key share has no score unit: it writes zero partials below)
    bool ok = U == 0 || mbar_wait(&s_full[0], 0, ab, 31);
    float scale2[kMaxMaps], bound2[kMaxMaps], off2[kMaxMaps], sum[kMaxMaps], mx[kMaxMaps];
    const float gsc = rsqrtf((float)p.group);
#pragma unroll
    for (int s = 0; s < kMaxMaps; ++s) {
      scale2[s] = bound2[s] = off2[s] = sum[s] = 0.f;
      mx[s] = -INFINITY;
      if (s < maps) {
        float qn2 = 0.f;
        if (ok) {
          const uint32_t qa = smem_u32(smem + L.off_q);
          for (int qb = s * L.kchunks; qb < (s + 1) * L.kchunks; ++qb)
#pragma unroll
            for (int c = 0; c < 8; ++c) {
              const uint4 w = ld_shared_v4(qa + qb * (kRows * 128) + sw128_offset(r, c));
              const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const float2 f = unpack2<T>(ws[e]);
                qn2 = fmaf(f.x, f.x, fmaf(f.y, f.y, qn2));
              }
            }
        }
        const float gamma = p.scales[s] * gsc;
        const float kmax = p.key_norm_max ? p.key_norm_max[b * p.maps + s] : p.key_norm_bound;
        scale2[s] = gamma * kLog2e;
        bound2[s] = gamma * sqrtf(qn2) * kmax * kLog2e;
      }
    }

    // Number of valid keys among the 32 columns starting at key k0.
    auto key_limit = [&](int k0) -> int {
      int lim = p.T - k0;
      if (p.causal) lim = min(lim, t - k0 + 1);
      return max(0, min(32, lim));
    };
    const uint32_t pv_leader = mapa_shared(smem_u32(&pv_full[0]), 0);
    // pb >= 0: this unit completed probability tile buffer pb
    auto finish_unit = [&](int u, int pb) {
      if (pb >= 0) fence_proxy_async();
      tc_fence_before();
      if (arriver && u < 256) trace_at(ft, 3074 + 4 * u);
      named_bar_sync(1, 128);
      if (arriver) {
        mbar_arrive_cluster_relaxed(pf_leader + (u % L.nsb) * 8);  // score buffer read
        if (pb >= 0) mbar_arrive_remote(pv_leader + pb * 8);         // probability tile written
      }
      if (arriver && u < 256) trace_at(ft, 3075 + 4 * u);
    };

    // ---- sweep 1 (several maps): exact per-map log-sum-exp
    if (kMix) {
      for (int u = 0; sweep1 && u < sweep_units; ++u) {
        const int j = u / maps, s = u % maps, sb = u % L.nsb;
        if (ok && u > 0) ok = mbar_wait(&s_full[sb], (u / L.nsb) & 1u, ab, 32);
        ok = __all_sync(0xffffffffu, ok);
        if (ok) {
          tc_fence_after();
          // the per-map state is indexed by a runtime map: accumulate in registers, store once
          const float sc = scale2[s], bd = bound2[s];
          float msum = 0.f, mmx = -INFINITY;
          for (int ch = 0; ch < hc / 32; ++ch) {
            float v[32];
            tmem_ld32(tmem + lane_base + L.tmem_s + (uint32_t)(sb * L.s_cols + ch * 32), v);
            tmem_wait_ld();
            const int lim = key_limit(ktile(j) * nk + half * hc + ch * 32);
#pragma unroll
            for (int i = 0; i < 32; ++i)
              if (i < lim) {
                const float a = v[i] * sc;
                mmx = fmaxf(mmx, a);
                msum += ex2(a - bd);
              }
          }
          sum[s] += msum;
          mx[s] = fmaxf(mx[s], mmx);
        }
        finish_unit(u, -1);
      }
      if (sweep1) {
        for (int s = 0; s < maps; ++s) {
          red[s * 128 + l] = sum[s];
          red[(4 + s) * 128 + l] = mx[s];
        }
        named_bar_sync(1, 128);
        for (int s = 0; s < maps; ++s) {
          sum[s] += red[s * 128 + (l ^ 64)];
          mx[s] = fmaxf(mx[s], red[(4 + s) * 128 + (l ^ 64)]);
        }
      }
      const bool live_row = t < p.T;
      const size_t pstride = (size_t)p.B * p.maps * p.T;  // one [B][maps][T] plane of the partials
      if (p.phase == 1 && live_row && half == 0) {       // this key share's row sums and maxima
        for (int s = 0; s < maps; ++s) {
          const size_t i = ((size_t)b * p.maps + s) * p.T + t;
          p.part_sum[(size_t)(2 * khalf) * pstride + i] = sum[s];
          p.part_sum[(size_t)(2 * khalf + 1) * pstride + i] = mx[s];
        }
      }
      if (p.phase == 2)  // every key share's sums, added in share order
        for (int s = 0; s < maps; ++s) {
          const size_t i = ((size_t)b * p.maps + s) * p.T + (live_row ? t : 0);
          sum[s] = 0.f;
          mx[s] = -INFINITY;
          for (int h = 0; h < p.ksplit; ++h) {
            sum[s] += p.part_sum[(size_t)(2 * h) * pstride + i];
            mx[s] = fmaxf(mx[s], p.part_sum[(size_t)(2 * h + 1) * pstride + i]);
          }
        }
      for (int s = 0; s < maps; ++s) {
        const float alpha = p.weights ? p.weights[s] : 1.f;
        const float lse2 = bound2[s] + log2f(sum[s]);
        off2[s] = lse2 - log2f(alpha);   // P term = 2^(S*scale2 - off2) = alpha * softmax
        bound2[s] = lse2;                // reported log-sum-exp (log2 units)
      }
      named_bar_sync(1, 128);
    }

    // ---- probability tiles for P.V
    float psum = 0.f, pmx = -INFINITY;
    float pm[kMix ? 64 : 1];
    for (int v = 0; v < nv; ++v) {
      const int pb = v % L.npb;
      const uint32_t pa = smem_u32(smem + L.off_p + pb * L.p_bytes);
      for (int s = 0; s < maps; ++s) {
        const int u = u2 + v * maps + s, sb = u % L.nsb;
        if (arriver && u < 256) trace_at(ft, 3072 + 4 * u);
        if (ok && u > 0) ok = mbar_wait(&s_full[sb], (u / L.nsb) & 1u, ab, 32);
        if (arriver && u < 256) trace_at(ft, 3073 + 4 * u);
        if (ok && s == 0 && v >= L.npb) ok = mbar_wait(&p_empty[pb], ((v - L.npb) / L.npb) & 1u, ab, 33);
        ok = __all_sync(0xffffffffu, ok);
        if (ok) {
          tc_fence_after();
          for (int ch = 0; ch < hc / 32; ++ch) {
            float sv[32];
            tmem_ld32(tmem + lane_base + L.tmem_s + (uint32_t)(sb * L.s_cols + ch * 32), sv);
            tmem_wait_ld();
            const int k0 = ktile(v) * nk + half * hc + ch * 32;
            const int lim = key_limit(k0);
            if constexpr (kMix) {
#pragma unroll
              for (int i = 0; i < 32; ++i) {
                const float e = i < lim ? ex2(sv[i] * scale2[s] - off2[s]) : 0.f;
                pm[ch * 32 + i] = s == 0 ? e : pm[ch * 32 + i] + e;
              }
            } else {
              uint32_t packed[16];
#pragma unroll
              for (int i = 0; i < 32; i += 2) {
                float e0 = 0.f, e1 = 0.f;
                if (i < lim) {
                  const float a = sv[i] * scale2[0];
                  pmx = fmaxf(pmx, a);
                  e0 = ex2(a - bound2[0]);
                }
                if (i + 1 < lim) {
                  const float a = sv[i + 1] * scale2[0];
                  pmx = fmaxf(pmx, a);
                  e1 = ex2(a - bound2[0]);
                }
                psum += e0 + e1;
                packed[i / 2] = pack_bf16x2(e0, e1);
              }
              const int kc = half * hc + ch * 32;  // key column inside the tile
              const uint32_t box = pa + (kc >> 6) * (kRows * 128);
              const int cb = (kc & 63) >> 3;
#pragma unroll
              for (int e = 0; e < 4; ++e)
                st_shared_v4(box + sw128_offset(r, cb + e), packed[4 * e], packed[4 * e + 1], packed[4 * e + 2],
                             packed[4 * e + 3]);
            }
          }
          if constexpr (kMix) {
            if (s == maps - 1) {
              for (int ch = 0; ch < hc / 32; ++ch) {
                const int kc = half * hc + ch * 32;
                const uint32_t box = pa + (kc >> 6) * (kRows * 128);
                const int cb = (kc & 63) >> 3;
#pragma unroll
                for (int e = 0; e < 4; ++e)
                  st_shared_v4(box + sw128_offset(r, cb + e),
                               pack_bf16x2(pm[ch * 32 + 8 * e], pm[ch * 32 + 8 * e + 1]),
                               pack_bf16x2(pm[ch * 32 + 8 * e + 2], pm[ch * 32 + 8 * e + 3]),
                               pack_bf16x2(pm[ch * 32 + 8 * e + 4], pm[ch * 32 + 8 * e + 5]),
                               pack_bf16x2(pm[ch * 32 + 8 * e + 6], pm[ch * 32 + 8 * e + 7]));
              }
            }
          }
        }
        finish_unit(u, (!kMix || s == maps - 1) ? pb : -1);
      }
    }

    // ---- epilogue
    if (ok) ok = mbar_wait(&o_full, 0, ab, 34);
    ok = __all_sync(0xffffffffu, ok);
    float inv_l = 1.f;
    if (!kMix) {
      red[l] = psum;
      red[128 + l] = pmx;
      named_bar_sync(1, 128);
      psum += red[l ^ 64];
      pmx = fmaxf(pmx, red[128 + (l ^ 64)]);
      named_bar_sync(1, 128);
      inv_l = 1.f / psum;
      mx[0] = pmx;
      bound2[0] = bound2[0] + log2f(psum);  // log-sum-exp in log2 units
    }
    tc_fence_after();
    const bool live = t < p.T;
    if (ok && p.phase != 1) {  // (the first-sweep launch of a key split has written its partials)
      const size_t row_off = ((size_t)b * p.T + (live ? t : 0)) * p.D;
      for (int i = 0; i < L.npv; ++i) {
        const int col0 = dcol0 + i * L.nc + half * (L.nc / 2);
        for (int c = 0; c < L.nc / 2; c += 32) {
          float o[32];
          if (nv > 0) {
            tmem_ld32(tmem + lane_base + (uint32_t)(i * (L.nc / 2) + c), o);
            tmem_wait_ld();
          } else {  // an empty key share adds nothing
#pragma unroll
            for (int e = 0; e < 32; ++e) o[e] = 0.f;
          }
          if (live && p.phase == 2) {  // this share's part of the (already normalised) output, fp32
            float4* dst = reinterpret_cast<float4*>(p.part_o + (size_t)khalf * p.B * p.T * p.D + row_off + col0 + c);
#pragma unroll
            for (int e = 0; e < 8; ++e) dst[e] = make_float4(o[4 * e], o[4 * e + 1], o[4 * e + 2], o[4 * e + 3]);
          } else if (live) {
            uint32_t w[16];
#pragma unroll
            for (int e = 0; e < 16; ++e) w[e] = pack2<T>(o[2 * e] * inv_l, o[2 * e + 1] * inv_l);
            uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<T*>(p.y) + row_off + col0 + c);
#pragma unroll
            for (int e = 0; e < 4; ++e) dst[e] = make_uint4(w[4 * e], w[4 * e + 1], w[4 * e + 2], w[4 * e + 3]);
          }
        }
      }
      // every value slice and key share forms the same row statistics: the first writes them
      if (live && half == 0 && dslice == 0 && khalf == 0) {
        const float kLn2 = 0.6931471805599453f;
        for (int s = 0; s < maps; ++s) {
          p.lse[((size_t)b * p.maps + s) * p.T + t] = bound2[s] * kLn2;
          // the largest term of a row must stay far above the fp32 range floor
          const float top = kMix ? mx[s] - (bound2[s] - log2f(sum[s])) : mx[0] - (bound2[0] - log2f(psum));
          if (top < -100.f) atomicOr(p.status, DA_DEV_LOW_MASS);
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync();
  if (warp == 1) tmem_dealloc<2>(tmem, L.tmem_cols);
}

// Value-column slices per query tile.  A tile's pair streams every key and
// value row of its causal prefix; when the tiles do not fill half the SMs,
// splitting D over 2 or 4 pairs (each recomputing the scores, R <= D) puts
// more SMs on the stream and shortens the longest pair.
inline int value_split(long pairs, int D, int sms) {
  int split = 1;
  while (split < 4 && D % (2 * split * 128) == 0 && pairs * 2 * split <= sms / 2) split *= 2;
  return split;
}

// Sum of the key shares' fp32 partial outputs, added in share order, in the output dtype.
template <typename T>
__global__ void __launch_bounds__(256) combine_kernel(const float* __restrict__ part_o, int ksplit, int64_t n, T* y) {
  grid_dependency_wait();
  grid_launch_dependents();
  const int64_t stride = (int64_t)gridDim.x * blockDim.x * 4;
  for (int64_t i = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * 4; i < n; i += stride) {
    float4 a = *reinterpret_cast<const float4*>(part_o + i);
    for (int h = 1; h < ksplit; ++h) {
      const float4 c = *reinterpret_cast<const float4*>(part_o + (size_t)h * n + i);
      a.x += c.x;
      a.y += c.y;
      a.z += c.z;
      a.w += c.w;
    }
    *reinterpret_cast<uint2*>(y + i) = make_uint2(pack2<T>(a.x, a.y), pack2<T>(a.z, a.w));
  }
}

template <typename T, bool kMix>
int launch(const AttnFwdArgs& a, cudaStream_t st) {
  const long pairs = (long)a.B * ((a.T + 127) / 128);
  const int ksplit = (kMix && a.part_sum) ? key_split(a.maps, pairs, sm_count()) : 1;
  const int dsplit = ksplit > 1 ? 1 : value_split(pairs, a.D, sm_count());
  const int Dp = a.D / dsplit;
  const bool coarse = pairs * dsplit >= sm_count();
  const Layout L = make_layout(a.maps, a.group, a.R, Dp, kMix, coarse);
  const CUtensorMapDataType qdt =
      std::is_same<T, __nv_bfloat16>::value ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUtensorMap tq, tk, tv;
  int rc = make_tmap_2d(&tq, a.q.ptr, qdt, 2, a.R, a.q.rows, (uint64_t)a.R * 2, 64, kRows);
  if (rc) return rc;
  {  // keys: [rows, R] as (64-column block, row, block index); a box is nk/2 rows x kbb blocks
    const uint64_t dims[3] = {64, (uint64_t)a.k.rows, (uint64_t)a.R / 64};
    const uint64_t strides[2] = {(uint64_t)a.R * 2, 128};
    const uint32_t box[3] = {64, (uint32_t)(L.nk / 2), (uint32_t)L.kbb};
    rc = make_tmap_blocks(&tk, a.k.ptr, qdt, 2, 3, dims, strides, box);
    if (rc) return rc;
  }
  {  // values: [B*T, D] as (64-column block, row, block inside an nc-wide group, group); a box is
     // 64 keys x this CTA's nc/128 blocks of each of the npv groups of its value slice
    const uint64_t dims[4] = {64, (uint64_t)a.B * a.T, (uint64_t)L.nc / 64, (uint64_t)a.D / L.nc};
    const uint64_t strides[3] = {(uint64_t)a.D * 2, 128, (uint64_t)L.nc * 2};
    const uint32_t box[4] = {64, 64, (uint32_t)L.per, (uint32_t)L.npv};
    rc = make_tmap_blocks(&tv, a.v, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, 4, dims, strides, box);
    if (rc) return rc;
  }
  FwdParams p;
  p.q_rows = a.q.rows;
  p.q_base = a.q.base;
  p.q_sb = a.q.sb;
  p.q_sbr = a.q.sbr;
  p.k_rows = a.k.rows;
  p.k_base = a.k.base;
  p.k_sb = a.k.sb;
  p.k_sbr = a.k.sbr;
  p.B = a.B;
  p.T = a.T;
  p.R = a.R;
  p.D = a.D;
  p.maps = a.maps;
  p.group = a.group;
  p.causal = a.causal;
  p.dsplit = dsplit;
  p.Dp = Dp;
  p.coarse = coarse ? 1 : 0;
  p.ksplit = ksplit;
  p.phase = 0;
  p.part_sum = a.part_sum;
  p.part_o = a.part_o;
  for (int s = 0; s < kMaxMaps; ++s) p.branch0[s] = a.branch0[s];
  p.scales = a.scales;
  p.weights = a.weights;
  p.key_norm_max = a.key_norm_max;
  p.key_norm_bound = a.key_norm_bound;
  p.y = a.y;
  p.lse = a.lse;
  p.status = a.status;
  p.trace = debug_trace();
  auto kern = coarse ? attn_fwd_kernel<T, kMix, false> : attn_fwd_kernel<T, kMix, true>;
  const int smem = L.smem + 1024;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
    return record_cuda_error();
  const dim3 grid((unsigned)(2 * pairs * dsplit * ksplit)), block(coarse ? fwd_threads<false>() : fwd_threads<true>());
  if (ksplit == 1) return launch_kernel(kern, grid, block, smem, st, true, tq, tk, tv, p);
  // key split: the first sweep over every share, then the second from the combined row sums, then the
  // shares' outputs added
  p.phase = 1;
  if (int rc = launch_kernel(kern, grid, block, smem, st, true, tq, tk, tv, p)) return rc;
  p.phase = 2;
  if (int rc = launch_kernel(kern, grid, block, smem, st, true, tq, tk, tv, p)) return rc;
  const int64_t n = (int64_t)a.B * a.T * a.D;
  const int64_t blocks = (n / 4 + 255) / 256;
  return launch_kernel(combine_kernel<T>, dim3((unsigned)(blocks < 4 * sm_count() ? blocks : 4 * sm_count())),
                       dim3(256), 0, st, false, (const float*)a.part_o, ksplit, n, reinterpret_cast<T*>(a.y));
}

int attn_fwd(const AttnFwdArgs& a, cudaStream_t st) {
  const bool bf16 = a.dtype == DA_BF16;
  if (a.maps > 1) return bf16 ? launch<__nv_bfloat16, true>(a, st) : launch<__half, true>(a, st);
  return bf16 ? launch<__nv_bfloat16, false>(a, st) : launch<__half, false>(a, st);
}

}  // namespace attn
}  // namespace da

extern "C" int64_t da_attn_fwd_workspace_size(int B, int T, int maps, int D) {
  if (B <= 0 || T <= 0 || maps < 1 || maps > da::attn::kMaxMaps || D <= 0) return -1;
  const long pairs = (long)B * ((T + 127) / 128);
  const int ks = da::attn::key_split(maps, pairs, da::sm_count());
  if (ks == 1) return 0;
  return ((int64_t)2 * ks * B * maps * T + (int64_t)ks * B * T * D) * (int64_t)sizeof(float);
}

namespace {

int attn_fwd_entry(const void* q, int64_t q_rows, int64_t q_base, int64_t q_sb, int64_t q_sbr, const void* k,
                   int64_t k_rows, int64_t k_base, int64_t k_sb, int64_t k_sbr, const void* v, int B, int T, int R,
                   int D, int maps, int group, const int* branch0, int causal, int dtype, const float* scales,
                   const float* weights, const float* key_norm_max, float key_norm_bound, void* y, float* lse,
                   void* workspace, int64_t workspace_bytes, int* status, void* stream) {
  using namespace da;
  if (!q || !k || !v || !branch0 || !scales || !y || !lse || !status) return DA_ERR_NULL;
  if (int rc = bind_device(q)) return rc;
  if (dtype != DA_BF16 && dtype != DA_F16) return DA_ERR_DTYPE;
  if (B <= 0 || T <= 0 || maps < 1 || maps > attn::kMaxMaps || group < 1) return DA_ERR_SHAPE;
  if (R % 64 || R <= 0) return DA_ERR_UNSUPPORTED;
  if (maps * group * R > 512) return DA_ERR_UNSUPPORTED;  // Q/K width per pair of rows
  if (D != 128 && D != 256 && D != 512) return DA_ERR_UNSUPPORTED;
  if (maps > 1 && !weights) return DA_ERR_NULL;
  {
    const attn::Layout L = attn::make_layout(maps, group, R, D, maps > 1);
    if (L.nks < 2 || L.nsb < 2) return DA_ERR_UNSUPPORTED;  // tile plan does not fit
  }
  if ((reinterpret_cast<uintptr_t>(y) & 15) || (reinterpret_cast<uintptr_t>(v) & 15)) return DA_ERR_ALIGN;
  attn::AttnFwdArgs a;
  a.q = {q, q_rows, q_base, q_sb, q_sbr};
  a.k = {k, k_rows, k_base, k_sb, k_sbr};
  a.v = v;
  a.B = B;
  a.T = T;
  a.R = R;
  a.D = D;
  a.maps = maps;
  a.group = group;
  for (int s = 0; s < attn::kMaxMaps; ++s) a.branch0[s] = s < maps ? branch0[s] : 0;
  a.causal = causal;
  a.dtype = dtype;
  a.scales = scales;
  a.weights = weights;
  a.key_norm_max = key_norm_max;
  a.key_norm_bound = key_norm_bound;
  a.y = y;
  a.lse = lse;
  a.status = status;
  if (workspace) {  // a key split runs when the size query asks for a workspace
    const int64_t need = da_attn_fwd_workspace_size(B, T, maps, D);
    if (need > 0) {
      if (workspace_bytes < need) return DA_ERR_WORKSPACE;
      if (reinterpret_cast<uintptr_t>(workspace) & 15) return DA_ERR_ALIGN;
      const int ks = attn::key_split(maps, (long)B * ((T + 127) / 128), sm_count());
      a.part_sum = static_cast<float*>(workspace);
      a.part_o = a.part_sum + (size_t)2 * ks * B * maps * T;
    }
  }
  return attn::attn_fwd(a, static_cast<cudaStream_t>(stream));
}

}  // namespace

extern "C" int da_attn_fwd(const void* q, int64_t q_rows, int64_t q_base, int64_t q_sb, int64_t q_sbr,
                           const void* k, int64_t k_rows, int64_t k_base, int64_t k_sb, int64_t k_sbr,
                           const void* v, int B, int T, int R, int D, int maps, int group, const int* branch0,
                           int causal, int dtype, const float* scales, const float* weights,
                           const float* key_norm_max, float key_norm_bound, void* y, float* lse, int* status,
                           void* stream) {
  return attn_fwd_entry(q, q_rows, q_base, q_sb, q_sbr, k, k_rows, k_base, k_sb, k_sbr, v, B, T, R, D, maps, group,
                        branch0, causal, dtype, scales, weights, key_norm_max, key_norm_bound, y, lse, nullptr, 0,
                        status, stream);
}

extern "C" int da_attn_fwd_ws(const void* q, int64_t q_rows, int64_t q_base, int64_t q_sb, int64_t q_sbr,
                              const void* k, int64_t k_rows, int64_t k_base, int64_t k_sb, int64_t k_sbr,
                              const void* v, int B, int T, int R, int D, int maps, int group, const int* branch0,
                              int causal, int dtype, const float* scales, const float* weights,
                              const float* key_norm_max, float key_norm_bound, void* y, float* lse, void* workspace,
                              int64_t workspace_bytes, int* status, void* stream) {
  return attn_fwd_entry(q, q_rows, q_base, q_sb, q_sbr, k, k_rows, k_base, k_sb, k_sbr, v, B, T, R, D, maps, group,
                        branch0, causal, dtype, scales, weights, key_norm_max, key_norm_bound, y, lse, workspace,
                        workspace_bytes, status, stream);
}
