// Outer routed attention, backward, all maps of a mixed attention at once.
//
// Reference: _routed_attention_triton_backward (triton_kernels.py:2093-2263)
// plus the gradient of the alpha mix (modules.py:265-272).  With maps s,
// S_s = gamma_s/sqrt(group) Q_s K_s^T, P_s = exp(S_s - lse_s) (causal) and
// Y = sum_s alpha_s P_s V:
//   dP      = dY V^T                       (the same for every map)
//   delta_s = sum_k P_s dP = <dY, P_s V>   (row sums)
//   dS_s    = alpha_s P_s (dP - delta_s)
//   dQ_s    = gamma_eff,s dS_s K_s,  dK_s = gamma_eff,s dS_s^T Q_s
//   dV      = (sum_s alpha_s P_s)^T dY     (one product for all maps)
//   dgamma_s = alpha_s sum (P dP S - (sum P dP)(sum P S)) / sqrt(group) per row
//   dalpha_s = sum_rows delta_s
// Three paired-CTA kernels (2-CTA clusters, cta_group::2 MMAs, folded TMEM):
//   * query-parallel (dQ): per key tile, dP once, then S_s map by map; with
//     no delta given, a first sweep over the keys computes delta_s exactly
//     (fp32 P and dP) and the second forms dS_s and accumulates dQ_s;
//   * key-parallel (dK): per query tile, dP^T once, then S_s^T, dS_s^T and dK_s
//     map by map;
//   * key-parallel (dV): per query tile, S_s^T map by map into the mixed
//     probabilities, then one dV product.
// Score and dP tiles are double-buffered in TMEM, so the tensor core works on
// the next unit while a softmax warpgroup handles the current one (dQ and dK:
// the two warpgroups take alternate units).  Operands stream through rings of
// 16 KB stages, each filled in exactly the order its MMA issuer consumes it.
// Each product is a chain of dependent K = 16 instructions into one TMEM
// accumulator; measured on B200, a lone chain of paired M = 128 instructions
// issues one per ~205 cycles whether N is 128 or 256, two interleaved chains
// ~146 and three ~97, so the score, dP and accumulation products have their
// own issuing threads and their chains interleave in the tensor pipe.
#include <math.h>

#include "attn_common.h"
#include "common.cuh"
#include "host_util.h"

namespace da {
namespace attn {
namespace bwdm {

// warps 0 and 12: TMA producers of the resident rows and the score / accumulation operands (even and
// odd ring stages); warp 1: their MMA issuer; warps 2-5 and 8-11: softmax, two warpgroups (dQ and dK:
// taking alternate units, each thread all 64 columns of its row half; dV: each taking 32 of a thread's
// 64 columns of every unit; one warp per SM sub-partition in each); warps 6 and 13: TMA producers of the dP operands (V and dY);
// warp 7: the dP issuer.  dP runs as its own stream so the other products never wait behind it.  A
// producer warp completes about one paired stage per microsecond whatever the stage holds, so each
// ring has two.
constexpr int kThreads = 448;
constexpr int kDpWarp = 6;
constexpr int kAccProducer = 12;  // TMA producer of the accumulation ring
constexpr int kAccIssuer = 13;    // issuer of the accumulating products (dQ, dK or dV)
constexpr int kSoftmax2 = 8;      // first warp of the second softmax warpgroup
constexpr int kRows = 64;      // rows (queries or keys) per CTA
constexpr int kTile = 128;     // columns (keys or queries) per tile and pair
constexpr int kStage = 16384;  // main ring stage bytes
constexpr int kDpBlocks = 1;    // 64-column blocks of each of V and dY per dP ring stage (dK kernel)
constexpr int kDpStage = 2 * kDpBlocks * kRows * 128;
constexpr int kDpStages = 3;
// The dQ kernel's dP stream (formed twice per key tile, in the delta sweep and the dS sweep): stages of
// kDpBlocksQ 64-column blocks of each of V and dY.  Measured: one-block stages x 3 (with 3 score-ring
// and 2 accumulation-ring stages) and two-block stages x 2 (2 + 2) run alike, as do other splits of
// the same ring space; the kernels are paced by their MMA chains (see the issuers), not by the rings.
constexpr int kDpBlocksQ = 1;
constexpr int kDpStageQ = 2 * kDpBlocksQ * kRows * 128;
constexpr int kDpStagesQ = 3;
constexpr int kAccStages = 2;  // accumulation-ring stages of the dQ and dK kernels
constexpr int kMaxStages = 8;
constexpr int kBox = kRows * 128;  // one 64-row x 128-byte swizzled box

struct Params {
  int64_t q_rows, q_base, q_sb, q_sbr;
  int64_t k_rows, k_base, k_sb, k_sbr;
  int B, T, R, D, maps, group, causal;
  int branch0[kMaxMaps];
  const float* scales;   // [maps] gamma_s
  const float* weights;  // [maps] alpha_s, or null for 1
  const float* lse;      // [B, maps, T] natural log
  float* delta;          // [B, maps, T]: read, or written by the dQ kernel's first sweep
  int delta_given;
  float* dq;             // fp32 [q_rows, R], +=  (overwrite: [q_rows, R] in the input dtype, =)
  float* dk;             // fp32 [k_rows, R], +=  (overwrite: as dq)
  float* dv;             // fp32 [B*T, D], +=     (overwrite: [B*T, D] in the input dtype, =)
  int overwrite;         // every gradient row has one writer: store it in the input dtype
  // Few pairs (several maps): every pair's key range (dQ, delta) or query range (dK, dV) split into ksplit
  // shares, each writing fp32 partial rows (zeros for an empty share) that a combine kernel adds in share
  // order.
  int ksplit;
  float* part;           // [ksplit][part_rows][R or D]: dQ/dK rows (b, map, branch, t), dV rows (b, t)
  int64_t part_rows;
  float* delta_part;     // delta sweep: [ksplit][B][maps][T]
  float* dscale;         // [maps] d gamma_s, += (may be null)
  float* dweight;        // [maps] d alpha_s, += (dQ kernel with the first sweep; may be null)
  float* scalar_part;    // [2, 2 * pairs, 4, maps]: per-(CTA, warp) partial sums of d alpha_s and d gamma_s,
                         // added in a fixed order by scalar_reduce_kernel (null: fp32 atomics)
  int* status;
  int* trace;            // optional post-mortem timeline (debug)
};

DA_DEV int64_t row_of(int64_t base, int64_t sb, int64_t sbr, int b, int branch, int t) {
  return base + (int64_t)b * sb + (int64_t)branch * sbr + t;
}

struct Layout {
  int kw, W, rpb, ncol, nins;
  int acc_merge;  // the accumulation operand (dQ: K, dK: Q rows, MN-major) comes as one 128-row box per stage
  int off_a, off_b, off_t, off_red, off_ring, nst, off_qring, nsq, off_pring, nsp, smem;
  int tmem_acc, tmem_s, tmem_p, tmem_cols;
  int nsb;  // score (TMEM) buffers
};

// kind 0: dQ, 1: dK, 2: dV.  The kernel's own rows of Q (dQ) or K (dK, dV) of
// every map stay resident; V and dY, needed only for dP, stream through the
// ring a 64-column chunk of each per stage (resident they would leave room
// for 3 stages, too few to cover the load latency).
__host__ __device__ inline Layout make_layout(int kind, int maps, int group, int R, int D) {
  Layout L;
  L.kw = group * R;
  L.W = maps * L.kw;
  L.rpb = R / 64;
  L.ncol = L.kw < 256 ? L.kw : 256;
  L.nins = L.kw / L.ncol;
  L.acc_merge = kind != 2 && L.ncol == 128;  // one 64-column block per CTA: both 64-row chunks in one box
  L.off_a = 0;
  L.off_b = L.off_a + kRows * L.W * 2;
  const int b_bytes = 0;
  L.off_t = L.off_b + b_bytes;                 // two dS / P tiles
  // The dQ kernel's row reductions (delta at the end of the first sweep, d gamma after the last product)
  // borrow the dS tiles' space, idle at both points; the key-parallel kernels stage each query tile's
  // log-sum-exp and delta in a buffer of their own (the dK kernel one per warpgroup).
  L.off_red = kind == 0 ? L.off_t : L.off_t + 2 * kRows * kTile * 2;
  L.off_ring = kind == 0 ? L.off_t + 2 * kRows * kTile * 2 : L.off_red + (kind == 1 ? 16384 : 8192);
  const int avail = 225 * 1024 - L.off_ring;
  // Stage depth over stage size: the score / accumulation ring holds a stage for the dS product of the
  // unit in the softmax while the next units' score operands load, so with three stages a score operand
  // waited on the product two units back and the load latency surfaced in every unit.  The dP operands
  // therefore come as three 16 KB stages (one 64-column block of each of V and dY), leaving four or
  // more ring stages.
  L.nsp = kind == 2 ? 0 : (kind == 1 ? kDpStages - 1 : kDpStagesQ);
  const int dp_stage = kind == 0 ? kDpStageQ : kDpStage;
  int rest = (avail - L.nsp * dp_stage) / kStage;
  if (rest > 2 * kMaxStages) rest = 2 * kMaxStages;
  // Two rings, each with its own producer and issuer: the score operands (run ahead as far as the two
  // score buffers allow) and the accumulation operands (held until the softmax hands over the unit's dS
  // or P tile).  The dV kernel's accumulation items are the four dY stages of a query tile.
  L.nsq = kind == 2 ? (rest - 3 < 4 ? rest - 3 : 4) : kAccStages;
  if (L.nsq > kMaxStages) L.nsq = kMaxStages;
  L.nst = rest - L.nsq;
  if (L.nst > kMaxStages) L.nst = kMaxStages;
  L.off_qring = L.off_ring + L.nst * kStage;
  L.off_pring = L.off_qring + L.nsq * kStage;
  L.smem = L.off_pring + L.nsp * dp_stage;
  L.tmem_acc = 0;
  const int acc = kind == 2 ? D / 2 : L.W / 2;
  L.tmem_s = acc;
  // score buffers: the dV kernel has no dP tiles, so its TMEM holds four (score products run three units
  // ahead of the softmax); the dQ and dK kernels hold two next to their two dP buffers
  L.nsb = kind == 2 ? 4 : 2;
  L.tmem_p = L.tmem_s + L.nsb * (kTile / 2);
  const int cols = L.tmem_p + (kind == 2 ? 0 : 2 * (kTile / 2));
  L.tmem_cols = cols <= 256 ? 256 : (cols <= 512 ? 512 : 1024);
  return L;
}

// Loads one 64-row K-major chunk of 128 map-local columns of a row-mapped [rows, R] matrix
// (map s, `nb` boxes) for rows starting at `t` of batch `b`.
struct MapRows {
  int64_t rows, base, sb, sbr;
};

DA_DEV void load_map_chunk(const CUtensorMap* tm, const MapRows& m, const Params& p, uint32_t bar, uint8_t* dst,
                           int b, int s, int cc, int nb, int t) {
  for (int bx = 0; bx < nb; ++bx) {
    const int mb = cc * 2 + bx, gi = mb / (p.R / 64), x = (mb % (p.R / 64)) * 64;
    const int64_t row = row_of(m.base, m.sb, m.sbr, b, p.branch0[s] + gi, t);
    tma_load_2d_pair(tm, bar, dst + bx * kBox, x, (int)min(row, m.rows - 1));
  }
}

// 32 consecutive gradient values of one row: added to the fp32 accumulator, or (overwrite) stored in
// the input dtype.
template <typename T>
DA_DEV void store_grad32(float* acc, int64_t off, const float* v, float scale, bool overwrite) {
  if (overwrite) {
    uint32_t w[16];
#pragma unroll
    for (int e = 0; e < 16; ++e) w[e] = pack2<T>(scale * v[2 * e], scale * v[2 * e + 1]);
    uint4* d = reinterpret_cast<uint4*>(reinterpret_cast<T*>(acc) + off);
#pragma unroll
    for (int e = 0; e < 4; ++e) d[e] = make_uint4(w[4 * e], w[4 * e + 1], w[4 * e + 2], w[4 * e + 3]);
    return;
  }
  float* dst = acc + off;
#pragma unroll
  for (int e = 0; e < 32; e += 4) {
    float4 o = *reinterpret_cast<float4*>(dst + e);
    o.x += scale * v[e];
    o.y += scale * v[e + 1];
    o.z += scale * v[e + 2];
    o.w += scale * v[e + 3];
    *reinterpret_cast<float4*>(dst + e) = o;
  }
}

// 32 consecutive values of one row of this share's fp32 partial plane (plain stores; an empty share stores
// zeros, so every partial row the combine reads is written).
DA_DEV void store_part32(float* part, int64_t off, const float* v, float scale, bool empty) {
  float4* d = reinterpret_cast<float4*>(part + off);
#pragma unroll
  for (int e = 0; e < 8; ++e)
    d[e] = empty ? make_float4(0.f, 0.f, 0.f, 0.f)
                 : make_float4(scale * v[4 * e], scale * v[4 * e + 1], scale * v[4 * e + 2], scale * v[4 * e + 3]);
}

// =============================================================================== dQ kernel
template <typename T>
__global__ void __launch_bounds__(kThreads, 1) dq_mixed_kernel(const __grid_constant__ CUtensorMap tq,
                                                               const __grid_constant__ CUtensorMap tk,
                                                               const __grid_constant__ CUtensorMap tv,
                                                               const __grid_constant__ CUtensorMap tdy,
                                                               const __grid_constant__ CUtensorMap tacc,
                                                               const Params p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ uint64_t in_full, o_full, s_done, r_full[kMaxStages], r_empty[kMaxStages];
  __shared__ uint64_t q_full[kMaxStages], q_empty[kMaxStages];
  __shared__ uint64_t rp_full[kMaxStages], rp_empty[kMaxStages], dp_done;
  __shared__ uint64_t s_full[2], s_free[2], p_full[2], dp_full[2], dp_free[2], ds_empty[2];
  __shared__ uint32_t tmem_base;
  __shared__ int abort_flag;

  constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
  const Layout L = make_layout(0, p.maps, p.group, p.R, p.D);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const uint32_t rank = cluster_ctarank() & 1u;
  const int tiles = (p.T + kTile - 1) / kTile;
  const int khalf = (blockIdx.x / 2) % p.ksplit;  // this pair's share of its key tiles
  const int pair = blockIdx.x / (2 * p.ksplit);
  // longest pairs first across every sequence (the latest query tiles see the most keys)
  const int b = pair % p.B;
  const int t0 = (tiles - 1 - pair / p.B) * kTile;
  const int nj_all = p.causal ? t0 / kTile + 1 : tiles;
  const int jspan = (nj_all + p.ksplit - 1) / p.ksplit;
  const int jb = khalf * jspan;                           // first key tile of this share
  const int nj = max(0, min(nj_all, jb + jspan) - jb);    // (the last share may be empty)
  const int maps = p.maps;
  // Without a given delta the first sweep computes it; with neither dQ nor d gamma requested that sweep
  // is all the launch does (the dK kernel can then start while another launch forms dQ).
  const bool delta_only = !p.delta_given && !p.dq && !p.dscale;
  const int sweeps = (p.delta_given || delta_only) ? 1 : 2;
  const int per_sweep = nj * maps;
  const int U = sweeps * per_sweep;
  const int u_dq = delta_only ? U : (sweeps - 1) * per_sweep;  // first unit that forms dS and accumulates dQ
  const MapRows qm{p.q_rows, p.q_base, p.q_sb, p.q_sbr}, km{p.k_rows, p.k_base, p.k_sb, p.k_sbr};
  const int64_t rowsBT = (int64_t)p.B * p.T;
  Abort ab{&abort_flag, p.status};
  // post-mortem per-unit timeline of the first pair (debug trace only): per CTA 16384 words, dP issuer
  // at 4g, MMA issuer at 1024 + 8u, softmax at 5120 + 4u, ring producers at 7168 + 4096 ring + 2 item
  int* ft = (p.trace && blockIdx.x < 2) ? p.trace + blockIdx.x * 16384 : nullptr;

  if (threadIdx.x == 0) {
    abort_flag = 0;
    mbar_init(&in_full, 1);
    mbar_init(&o_full, 1);
    mbar_init(&s_done, 1);
    for (int i = 0; i < kMaxStages; ++i) {
      mbar_init(&r_full[i], 1);
      mbar_init(&r_empty[i], 1);
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 1);
      mbar_init(&rp_full[i], 1);
      mbar_init(&rp_empty[i], 1);
    }
    mbar_init(&dp_done, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], 8);  // score tile read out of TMEM: each warp of the owning warpgroup, both CTAs
      mbar_init(&p_full[i], 2);
      mbar_init(&dp_full[i], 1);
      // dP tile released by each softmax warp that read it, in both CTAs (with one map a key tile is one
      // unit, read by one warpgroup)
      mbar_init(&dp_free[i], maps == 1 ? 8 : 16);
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
  grid_dependency_wait();  // predecessors' outputs are visible from here on
  grid_launch_dependents();
  const uint32_t tmem = tmem_base;

  // unit u -> (sweep tile g, tile j within the sweep, map s)
  auto unit_j = [&](int u) { return (u % per_sweep) / maps; };
  auto unit_s = [&](int u) { return u % maps; };
  auto unit_g = [&](int u) { return u / maps; };  // sweep-major tile counter (dP products)

  const int tq_row = t0 + 64 * (int)rank;
  const int dy_row = (int)min((int64_t)b * p.T + tq_row, rowsBT - 1);
  const int dps = sweeps * nj;  // dP products: one per key tile and sweep
  if ((warp == 0 || warp == kAccProducer) && lane == 0) {
    // ---------------------------------------------------------------- TMA producers: warp 0 loads the
    // resident Q rows, then the score operands (K rows of this CTA's 64 keys, per map) into the score
    // ring; warp 12 loads the dQ operands (K rows of all 128 keys, MN-major) into the accumulation ring
    const int acc = warp == kAccProducer ? 1 : 0;
    prefetch_tmap(&tk);
    prefetch_tmap(&tacc);
    if (!acc) {
      prefetch_tmap(&tq);
      const uint32_t inf = mapa_shared(smem_u32(&in_full), 0);
      if (rank == 0) mbar_arrive_expect_tx(&in_full, 2 * (kRows * L.W * 2));
      for (int s = 0; s < maps; ++s)
        for (int cc = 0; cc < L.kw / 128; ++cc)
          load_map_chunk(&tq, qm, p, inf, smem + L.off_a + (s * (L.kw / 64) + cc * 2) * kBox, b, s, cc, 2, tq_row);
    }
    const int nst = acc ? L.nsq : L.nst;
    uint64_t* fullb = acc ? q_full : r_full;
    uint64_t* emptyb = acc ? q_empty : r_empty;
    uint8_t* ring = smem + (acc ? L.off_qring : L.off_ring);
    int it = 0;
    bool ok = true;
    auto stage = [&](int bytes) -> uint8_t* {
      const int st = it % nst;
      if (it < 2048) trace_at(ft, 7168 + 4096 * acc + 2 * it);
      if (!mbar_wait(&emptyb[st], ((it / nst) & 1u) ^ 1u, ab, 11 + acc)) { ok = false; return nullptr; }
      if (it < 2048) trace_at(ft, 7169 + 4096 * acc + 2 * it);
      if (rank == 0) mbar_arrive_expect_tx(&fullb[st], 2 * bytes);
      return ring + st * kStage;
    };
    auto stage_bar = [&]() { return mapa_shared(smem_u32(&fullb[it % nst]), 0); };
    auto emit_s = [&](int u) {  // key rows of map s for this CTA's 64 keys
      const int krow0 = (jb + unit_j(u)) * kTile + 64 * (int)rank;
      for (int cc = 0; ok && cc < L.kw / 128; ++cc, ++it) {
        uint8_t* dst = stage(2 * kBox);
        if (!ok) return;
        load_map_chunk(&tk, km, p, stage_bar(), dst, b, unit_s(u), cc, 2, krow0);
      }
    };
    auto emit_dq = [&](int u) {  // key rows of all 128 keys, MN-major, this CTA's half of each N block
      const int per = (L.ncol / 2) / 64, s = unit_s(u), j = unit_j(u);
      if (L.acc_merge) {  // one stage per N block: a 128-key x 64-column box
        for (int ins = 0; ok && ins < L.nins; ++ins, ++it) {
          uint8_t* dst = stage(2 * kBox);
          if (!ok) return;
          const int mb = (ins * L.ncol + (int)rank * (L.ncol / 2)) / 64;
          const int gi = mb / L.rpb, x = (mb % L.rpb) * 64;
          const int64_t row = row_of(km.base, km.sb, km.sbr, b, p.branch0[s] + gi, (jb + j) * kTile);
          tma_load_2d_pair(&tacc, stage_bar(), dst, x, (int)min(row, km.rows - 1));
        }
        return;
      }
      for (int kc = 0; ok && kc < kTile / 64; ++kc)
        for (int ins = 0; ok && ins < L.nins; ++ins, ++it) {
          uint8_t* dst = stage(per * kBox);
          if (!ok) return;
          const uint32_t bar = stage_bar();
          for (int bx = 0; bx < per; ++bx) {
            const int mb = (ins * L.ncol + (int)rank * (L.ncol / 2)) / 64 + bx;
            const int gi = mb / L.rpb, x = (mb % L.rpb) * 64;
            const int64_t row = row_of(km.base, km.sb, km.sbr, b, p.branch0[s] + gi, (jb + j) * kTile + kc * 64);
            tma_load_2d_pair(&tk, bar, dst + bx * kBox, x, (int)min(row, km.rows - 1));
          }
        }
    };
    if (!acc)
      for (int u = 0; ok && u < U; ++u) emit_s(u);  // same order as the score issuer
    else
      for (int u = u_dq; ok && u < U; ++u) emit_dq(u);  // same order as the dQ issuer
    if (rank == 0) {  // drain: none of this producer's loads may be in flight at teardown
      if (!acc) mbar_wait_drain(&in_full, 0);
      for (int i = (it > nst ? it - nst : 0); i < it; ++i) mbar_wait_drain(&fullb[i % nst], (i / nst) & 1u);
    }
  } else if (warp == kDpWarp && lane == 0) {
    // ---------------------------------------------------------------- TMA producer: V and dY for dP
    prefetch_tmap(&tv);
    prefetch_tmap(&tdy);
    int it = 0;
    bool ok = true;
    for (int g = 0; ok && g < dps; ++g) {
      const int y = (int)min((int64_t)b * p.T + (jb + g % nj) * kTile + 64 * (int)rank, rowsBT - 1);
      for (int cb = 0; cb < p.D / (64 * kDpBlocksQ); ++cb, ++it) {  // V rows of 64 keys, then dY rows
        const int st = it % L.nsp;
        if (!mbar_wait(&rp_empty[st], ((it / L.nsp) & 1u) ^ 1u, ab, 13)) { ok = false; break; }
        if (rank == 0) mbar_arrive_expect_tx(&rp_full[st], 2 * kDpStageQ);
        const uint32_t bar = mapa_shared(smem_u32(&rp_full[st]), 0);
        uint8_t* dst = smem + L.off_pring + st * kDpStageQ;
        tma_load_3d_pair(&tv, bar, dst, 0, y, cb * kDpBlocksQ);
        tma_load_3d_pair(&tdy, bar, dst + kDpBlocksQ * kBox, 0, dy_row, cb * kDpBlocksQ);
      }
    }
    if (rank == 0)
      for (int i = (it > L.nsp ? it - L.nsp : 0); i < it; ++i) mbar_wait_drain(&rp_full[i % L.nsp], (i / L.nsp) & 1u);
  } else if (warp == kDpWarp + 1 && lane == 0 && rank == 0) {
    // ---------------------------------------------------------------- dP issuer (leader): dP = dY V^T
    // Its own thread, so the score and dQ products never wait behind the value stream.
    const uint32_t idesc = idesc_f16(128, kTile, kBf16, false, false);
    int it = 0;
    bool ok = true;
    for (int g = 0; ok && g < dps; ++g) {
      const int db = g & 1;
      if (g < 256) trace_at(ft, 4 * g);
      if (g >= 2 && !mbar_wait(&dp_free[db], ((g - 2) >> 1) & 1u, ab, 27)) break;
      if (g < 256) trace_at(ft, 4 * g + 1);
      for (int cb = 0; cb < p.D / (64 * kDpBlocksQ); ++cb, ++it) {  // stage: [V blocks | dY blocks]
        const int st = it % L.nsp;
        if (!mbar_wait(&rp_full[st], (it / L.nsp) & 1u, ab, 28)) { ok = false; break; }
        tc_fence_after();
        const uint32_t sa = smem_u32(smem + L.off_pring + st * kDpStageQ);
        for (int k = 0; k < 4 * kDpBlocksQ; ++k) {
          const uint32_t blk = (uint32_t)(k >> 2) * kBox + (k & 3) * 32;
          const uint64_t ad = sdesc_sw128(sa + kDpBlocksQ * kBox + blk, 16, 1024);
          const uint64_t bd = sdesc_sw128(sa + blk, 16, 1024);
          mma_f16_ss<2>(tmem + L.tmem_p + db * (kTile / 2), ad, bd, idesc, (cb | k) ? 1u : 0u);
        }
        mma_commit_pair(smem_u32(&rp_empty[st]));
      }
      if (!ok) break;
      mma_commit_pair(smem_u32(&dp_full[db]));
      if (g < 256) trace_at(ft, 4 * g + 2);
    }
    mma_commit<2>(smem_u32(&dp_done));  // every dP product has completed before teardown
    mbar_wait_drain(&dp_done, 0);
  } else if ((warp == 1 || warp == kAccIssuer) && lane == 0 && rank == 0) {
    // ---------------------------------------------------------------- MMA issuers (leader): warp 1 the
    // score products S_s = Q_s K_s^T, warp 13 the dQ products; each consumes its own ring, so a score
    // product never waits behind the hand-over of a dS tile
    const int acc = warp == kAccIssuer ? 1 : 0;
    const uint32_t idesc_s = idesc_f16(128, kTile, kBf16, false, false);
    const uint32_t idesc_q = idesc_f16(128, L.ncol, kBf16, false, true);  // B = K rows, MN-major
    auto commit_both = [&](uint64_t* bar) { mma_commit_pair(smem_u32(bar)); };
    const int nst = acc ? L.nsq : L.nst;
    uint64_t* fullb = acc ? q_full : r_full;
    uint64_t* emptyb = acc ? q_empty : r_empty;
    uint8_t* ring = smem + (acc ? L.off_qring : L.off_ring);
    int it = 0;
    auto take = [&](uint32_t* addr) -> bool {
      const int st = it % nst;
      if (!mbar_wait(&fullb[st], (it / nst) & 1u, ab, 23)) return false;
      tc_fence_after();
      *addr = smem_u32(ring + st * kStage);
      return true;
    };
    auto give = [&]() { commit_both(&emptyb[it % nst]); ++it; };
    const uint32_t qa = smem_u32(smem + L.off_a);
    auto issue_s = [&](int u) -> bool {
      const int sb = u & 1, s = unit_s(u);
      if (u < 512) trace_at(ft, 1024 + 8 * u);
      if (u >= 2 && !mbar_wait(&s_free[sb], ((u - 2) >> 1) & 1u, ab, 22)) return false;
      if (u < 512) trace_at(ft, 1025 + 8 * u);
      for (int cc = 0; cc < L.kw / 128; ++cc) {
        uint32_t st;
        if (!take(&st)) return false;
        if (u < 512 && cc == 0) trace_at(ft, 1026 + 8 * u);
        for (int k = 0; k < 8; ++k) {
          const uint64_t ad =
              sdesc_sw128(qa + (s * (L.kw / 64) + cc * 2 + (k >> 2)) * kBox + (k & 3) * 32, 16, 1024);
          const uint64_t bd = sdesc_sw128(st + (k >> 2) * kBox + (k & 3) * 32, 16, 1024);
          mma_f16_ss<2>(tmem + L.tmem_s + sb * (kTile / 2), ad, bd, idesc_s, (cc | k) ? 1u : 0u);
        }
        give();
      }
      commit_both(&s_full[sb]);
      if (u < 512) trace_at(ft, 1027 + 8 * u);
      return true;
    };
    auto issue_dq = [&](int u) -> bool {
      const int v = u - u_dq, s = unit_s(u), j = unit_j(u);
      if (u < 512) trace_at(ft, 1028 + 8 * u);
      if (!mbar_wait(&p_full[v & 1], (v >> 1) & 1u, ab, 24)) return false;
      if (u < 512) trace_at(ft, 1029 + 8 * u);
      tc_fence_after();
      const uint32_t dsa = smem_u32(smem + L.off_t + (v & 1) * (kRows * kTile * 2));
      if (L.acc_merge) {  // stage = 128 keys x 64 columns: both 64-key chunks
        for (int ins = 0; ins < L.nins; ++ins) {
          uint32_t st;
          if (!take(&st)) return false;
          if (u < 512 && ins == 0) trace_at(ft, 1030 + 8 * u);
          for (int k = 0; k < 8; ++k) {
            const int kc = k >> 2, kk = k & 3;
            const uint64_t ad = sdesc_sw128(dsa + kc * kBox + kk * 32, 16, 1024);
            const uint64_t bd = sdesc_sw128(st + kc * kBox + kk * 16 * 128, 64 * 128, 1024);
            mma_f16_ss<2>(tmem + L.tmem_acc + s * (L.kw / 2) + ins * (L.ncol / 2), ad, bd, idesc_q,
                          (j | k) ? 1u : 0u);
          }
          give();
        }
      } else {
        for (int kc = 0; kc < kTile / 64; ++kc)
          for (int ins = 0; ins < L.nins; ++ins) {
            uint32_t st;
            if (!take(&st)) return false;
            for (int kk = 0; kk < 4; ++kk) {
              const uint64_t ad = sdesc_sw128(dsa + kc * kBox + kk * 32, 16, 1024);
              const uint64_t bd = sdesc_sw128(st + kk * 16 * 128, 64 * 128, 1024);
              mma_f16_ss<2>(tmem + L.tmem_acc + s * (L.kw / 2) + ins * (L.ncol / 2), ad, bd, idesc_q,
                            (j | kc | kk) ? 1u : 0u);
            }
            give();
          }
      }
      commit_both(&ds_empty[v & 1]);
      if (u < 512) trace_at(ft, 1031 + 8 * u);
      return true;
    };
    if (!acc) {
      bool ok = mbar_wait(&in_full, 0, ab, 21);
      tc_fence_after();
      for (int u = 0; ok && u < U; ++u) ok = issue_s(u);
      mma_commit<2>(smem_u32(&s_done));  // every score product has completed before teardown
      mbar_wait_drain(&s_done, 0);
    } else {
      bool ok = true;
      for (int u = u_dq; ok && u < U; ++u) ok = issue_dq(u);
      commit_both(&o_full);
      mbar_wait_drain(&o_full, 0);
    }
  } else if ((warp >= 2 && warp < 6) || (warp >= kSoftmax2 && warp < kSoftmax2 + 4)) {
    // ---------------------------------------------------------------- softmax + epilogue: two warpgroups
    // taking alternate units (warps 2-5 the even ones, 8-11 the odd ones), each thread all 64 key columns
    // of its row half in two 32-column chunks, so that one unit's hand-off chain (dS stores, barrier,
    // hand-over to the dQ issuer, the wait for a free dS tile) overlaps the other warpgroup's arithmetic
    const int wg = warp >= kSoftmax2 ? 1 : 0;
    const int quad = warp & 3;
    const int l = quad * 32 + lane;
    const int r = l & 63, half = l >> 6;
    const int t = t0 + 64 * (int)rank + r;
    const bool live = t < p.T;
    const uint32_t lane_base = (uint32_t)(quad * 32) << 16;
    const uint32_t pf_leader = mapa_shared(smem_u32(&p_full[0]), 0);
    const uint32_t df_leader = mapa_shared(smem_u32(&dp_free[0]), 0);
    const uint32_t sf_leader = mapa_shared(smem_u32(&s_free[0]), 0);
    const bool arriver = (warp == 2 || warp == kSoftmax2) && lane == 0;  // one per warpgroup
    float* red = reinterpret_cast<float*>(smem + L.off_red);
    const float kLog2e = 1.4426950408889634f;
    // with a given delta, d gamma is corrected to this kernel's own exact row sum of P dP -- a product of
    // whole-row sums, so a key share (ksplit > 1, whose delta comes from the split's own exact delta sweep)
    // keeps the given delta instead
    const bool exact_corr = p.delta_given && p.ksplit == 1;
    const float gsc = rsqrtf((float)p.group);
    float scale2[kMaxMaps], lse2[kMaxMaps], delta[kMaxMaps], alpha[kMaxMaps];
    // per map: sum of dS * S (d gamma), and with a given delta also sum P * S and sum P * dP (the exact
    // row delta), which correct d gamma from the given delta to this kernel's own P and dP
    float sA[kMaxMaps], sB[kMaxMaps], sC[kMaxMaps];
#pragma unroll
    for (int s = 0; s < kMaxMaps; ++s) {
      scale2[s] = lse2[s] = delta[s] = sA[s] = sB[s] = sC[s] = 0.f;
      alpha[s] = 1.f;
      if (s < maps) {
        scale2[s] = p.scales[s] * gsc * kLog2e;
        alpha[s] = p.weights ? p.weights[s] : 1.f;
        if (live) {
          lse2[s] = p.lse[((int64_t)b * maps + s) * p.T + t] * kLog2e;
          if (p.delta_given) delta[s] = p.delta[((int64_t)b * maps + s) * p.T + t];
        }
      }
    }
    bool ok = true;
    // Whole-row delta_s at the end of the first sweep (two halves x two warpgroups), stored for the
    // key-parallel kernels.  Both warpgroups come here once, after their last first-sweep unit; the
    // buffer is the dS tiles' space, which no first-sweep unit writes.
    auto sweep_end = [&]() {
      for (int m = 0; m < maps; ++m) red[(m * 2 + wg) * 128 + l] = delta[m];
      named_bar_sync(1, 256);
      for (int m = 0; m < maps; ++m)
        delta[m] = red[(m * 2) * 128 + l] + red[(m * 2) * 128 + (l ^ 64)] + red[(m * 2 + 1) * 128 + l] +
                   red[(m * 2 + 1) * 128 + (l ^ 64)];
      named_bar_sync(1, 256);
      for (int m = 0; m < maps; ++m) {
        if (ok && live && half == 0 && wg == 0) {  // the row's delta, or this key share's part of it
          const int64_t i = ((int64_t)b * maps + m) * p.T + t;
          if (p.ksplit > 1) p.delta_part[(int64_t)khalf * p.B * maps * p.T + i] = delta[m];
          else p.delta[i] = delta[m];
        }
        if (p.dweight && wg == 0) {
          float w = (ok && live && half == 0) ? delta[m] : 0.f;
          for (int o = 16; o; o >>= 1) w += __shfl_xor_sync(0xffffffffu, w, o);
          if (p.scalar_part) {
            if (lane == 0) p.scalar_part[((size_t)blockIdx.x * 4 + quad) * maps + m] = w;
          } else if (lane == 0 && w != 0.f) {
            atomicAdd(p.dweight + m, w);
          }
        }
      }
    };
    bool reduced = p.delta_given != 0;
    // Warpgroup wg takes units wg, wg + 2, ...: score buffer u & 1 and dS tile v & 1 are its own, so it
    // waits for their phases in order; the dP tile of a key tile is read by both warpgroups.
    for (int u = wg; u < U; u += 2) {
      if (!reduced && u >= per_sweep) {
        sweep_end();
        reduced = true;
      }
      const int sb = u & 1, s = unit_s(u), j = unit_j(u), g = unit_g(u);
      const bool form_ds = u >= u_dq;
      const int v = u - u_dq;
      if (arriver && u < 512) trace_at(ft, 5120 + 4 * u);
      if (ok) ok = mbar_wait(&s_full[sb], (u >> 1) & 1u, ab, 32);
      // the first unit of key tile g this warpgroup takes (maps s = 0 and 1, or the tile's only unit)
      if (ok && s < 2) ok = mbar_wait(&dp_full[g & 1], (g >> 1) & 1u, ab, 35);
      if (arriver && u < 512) trace_at(ft, 5121 + 4 * u);
      ok = __all_sync(0xffffffffu, ok);
      const bool entered = ok;  // the unit's TMEM reads (and s_free arrival) happen only then
      if (ok) {
        tc_fence_after();
        const uint32_t dsa = smem_u32(smem + L.off_t + (v & 1) * (kRows * kTile * 2));
        // this map's row constants in registers (the per-map arrays live in local memory)
        const float sc2 = scale2[s], ls2 = lse2[s], dl = delta[s], al = alpha[s];
        float dsum = 0.f, a_acc = 0.f, b_acc = 0.f, c_acc = 0.f;
        const int kb = (jb + j) * kTile + half * 64;  // first key column of this thread's 64
        int lim_row = p.T - kb;
        if (p.causal) lim_row = min(lim_row, t - kb + 1);
        if (!live) lim_row = 0;
        bool free_tile = true;
#pragma unroll 1
        for (int ch = 0; ch < 2; ++ch) {
          float sv[32], pv[32];
          tmem_ld32(tmem + lane_base + L.tmem_s + sb * (kTile / 2) + ch * 32, sv);
          tmem_ld32(tmem + lane_base + L.tmem_p + (g & 1) * (kTile / 2) + ch * 32, pv);
          tmem_wait_ld();
          if (ch == 1) {  // the score buffer is free for the unit after next while this warp computes
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
              mbar_arrive_cluster_relaxed(sf_leader + sb * 8);
              // this warpgroup's last unit of key tile g: this warp is done with the dP buffer
              if (s + 2 >= maps) mbar_arrive_cluster_relaxed(df_leader + (g & 1) * 8);
            }
          }
          const int lim = lim_row - ch * 32;
          uint32_t packed[16];
          // masked columns get probability 0 (a select, so any value the exponential takes there is
          // discarded; tiles below the diagonal skip the selects); two partial sums shorten the chains
          if (form_ds) {
            // dS = alpha P (dP - delta) = P (alpha dP - alpha delta); d gamma accumulates dS * S
            const float ald = al * dl;
            float a0 = 0.f, a1 = 0.f, b0 = 0.f, b1 = 0.f, c0 = 0.f, c1 = 0.f;
            auto body = [&](auto masked, auto exact) {
#pragma unroll
              for (int i = 0; i < 32; i += 2) {
                float p0 = ex2(fmaf(sv[i], sc2, -ls2)), p1 = ex2(fmaf(sv[i + 1], sc2, -ls2));
                if (masked) {
                  p0 = i < lim ? p0 : 0.f;
                  p1 = i + 1 < lim ? p1 : 0.f;
                }
                const float d0 = p0 * fmaf(al, pv[i], -ald), d1 = p1 * fmaf(al, pv[i + 1], -ald);
                a0 = fmaf(d0, sv[i], a0);
                a1 = fmaf(d1, sv[i + 1], a1);
                if (exact) {
                  b0 = fmaf(p0, sv[i], b0);
                  b1 = fmaf(p1, sv[i + 1], b1);
                  c0 = fmaf(p0, pv[i], c0);
                  c1 = fmaf(p1, pv[i + 1], c1);
                }
                packed[i / 2] = pack2<T>(d0, d1);
              }
            };
            if (exact_corr) {
              if (lim >= 32) body(std::false_type{}, std::true_type{});
              else body(std::true_type{}, std::true_type{});
            } else {
              if (lim >= 32) body(std::false_type{}, std::false_type{});
              else body(std::true_type{}, std::false_type{});
            }
            a_acc += a0 + a1;
            b_acc += b0 + b1;
            c_acc += c0 + c1;
            if (ch == 0) {
              // the dS tile of this warpgroup's previous unit must have been read by its dQ product:
              // waited for only now, so the arithmetic above overlaps that product
              free_tile = v < 2 || mbar_wait(&ds_empty[v & 1], ((v - 2) >> 1) & 1u, ab, 33);
              free_tile = __all_sync(0xffffffffu, free_tile);
            }
            if (free_tile) {
#pragma unroll
              for (int e = 0; e < 4; ++e)
                st_shared_v4(dsa + half * kBox + sw128_offset(r, ch * 4 + e), packed[4 * e], packed[4 * e + 1],
                             packed[4 * e + 2], packed[4 * e + 3]);
            }
          } else {
            float d0 = 0.f, d1 = 0.f;
            if (lim >= 32) {
#pragma unroll
              for (int i = 0; i < 32; i += 2) {
                d0 = fmaf(ex2(fmaf(sv[i], sc2, -ls2)), pv[i], d0);
                d1 = fmaf(ex2(fmaf(sv[i + 1], sc2, -ls2)), pv[i + 1], d1);
              }
            } else {
#pragma unroll
              for (int i = 0; i < 32; i += 2) {
                const float e0 = ex2(fmaf(sv[i], sc2, -ls2)), e1 = ex2(fmaf(sv[i + 1], sc2, -ls2));
                d0 = fmaf(i < lim ? e0 : 0.f, pv[i], d0);
                d1 = fmaf(i + 1 < lim ? e1 : 0.f, pv[i + 1], d1);
              }
            }
            dsum += d0 + d1;
          }
        }
        if (!free_tile) ok = false;
        if (form_ds) {
          sA[s] += a_acc;
          sB[s] += b_acc;
          sC[s] += c_acc;
          fence_proxy_async();
        } else {
          delta[s] += dsum;
        }
      }
      if (arriver && u < 512) trace_at(ft, 5122 + 4 * u);
      if (!entered && lane == 0) {  // aborted unit: counts stay whole
        mbar_arrive_cluster_relaxed(sf_leader + sb * 8);
        if (s + 2 >= maps) mbar_arrive_cluster_relaxed(df_leader + (g & 1) * 8);
      }
      if (form_ds) {
        // dS tile v handed to the dQ issuer once all four warps stored their rows (phase v / 2 of barrier
        // v % 2, which the issuer waits for in order; this warpgroup cannot run two phases ahead, as its
        // next unit on that tile first waits for the product of unit v).  First-sweep units hand nothing
        // over, so the warps of a warpgroup pass them without a barrier.
        tc_fence_before();
        named_bar_sync(3 + wg, 128);
        if (arriver) {
          if (u < 512) trace_at(ft, 5123 + 4 * u);
          mbar_arrive_remote(pf_leader + (v & 1) * 8);
        }
      }
    }
    if (!reduced) sweep_end();
    // ---- d gamma_s from each row's own sums (both warpgroups, both halves), then the dQ epilogue.  The
    // reduction buffer shares the dS tiles' space: every product (the last dQ ones read those tiles) has
    // completed first.
    if (ok) ok = mbar_wait(&o_full, 0, ab, 34);
    ok = __all_sync(0xffffffffu, ok);
    tc_fence_after();
    if (p.dscale) {
      if (wg == 1)
        for (int m = 0; m < maps; ++m) {
          red[(3 * m) * 128 + l] = sA[m];
          red[(3 * m + 1) * 128 + l] = sB[m];
          red[(3 * m + 2) * 128 + l] = sC[m];
        }
      named_bar_sync(1, 256);
      if (wg == 0)
        for (int m = 0; m < maps; ++m) {
          sA[m] += red[(3 * m) * 128 + l];
          sB[m] += red[(3 * m + 1) * 128 + l];
          sC[m] += red[(3 * m + 2) * 128 + l];
        }
      named_bar_sync(1, 256);
    }
    if (p.dscale && wg == 0) {
      for (int m = 0; m < maps; ++m) {
        red[(3 * m) * 128 + l] = sA[m];
        red[(3 * m + 1) * 128 + l] = sB[m];
        red[(3 * m + 2) * 128 + l] = sC[m];
      }
      named_bar_sync(2, 128);
      for (int m = 0; m < maps; ++m) {
        float dg = 0.f;
        if (half == 0 && live && ok) {
          const float A = sA[m] + red[(3 * m) * 128 + (l ^ 64)];
          const float Bs = sB[m] + red[(3 * m + 1) * 128 + (l ^ 64)];
          const float C = sC[m] + red[(3 * m + 2) * 128 + (l ^ 64)];
          // sum dS S = alpha (sum P dP S - delta sum P S); with a given delta, delta -> the exact sum P dP
          dg = exact_corr ? A + alpha[m] * (delta[m] - C) * Bs : A;
        }
        for (int o = 16; o; o >>= 1) dg += __shfl_xor_sync(0xffffffffu, dg, o);
        if (p.scalar_part) {
          if (lane == 0) p.scalar_part[(((size_t)gridDim.x + blockIdx.x) * 4 + quad) * maps + m] = dg * gsc;
        } else if (lane == 0 && dg != 0.f) {
          atomicAdd(p.dscale + m, dg * gsc);
        }
      }
    }
    if (wg == 0 && ok && p.dq) {
      for (int m = 0; m < maps; ++m) {
        const float gamma = p.scales[m] * gsc;
        for (int ins = 0; ins < L.nins; ++ins)
          for (int c = 0; c < L.ncol / 2; c += 32) {
            float vv[32];
            if (nj > 0) {  // (an empty key share has no accumulator: its partial is zero)
              tmem_ld32(tmem + lane_base + L.tmem_acc + m * (L.kw / 2) + ins * (L.ncol / 2) + c, vv);
              tmem_wait_ld();
            }
            if (live) {
              const int col = ins * L.ncol + half * (L.ncol / 2) + c;  // map-local column, one branch
              const int gi = col / p.R;
              const int64_t row = row_of(qm.base, qm.sb, qm.sbr, b, p.branch0[m] + gi, t);
              if (p.ksplit > 1) {  // compact partial row (b, map, branch, query)
                const int64_t crow = (((int64_t)b * maps + m) * p.group + gi) * p.T + t;
                store_part32(p.part, ((int64_t)khalf * p.part_rows + crow) * p.R + (col % p.R), vv, gamma, nj == 0);
              } else {
                store_grad32<T>(p.dq, row * p.R + (col % p.R), vv, gamma, p.overwrite != 0);
              }
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

// =============================================================================== dK / dV kernels
// kDK: dK_s += dS_s^T Q_s (per map); else dV += (sum_s alpha_s P_s)^T dY (once per query tile).
template <typename T, bool kDK>
__global__ void __launch_bounds__(kThreads, 1) dkv_mixed_kernel(const __grid_constant__ CUtensorMap tq,
                                                                const __grid_constant__ CUtensorMap tk,
                                                                const __grid_constant__ CUtensorMap tv,
                                                                const __grid_constant__ CUtensorMap tdy,
                                                                const __grid_constant__ CUtensorMap tacc,
                                                                const Params p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ uint64_t in_full, o_full, s_done, r_full[kMaxStages], r_empty[kMaxStages];
  __shared__ uint64_t q_full[kMaxStages], q_empty[kMaxStages];
  __shared__ uint64_t rp_full[kMaxStages], rp_empty[kMaxStages], dp_done;
  constexpr int kNSB = kDK ? 2 : 4;  // score buffers (Layout::nsb)
  __shared__ uint64_t s_full[kNSB], s_free[kNSB], p_full[2], dp_full[2], dp_free[2], t_empty[2];
  __shared__ uint32_t tmem_base;
  __shared__ int abort_flag;

  constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
  const Layout L = make_layout(kDK ? 1 : 2, p.maps, p.group, p.R, p.D);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const uint32_t rank = cluster_ctarank() & 1u;
  const int tiles = (p.T + kTile - 1) / kTile;
  const int khalf = (blockIdx.x / 2) % p.ksplit;  // this pair's share of its query tiles
  const int pair = blockIdx.x / (2 * p.ksplit);
  // longest pairs first across every sequence (early keys have the most queries)
  const int b = pair % p.B;
  const int k0 = (pair / p.B) * kTile;        // first key of this pair
  const int i00 = p.causal ? k0 / kTile : 0;  // first query tile of the pair
  const int ispan = (tiles - i00 + p.ksplit - 1) / p.ksplit;
  const int i0 = i00 + khalf * ispan;                  // first query tile of this share
  const int ni = max(0, min(tiles, i0 + ispan) - i0);  // (the last share may be empty)
  const int maps = p.maps;
  const int U = ni * maps;
  const int dn = p.D < 256 ? p.D : 256;      // N of one dV instruction
  const int dins = p.D / dn;
  const MapRows qm{p.q_rows, p.q_base, p.q_sb, p.q_sbr}, km{p.k_rows, p.k_base, p.k_sb, p.k_sbr};
  const int64_t rowsBT = (int64_t)p.B * p.T;
  Abort ab{&abort_flag, p.status};

  if (threadIdx.x == 0) {
    abort_flag = 0;
    mbar_init(&in_full, 1);
    mbar_init(&o_full, 1);
    mbar_init(&s_done, 1);
    for (int i = 0; i < kMaxStages; ++i) {
      mbar_init(&r_full[i], 1);
      mbar_init(&r_empty[i], 1);
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 1);
      mbar_init(&rp_full[i], 1);
      mbar_init(&rp_empty[i], 1);
    }
    mbar_init(&dp_done, 1);
    for (int i = 0; i < kNSB; ++i) {
      mbar_init(&s_full[i], 1);
      // score tile read out of TMEM: each warp of the owning warpgroup (dK) or of both (dV), both CTAs
      mbar_init(&s_free[i], kDK ? 8 : 16);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&p_full[i], 2);
      mbar_init(&dp_full[i], 1);
      // dP^T tile released by each softmax warp that read it, in both CTAs (one map: a query tile is one
      // unit, read by one warpgroup)
      mbar_init(&dp_free[i], maps == 1 ? 8 : 16);
      mbar_init(&t_empty[i], 1);
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

  auto unit_g = [&](int u) { return u / maps; };  // query tile (0 .. ni-1)
  auto unit_s = [&](int u) { return u % maps; };

  const int krow = k0 + 64 * (int)rank;
  const int vy = (int)min((int64_t)b * p.T + krow, rowsBT - 1);
  if ((warp == 0 || warp == kAccProducer) && lane == 0) {
    // ---------------------------------------------------------------- TMA producers: warp 0 loads the
    // resident K rows, then the score operands (Q rows of this CTA's 64 queries, per map) into the score
    // ring; warp 12 loads the operands of the accumulating product (dK: Q rows of all 128 queries,
    // MN-major; dV: dY rows) into the accumulation ring
    const int acc = warp == kAccProducer ? 1 : 0;
    prefetch_tmap(&tq);
    prefetch_tmap(&tdy);
    prefetch_tmap(&tacc);
    if (!acc) {
      prefetch_tmap(&tk);
      const uint32_t inf = mapa_shared(smem_u32(&in_full), 0);
      if (rank == 0) mbar_arrive_expect_tx(&in_full, 2 * (kRows * L.W * 2));
      for (int s = 0; s < maps; ++s)
        for (int cc = 0; cc < L.kw / 128; ++cc)
          load_map_chunk(&tk, km, p, inf, smem + L.off_a + (s * (L.kw / 64) + cc * 2) * kBox, b, s, cc, 2, krow);
    }
    const int nst = acc ? L.nsq : L.nst;
    uint64_t* fullb = acc ? q_full : r_full;
    uint64_t* emptyb = acc ? q_empty : r_empty;
    uint8_t* ring = smem + (acc ? L.off_qring : L.off_ring);
    int it = 0;
    bool ok = true;
    auto stage = [&](int bytes) -> uint8_t* {
      const int st = it % nst;
      if (!mbar_wait(&emptyb[st], ((it / nst) & 1u) ^ 1u, ab, 11 + acc)) { ok = false; return nullptr; }
      if (rank == 0) mbar_arrive_expect_tx(&fullb[st], 2 * bytes);
      return ring + st * kStage;
    };
    auto stage_bar = [&]() { return mapa_shared(smem_u32(&fullb[it % nst]), 0); };
    auto emit_s = [&](int u) {  // query rows of map s for this CTA's 64 queries
      const int q = (i0 + unit_g(u)) * kTile + 64 * (int)rank;
      for (int cc = 0; ok && cc < L.kw / 128; ++cc, ++it) {
        uint8_t* dst = stage(2 * kBox);
        if (!ok) return;
        load_map_chunk(&tq, qm, p, stage_bar(), dst, b, unit_s(u), cc, 2, q);
      }
    };
    auto emit_acc = [&](int u) {  // MN-major operand of the accumulating product, all 128 queries
      const int i = i0 + unit_g(u), s = unit_s(u);
      if (kDK && L.acc_merge) {  // one stage per N block: a 128-query x 64-column box
        for (int ins = 0; ok && ins < L.nins; ++ins, ++it) {
            uint8_t* dst = stage(2 * kBox);
          if (!ok) return;
          const int mb = (ins * L.ncol + (int)rank * (L.ncol / 2)) / 64;
          const int gi = mb / L.rpb, x = (mb % L.rpb) * 64;
          const int64_t row = row_of(qm.base, qm.sb, qm.sbr, b, p.branch0[s] + gi, i * kTile);
          tma_load_2d_pair(&tacc, stage_bar(), dst, x, (int)min(row, qm.rows - 1));
        }
      } else if (kDK) {
        const int per = (L.ncol / 2) / 64;
        for (int qc = 0; ok && qc < kTile / 64; ++qc)
          for (int ins = 0; ok && ins < L.nins; ++ins, ++it) {
                uint8_t* dst = stage(per * kBox);
            if (!ok) return;
            const uint32_t bar = stage_bar();
            for (int bx = 0; bx < per; ++bx) {
              const int mb = (ins * L.ncol + (int)rank * (L.ncol / 2)) / 64 + bx;
              const int gi = mb / L.rpb, x = (mb % L.rpb) * 64;
              const int64_t row = row_of(qm.base, qm.sb, qm.sbr, b, p.branch0[s] + gi, i * kTile + qc * 64);
              tma_load_2d_pair(&tq, bar, dst + bx * kBox, x, (int)min(row, qm.rows - 1));
            }
          }
      } else {
        const int dper = (dn / 2) / 64;
        for (int qc = 0; ok && qc < kTile / 64; ++qc) {
          const int y = (int)min((int64_t)b * p.T + i * kTile + qc * 64, rowsBT - 1);
          for (int ins = 0; ok && ins < dins; ++ins, ++it) {
                uint8_t* dst = stage(dper * kBox);  // dper = 2 (dn = 256): one box of two column blocks
            if (!ok) return;
            tma_load_3d_pair(&tdy, stage_bar(), dst, 0, y, (ins * dn + (int)rank * (dn / 2)) / 64);
          }
        }
      }
    };
    // same orders as the two issuers below
    if (!acc)
      for (int u = 0; ok && u < U; ++u) emit_s(u);
    else
      for (int u = 0; ok && u < U; ++u)
        if (kDK || unit_s(u) == maps - 1) emit_acc(u);
    if (rank == 0) {  // drain: none of this producer's loads may be in flight at teardown
      if (!acc) mbar_wait_drain(&in_full, 0);
      for (int i = (it > nst ? it - nst : 0); i < it; ++i) mbar_wait_drain(&fullb[i % nst], (i / nst) & 1u);
    }
  } else if (kDK && warp == kDpWarp && lane == 0) {
    // ---------------------------------------------------------------- TMA producer: dY and V for dP^T
    prefetch_tmap(&tv);
    prefetch_tmap(&tdy);
    int it = 0;
    bool ok = true;
    for (int g = 0; ok && g < ni; ++g) {
      const int y = (int)min((int64_t)b * p.T + (i0 + g) * kTile + 64 * (int)rank, rowsBT - 1);
      for (int cb = 0; cb < p.D / (64 * kDpBlocks); ++cb, ++it) {  // dY rows of 64 queries, then V rows
        const int st = it % L.nsp;
        if (!mbar_wait(&rp_empty[st], ((it / L.nsp) & 1u) ^ 1u, ab, 13)) { ok = false; break; }
        if (rank == 0) mbar_arrive_expect_tx(&rp_full[st], 2 * kDpStage);
        const uint32_t bar = mapa_shared(smem_u32(&rp_full[st]), 0);
        uint8_t* dst = smem + L.off_pring + st * kDpStage;
        tma_load_3d_pair(&tdy, bar, dst, 0, y, cb * kDpBlocks);
        tma_load_3d_pair(&tv, bar, dst + kDpBlocks * kBox, 0, vy, cb * kDpBlocks);
      }
    }
    if (rank == 0)
      for (int i = (it > L.nsp ? it - L.nsp : 0); i < it; ++i) mbar_wait_drain(&rp_full[i % L.nsp], (i / L.nsp) & 1u);
  } else if (kDK && warp == kDpWarp + 1 && lane == 0 && rank == 0) {
    // ---------------------------------------------------------------- dP^T issuer (leader): dP^T = V dY^T
    const uint32_t idesc = idesc_f16(128, kTile, kBf16, false, false);
    int it = 0;
    bool ok = true;
    for (int g = 0; ok && g < ni; ++g) {
      const int db = g & 1;
      if (g >= 2 && !mbar_wait(&dp_free[db], ((g - 2) >> 1) & 1u, ab, 27)) break;
      for (int cb = 0; cb < p.D / (64 * kDpBlocks); ++cb, ++it) {  // stage: [dY blocks | V blocks]
        const int st = it % L.nsp;
        if (!mbar_wait(&rp_full[st], (it / L.nsp) & 1u, ab, 28)) { ok = false; break; }
        tc_fence_after();
        const uint32_t sa = smem_u32(smem + L.off_pring + st * kDpStage);
        for (int k = 0; k < 4 * kDpBlocks; ++k) {
          const uint32_t blk = (uint32_t)(k >> 2) * kBox + (k & 3) * 32;
          const uint64_t ad = sdesc_sw128(sa + kDpBlocks * kBox + blk, 16, 1024);
          const uint64_t bd = sdesc_sw128(sa + blk, 16, 1024);
          mma_f16_ss<2>(tmem + L.tmem_p + db * (kTile / 2), ad, bd, idesc, (cb | k) ? 1u : 0u);
        }
        mma_commit_pair(smem_u32(&rp_empty[st]));
      }
      if (!ok) break;
      mma_commit_pair(smem_u32(&dp_full[db]));
    }
    mma_commit<2>(smem_u32(&dp_done));  // every dP^T product has completed before teardown
    mbar_wait_drain(&dp_done, 0);
  } else if ((warp == 1 || warp == kAccIssuer) && lane == 0 && rank == 0) {
    // ---------------------------------------------------------------- MMA issuers (leader): warp 1 the
    // score products S_s^T = K_s Q_s^T, warp 13 the dK (or dV) products, each on its own ring
    const int acc = warp == kAccIssuer ? 1 : 0;
    const uint32_t idesc_s = idesc_f16(128, kTile, kBf16, false, false);
    const uint32_t idesc_acc = kDK ? idesc_f16(128, L.ncol, kBf16, false, true)   // B = Q rows, MN-major
                                   : idesc_f16(128, dn, kBf16, false, true);      // B = dY rows, MN-major
    auto commit_both = [&](uint64_t* bar) { mma_commit_pair(smem_u32(bar)); };
    const int nst = acc ? L.nsq : L.nst;
    uint64_t* fullb = acc ? q_full : r_full;
    uint64_t* emptyb = acc ? q_empty : r_empty;
    uint8_t* ring = smem + (acc ? L.off_qring : L.off_ring);
    int it = 0;
    auto take = [&](uint32_t* addr) -> bool {
      const int st = it % nst;
      if (!mbar_wait(&fullb[st], (it / nst) & 1u, ab, 23)) return false;
      tc_fence_after();
      *addr = smem_u32(ring + st * kStage);
      return true;
    };
    auto give = [&]() { commit_both(&emptyb[it % nst]); ++it; };
    const uint32_t ka = smem_u32(smem + L.off_a);
    auto issue_s = [&](int u) -> bool {  // S^T = K_s Q_s^T
      const int sb = u % kNSB, s = unit_s(u);
      if (u >= kNSB && !mbar_wait(&s_free[sb], ((u / kNSB) - 1) & 1u, ab, 22)) return false;
      for (int cc = 0; cc < L.kw / 128; ++cc) {
        uint32_t st;
        if (!take(&st)) return false;
        for (int k = 0; k < 8; ++k) {
          const uint64_t ad =
              sdesc_sw128(ka + (s * (L.kw / 64) + cc * 2 + (k >> 2)) * kBox + (k & 3) * 32, 16, 1024);
          const uint64_t bd = sdesc_sw128(st + (k >> 2) * kBox + (k & 3) * 32, 16, 1024);
          mma_f16_ss<2>(tmem + L.tmem_s + sb * (kTile / 2), ad, bd, idesc_s, (cc | k) ? 1u : 0u);
        }
        give();
      }
      commit_both(&s_full[sb]);
      return true;
    };
    // dK: after every unit (dS_s^T in tile buffer u&1); dV: after the last map of a query tile
    // (mixed P^T in tile buffer g&1).
    auto issue_acc = [&](int u) -> bool {
      const int g = unit_g(u), s = unit_s(u);
      const int tb = kDK ? (u & 1) : (g & 1);
      // dK: one dS tile per unit; dV: one mixed-probability tile per query tile
      if (kDK ? !mbar_wait(&p_full[u & 1], (u >> 1) & 1u, ab, 24) : !mbar_wait(&p_full[g & 1], (g >> 1) & 1u, ab, 24))
        return false;
      tc_fence_after();
      const uint32_t ta = smem_u32(smem + L.off_t + tb * (kRows * kTile * 2));
      const int nins = kDK ? L.nins : dins;
      const int ncol = kDK ? L.ncol : dn;
      if (kDK && L.acc_merge) {  // stage = 128 queries x 64 columns: both 64-query chunks
        for (int ins = 0; ins < nins; ++ins) {
          uint32_t st;
          if (!take(&st)) return false;
          for (int k = 0; k < 8; ++k) {
            const int qc = k >> 2, kk = k & 3;
            const uint64_t ad = sdesc_sw128(ta + qc * kBox + kk * 32, 16, 1024);
            const uint64_t bd = sdesc_sw128(st + qc * kBox + kk * 16 * 128, 64 * 128, 1024);
            const uint32_t d = tmem + L.tmem_acc + s * (L.kw / 2) + ins * (ncol / 2);
            mma_f16_ss<2>(d, ad, bd, idesc_acc, (g | k) ? 1u : 0u);
          }
          give();
        }
        commit_both(&t_empty[tb]);
        return true;
      }
      for (int qc = 0; qc < kTile / 64; ++qc)
        for (int ins = 0; ins < nins; ++ins) {
          uint32_t st;
          if (!take(&st)) return false;
          for (int kk = 0; kk < 4; ++kk) {
            const uint64_t ad = sdesc_sw128(ta + qc * kBox + kk * 32, 16, 1024);
            const uint64_t bd = sdesc_sw128(st + kk * 16 * 128, 64 * 128, 1024);
            const uint32_t d = tmem + L.tmem_acc + (kDK ? s * (L.kw / 2) : 0) + ins * (ncol / 2);
            mma_f16_ss<2>(d, ad, bd, idesc_acc, (g | qc | kk) ? 1u : 0u);
          }
          give();
        }
      commit_both(&t_empty[tb]);
      return true;
    };
    if (!acc) {
      bool ok = mbar_wait(&in_full, 0, ab, 21);
      tc_fence_after();
      for (int u = 0; ok && u < U; ++u) ok = issue_s(u);
      mma_commit<2>(smem_u32(&s_done));  // every score product has completed before teardown
      mbar_wait_drain(&s_done, 0);
    } else {
      bool ok = true;
      for (int u = 0; ok && u < U; ++u)
        if (kDK || unit_s(u) == maps - 1) ok = issue_acc(u);
      commit_both(&o_full);
      mbar_wait_drain(&o_full, 0);
    }
  } else if ((warp >= 2 && warp < 6) || (warp >= kSoftmax2 && warp < kSoftmax2 + 4)) {
    // ---------------------------------------------------------------- softmax + epilogue: two warpgroups
    // (warps 2-5 and 8-11); dK: alternate units, dV: warps 2-5 the first 32 of each thread's 64 query
    // columns and warps 8-11 the other 32
    const int wg = warp >= kSoftmax2 ? 1 : 0;
    const int quad = warp & 3;
    const int l = quad * 32 + lane;
    const int r = l & 63, half = l >> 6;
    const int key = k0 + 64 * (int)rank + r;
    const bool live = key < p.T;
    const uint32_t lane_base = (uint32_t)(quad * 32) << 16;
    const uint32_t pf_leader = mapa_shared(smem_u32(&p_full[0]), 0);
    const uint32_t df_leader = mapa_shared(smem_u32(&dp_free[0]), 0);
    const uint32_t sf_leader = mapa_shared(smem_u32(&s_free[0]), 0);
    const bool arriver = lane == 0 && (warp == 2 || (kDK && warp == kSoftmax2));  // dK: one per warpgroup
    // [warpgroup (dK)][tile parity][2][maps][128]: lse2, alpha * delta
    float* red = reinterpret_cast<float*>(smem + L.off_red);
    const float kLog2e = 1.4426950408889634f;
    const float gsc = rsqrtf((float)p.group);
    float scale2[kMaxMaps], alpha[kMaxMaps];
#pragma unroll
    for (int s = 0; s < kMaxMaps; ++s) {
      scale2[s] = s < maps ? p.scales[s] * gsc * kLog2e : 0.f;
      alpha[s] = (s < maps && p.weights) ? p.weights[s] : 1.f;
    }
    float pm[kDK ? 1 : 32];
    bool ok = true;
    // dK: warpgroup wg takes units wg, wg + 2, ... (score buffer u & 1 and dS^T tile u & 1 are its own, so
    // it waits for their phases in order), each thread all 64 query columns of its row half in two
    // 32-column chunks, with its own copy of the staged row constants; the dP^T tile of a query tile is
    // read by both warpgroups.  dV: both warpgroups take every unit, 32 of a thread's 64 columns each
    // (the mixed probabilities of a query tile sum over all its maps).
    constexpr bool kPing = kDK;
    constexpr int kChunks = kPing ? 2 : 1;
    for (int u = kPing ? wg : 0; u < U; u += kPing ? 2 : 1) {
      const int sb = u % kNSB, s = unit_s(u), g = unit_g(u);
      const int qt = (i0 + g) * kTile;
      float* rt = red + (kPing ? wg * (4 * kMaxMaps * 128) : 0) + (g & 1) * (2 * kMaxMaps * 128);
      const bool first = kPing ? s < 2 : s == 0;  // this warpgroup's first unit of query tile g
      if (first && (kPing || wg == 0)) {  // stage this query tile's log-sum-exp (and delta) of every map
        for (int m = 0; m < maps; ++m) {
          const int q = qt + l;
          const bool qv = q < p.T;
          rt[m * 128 + l] = qv ? p.lse[((int64_t)b * maps + m) * p.T + q] * kLog2e : 0.f;
          if (kDK) rt[(kMaxMaps + m) * 128 + l] = qv ? alpha[m] * p.delta[((int64_t)b * maps + m) * p.T + q] : 0.f;
        }
      }
      if (ok) ok = mbar_wait(&s_full[sb], (u / kNSB) & 1u, ab, 32);
      if (ok && kDK && first) ok = mbar_wait(&dp_full[g & 1], (g >> 1) & 1u, ab, 35);
      if (first) named_bar_sync(kPing ? 3 + wg : 1, kPing ? 128 : 256);  // staged lse / delta visible
      ok = __all_sync(0xffffffffu, ok);
      const bool entered = ok;  // the unit's TMEM reads (and s_free arrival) happen only then
      if (ok) {
        tc_fence_after();
        const uint32_t ta = smem_u32(smem + L.off_t + (kDK ? (u & 1) : (g & 1)) * (kRows * kTile * 2));
        const float sc2 = scale2[s], al = alpha[s];
        const float* lse_row = rt + s * 128;
        const float* delta_row = rt + (kMaxMaps + s) * 128;
        bool free_tile = true;
#pragma unroll 1
        for (int c = 0; c < kChunks; ++c) {
          const int ch = kPing ? c : wg;
          float sv[32], dpv[32];
          tmem_ld32(tmem + lane_base + L.tmem_s + sb * (kTile / 2) + ch * 32, sv);
          if (kDK) tmem_ld32(tmem + lane_base + L.tmem_p + (g & 1) * (kTile / 2) + ch * 32, dpv);
          tmem_wait_ld();
          if (c == kChunks - 1) {  // the score buffer is free for the next product while this warp computes
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
              mbar_arrive_cluster_relaxed(sf_leader + sb * 8);
              // dK: this warpgroup's last unit of query tile g: this warp is done with the dP^T buffer
              if (kDK && s + 2 >= maps) mbar_arrive_cluster_relaxed(df_leader + (g & 1) * 8);
            }
          }
          const int qc0 = half * 64 + ch * 32;  // query column inside the tile
          // valid query columns e: lo <= e < hi (causal: queries at or after this key)
          const int hi = live ? p.T - (qt + qc0) : 0;
          const int lo = p.causal ? key - (qt + qc0) : 0;
          uint32_t packed[16];
          // staged per query column: log2-domain log-sum-exp and alpha_s * delta (16-byte aligned rows)
          const float4* lse4 = reinterpret_cast<const float4*>(lse_row + qc0);
          const float4* ald4 = reinterpret_cast<const float4*>(delta_row + qc0);
          auto body = [&](auto masked) {
#pragma unroll
            for (int e4 = 0; e4 < 8; ++e4) {
              const float4 ls = lse4[e4];
              float4 ad = make_float4(0.f, 0.f, 0.f, 0.f);
              if (kDK) ad = ald4[e4];
              const float lsv[4] = {ls.x, ls.y, ls.z, ls.w}, adv[4] = {ad.x, ad.y, ad.z, ad.w};
#pragma unroll
              for (int cc = 0; cc < 4; cc += 2) {
                const int e = e4 * 4 + cc;
                float p0 = ex2(fmaf(sv[e], sc2, -lsv[cc])), p1 = ex2(fmaf(sv[e + 1], sc2, -lsv[cc + 1]));
                if (masked) {
                  p0 = (e >= lo && e < hi) ? p0 : 0.f;
                  p1 = (e + 1 >= lo && e + 1 < hi) ? p1 : 0.f;
                }
                if (kDK) {  // dS^T = P^T (alpha dP^T - alpha delta)
                  packed[e / 2] = pack2<T>(p0 * fmaf(al, dpv[e], -adv[cc]), p1 * fmaf(al, dpv[e + 1], -adv[cc + 1]));
                } else {
                  pm[e] = s == 0 ? al * p0 : fmaf(al, p0, pm[e]);
                  pm[e + 1] = s == 0 ? al * p1 : fmaf(al, p1, pm[e + 1]);
                  packed[e / 2] = pack2<T>(pm[e], pm[e + 1]);
                }
              }
            }
          };
          if (lo <= 0 && hi >= 32) body(std::false_type{});
          else body(std::true_type{});
          if (kDK || s == maps - 1) {
            // the tile buffer written here must have been read by the product two uses ago (dK: this
            // warpgroup's previous unit, u - 2; dV: query tile g - 2); waited for only now, so the
            // arithmetic above overlaps that product
            if (c == 0) {
              if (kDK && u >= 2) free_tile = mbar_wait(&t_empty[u & 1], ((u - 2) >> 1) & 1u, ab, 33);
              if (!kDK && g >= 2) free_tile = mbar_wait(&t_empty[g & 1], ((g - 2) >> 1) & 1u, ab, 33);
              free_tile = __all_sync(0xffffffffu, free_tile);
            }
            if (free_tile) {
#pragma unroll
              for (int e = 0; e < 4; ++e)
                st_shared_v4(ta + half * kBox + sw128_offset(r, ch * 4 + e), packed[4 * e], packed[4 * e + 1],
                             packed[4 * e + 2], packed[4 * e + 3]);
            }
          }
        }
        if (!free_tile) ok = false;
        if (kDK || s == maps - 1) fence_proxy_async();
      }
      if (!entered && lane == 0) {  // aborted unit: counts stay whole
        mbar_arrive_cluster_relaxed(sf_leader + sb * 8);
        if (kDK && s + 2 >= maps) mbar_arrive_cluster_relaxed(df_leader + (g & 1) * 8);
      }
      // the unit's tile (dK: dS^T every unit; dV: the mixed P^T after a query tile's last map) handed to
      // the accumulation issuer once every warp stored its rows; dV units before the last map hand nothing
      // over and pass without a barrier
      if (kDK || s == maps - 1) {
        tc_fence_before();
        named_bar_sync(kPing ? 3 + wg : 1, kPing ? 128 : 256);
        if (arriver) mbar_arrive_remote(pf_leader + (kDK ? (u & 1) : (g & 1)) * 8);
      }
    }
    if (wg == 0 && ok) ok = mbar_wait(&o_full, 0, ab, 34);
    ok = __all_sync(0xffffffffu, ok);
    tc_fence_after();
    if (wg == 0 && ok && kDK && p.dk) {
      for (int m = 0; m < maps; ++m) {
        const float gamma = p.scales[m] * gsc;
        for (int ins = 0; ins < L.nins; ++ins)
          for (int c = 0; c < L.ncol / 2; c += 32) {
            float vv[32];
            if (ni > 0) {  // (an empty query share has no accumulator: its partial is zero)
              tmem_ld32(tmem + lane_base + L.tmem_acc + m * (L.kw / 2) + ins * (L.ncol / 2) + c, vv);
              tmem_wait_ld();
            }
            if (live) {
              const int col = ins * L.ncol + half * (L.ncol / 2) + c;
              const int gi = col / p.R;
              const int64_t row = row_of(km.base, km.sb, km.sbr, b, p.branch0[m] + gi, key);
              if (p.ksplit > 1) {  // compact partial row (b, map, branch, key)
                const int64_t crow = (((int64_t)b * maps + m) * p.group + gi) * p.T + key;
                store_part32(p.part, ((int64_t)khalf * p.part_rows + crow) * p.R + (col % p.R), vv, gamma, ni == 0);
              } else {
                store_grad32<T>(p.dk, row * p.R + (col % p.R), vv, gamma, p.overwrite != 0);
              }
            }
          }
      }
    }
    if (wg == 0 && ok && !kDK && p.dv) {
      for (int ins = 0; ins < dins; ++ins)
        for (int c = 0; c < dn / 2; c += 32) {
          float vv[32];
          if (ni > 0) {
            tmem_ld32(tmem + lane_base + L.tmem_acc + ins * (dn / 2) + c, vv);
            tmem_wait_ld();
          }
          const int64_t off = ((int64_t)b * p.T + key) * p.D + ins * dn + half * (dn / 2) + c;
          if (live && p.ksplit > 1) store_part32(p.part, (int64_t)khalf * p.part_rows * p.D + off, vv, 1.f, ni == 0);
          else if (live) store_grad32<T>(p.dv, off, vv, 1.f, p.overwrite != 0);
        }
    }
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();
  if (warp == 1) tmem_dealloc<2>(tmem, L.tmem_cols);
}

// d alpha_s (kind 0) and d gamma_s (kind 1) += (store: =) the sum of the dQ kernel's n per-(CTA, warp)
// partials of map s: every thread adds a strided subset in index order, then a fixed-shape tree over the
// block.
__global__ void __launch_bounds__(256) scalar_reduce_kernel(const float* part, int n, int maps, float* dweight,
                                                            float* dscale, int store) {
  __shared__ float red[256];
  grid_dependency_wait();
  grid_launch_dependents();
  const int m = blockIdx.x, kind = blockIdx.y;
  float* out = kind == 0 ? dweight : dscale;
  if (!out) return;
  const float* src = part + (size_t)kind * n * maps;
  float s = 0.f;
  for (int i = threadIdx.x; i < n; i += 256) s += src[(size_t)i * maps + m];
  red[threadIdx.x] = s;
  __syncthreads();
  for (int w = 128; w; w >>= 1) {
    if (threadIdx.x < w) red[threadIdx.x] += red[threadIdx.x + w];
    __syncthreads();
  }
  if (threadIdx.x == 0) out[m] = store ? red[0] : out[m] + red[0];
}

// Destination rows of a split launch's compact partial rows: c = ((b * maps + s) * group + gi) * T + t
// -> row_of(base, sb, sbr, b, branch0[s] + gi, t) (dQ, dK), or row c itself when maps == 0 (dV).
struct SplitRows {
  int64_t base, sb, sbr;
  int maps, group, T;
  int branch0[kMaxMaps];
};

// The shares of a split launch added in share order (fp32) and stored into the gradient: once in T
// (overwrite), else added to its fp32 row.  Every thread takes 4 consecutive columns of one row.
template <typename T>
__global__ void __launch_bounds__(256) split_combine_kernel(const float* __restrict__ part, int ksplit, int64_t rows,
                                                            int cols, SplitRows d, void* dst, int overwrite) {
  grid_dependency_wait();
  grid_launch_dependents();
  const int c4 = cols / 4;
  const int64_t n = rows * c4, plane = rows * cols;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t c = i / c4;
    const int x = (int)(i % c4) * 4;
    float4 a = *reinterpret_cast<const float4*>(part + c * cols + x);
    for (int h = 1; h < ksplit; ++h) {
      const float4 e = *reinterpret_cast<const float4*>(part + h * plane + c * cols + x);
      a.x += e.x;
      a.y += e.y;
      a.z += e.z;
      a.w += e.w;
    }
    int64_t row = c;
    if (d.maps) {
      const int t = (int)(c % d.T);
      int64_t r = c / d.T;
      const int gi = (int)(r % d.group);
      r /= d.group;
      row = row_of(d.base, d.sb, d.sbr, (int)(r / d.maps), d.branch0[r % d.maps] + gi, t);
    }
    if (overwrite) {
      *reinterpret_cast<uint2*>(static_cast<T*>(dst) + row * cols + x) =
          make_uint2(pack2<T>(a.x, a.y), pack2<T>(a.z, a.w));
    } else {
      float4* o = reinterpret_cast<float4*>(static_cast<float*>(dst) + row * cols + x);
      float4 v = *o;
      v.x += a.x;
      v.y += a.y;
      v.z += a.z;
      v.w += a.w;
      *o = v;
    }
  }
}

// delta[i] = the shares' partial row sums of a split delta sweep, added in share order.
__global__ void __launch_bounds__(256) delta_combine_kernel(const float* __restrict__ part, int ksplit, int64_t n,
                                                            float* delta) {
  grid_dependency_wait();
  grid_launch_dependents();
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    float a = part[i];
    for (int h = 1; h < ksplit; ++h) a += part[h * n + i];
    delta[i] = a;
  }
}

// Byte offsets of the split form's regions in the caller's workspace (each 256-byte aligned): the
// per-(CTA, warp) scalar partials of every share, the delta sweep's partial row sums, and the fp32
// partial planes of dQ, dK (compact rows) and dV.
struct SplitWorkspace {
  int64_t scalar, delta, dq, dk, dv, total;
};

inline SplitWorkspace split_workspace(int B, int T, int R, int D, int maps, int group, int ksplit) {
  auto up = [](int64_t x) { return (x + 255) & ~(int64_t)255; };
  const int64_t pairs = (int64_t)B * ((T + kTile - 1) / kTile);
  const int64_t f = (int64_t)sizeof(float);
  const int64_t qk = (int64_t)ksplit * B * maps * group * T * R * f;
  SplitWorkspace w;
  w.scalar = 0;
  w.delta = up(2 * (2 * pairs * ksplit * 4) * maps * f);
  w.dq = w.delta + up((int64_t)ksplit * B * maps * T * f);
  w.dk = w.dq + up(qk);
  w.dv = w.dk + up(qk);
  w.total = w.dv + up((int64_t)ksplit * B * T * D * f);
  return w;
}

// Two shares when the split launches' CTAs (four per pair) fit on the SMs at once and there are several
// maps (one map keeps its given delta's exact correction of d gamma, which needs whole rows).  Measured at
// T = 2048, four maps, three streams: B2 (32 pairs) 219 -> 178 us; B4, where the split launches' 256 CTAs
// queue for 148 SMs, 276 -> 322 us.
inline int bwd_split(int maps, int64_t pairs, int sms) { return (maps > 1 && 4 * pairs <= sms) ? 2 : 1; }

template <typename Kern>
int launch_pair(Kern kern, const Layout& L, int pairs, const CUtensorMap& tq, const CUtensorMap& tk,
                const CUtensorMap& tv, const CUtensorMap& tdy, const CUtensorMap& tacc, const Params& p,
                cudaStream_t st) {
  const int smem = (L.smem < 120 * 1024 ? 120 * 1024 : L.smem) + 1024;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
    return record_cuda_error();
  return launch_kernel(kern, dim3((unsigned)(2 * pairs), 1, 1), dim3(kThreads, 1, 1), smem, st, true, tq, tk, tv, tdy,
                       tacc, p);
}

}  // namespace bwdm
}  // namespace attn
}  // namespace da

extern "C" int64_t da_attn_bwd_workspace_size(int B, int T, int maps) {
  if (B <= 0 || T <= 0 || maps < 1 || maps > da::attn::kMaxMaps) return -1;
  const int64_t pairs = (int64_t)B * ((T + da::attn::bwdm::kTile - 1) / da::attn::bwdm::kTile);
  return 2 * (2 * pairs * 4) * maps * (int64_t)sizeof(float);
}

extern "C" int64_t da_attn_bwd_split_workspace_size(int B, int T, int R, int D, int maps, int group) {
  using namespace da::attn::bwdm;
  if (B <= 0 || T <= 0 || R <= 0 || D <= 0 || group < 1 || maps < 1 || maps > da::attn::kMaxMaps) return -1;
  const int64_t pairs = (int64_t)B * ((T + kTile - 1) / kTile);
  const int ks = bwd_split(maps, pairs, da::sm_count());
  return ks > 1 ? split_workspace(B, T, R, D, maps, group, ks).total : 0;
}

namespace {

int attn_bwd_entry(const void* q, int64_t q_rows, int64_t q_base, int64_t q_sb, int64_t q_sbr, const void* k,
                   int64_t k_rows, int64_t k_base, int64_t k_sb, int64_t k_sbr, const void* v, const void* dy, int B,
                   int T, int R, int D, int maps, int group, const int* branch0, int causal, int dtype,
                   const float* scales, const float* weights, const float* lse, float* delta, int delta_given,
                   float* dq, float* dk, float* dv, float* dscale, float* dweight, void* workspace,
                   int64_t workspace_bytes, int overwrite, int* status, void* stream) {
  using namespace da;
  using namespace da::attn::bwdm;
  if (!q || !k || !v || !dy || !branch0 || !scales || !lse || !delta || !status) return DA_ERR_NULL;
  if (dtype != DA_BF16 && dtype != DA_F16) return DA_ERR_DTYPE;
  if (int rc = bind_device(q)) return rc;
  if (B <= 0 || T <= 0 || group < 1 || R <= 0 || R % 64 || maps < 1 || maps > attn::kMaxMaps) return DA_ERR_SHAPE;
  if (D != 256 && D != 512) return DA_ERR_UNSUPPORTED;
  const int kw = group * R;
  if ((kw != 128 && kw != 256 && kw != 512) || maps * kw > 512) return DA_ERR_UNSUPPORTED;
  for (int kind = 0; kind < 3; ++kind) {
    const Layout L = make_layout(kind, maps, group, R, D);
    if (L.nst < 2 || L.nsq < 2 || L.tmem_cols > 512) return DA_ERR_UNSUPPORTED;
  }
  if ((reinterpret_cast<uintptr_t>(dq) | reinterpret_cast<uintptr_t>(dk) | reinterpret_cast<uintptr_t>(dv)) & 15)
    return DA_ERR_ALIGN;
  Params p;
  p.q_rows = q_rows; p.q_base = q_base; p.q_sb = q_sb; p.q_sbr = q_sbr;
  p.k_rows = k_rows; p.k_base = k_base; p.k_sb = k_sb; p.k_sbr = k_sbr;
  p.B = B; p.T = T; p.R = R; p.D = D; p.maps = maps; p.group = group; p.causal = causal;
  for (int s = 0; s < attn::kMaxMaps; ++s) {
    p.branch0[s] = s < maps ? branch0[s] : 0;
    if (s < maps) {
      if (p.branch0[s] < 0) return DA_ERR_SHAPE;
      // every row a launch can address lies inside the row maps
      const int64_t last_b = (int64_t)(B - 1), last_br = (int64_t)(p.branch0[s] + group - 1);
      if (q_base + last_b * q_sb + last_br * q_sbr + (T - 1) >= q_rows) return DA_ERR_SHAPE;
      if (k_base + last_b * k_sb + last_br * k_sbr + (T - 1) >= k_rows) return DA_ERR_SHAPE;
    }
  }
  if (q_base < 0 || k_base < 0) return DA_ERR_SHAPE;
  p.scales = scales; p.weights = weights; p.lse = lse; p.delta = delta; p.delta_given = delta_given;
  if (overwrite)  // one writer per gradient row: the maps' branch ranges must not overlap
    for (int s1 = 0; s1 < maps; ++s1)
      for (int s2 = s1 + 1; s2 < maps; ++s2)
        if (branch0[s1] < branch0[s2] + group && branch0[s2] < branch0[s1] + group) return DA_ERR_UNSUPPORTED;
  p.dq = dq; p.dk = dk; p.dv = dv; p.dscale = dscale; p.dweight = dweight; p.status = status;
  p.overwrite = overwrite ? 1 : 0;
  p.ksplit = 1;
  p.part = nullptr;
  p.part_rows = 0;
  p.delta_part = nullptr;
  const int npairs = B * ((T + kTile - 1) / kTile);
  // The split form (bwd_split) when the caller's workspace holds it and every gradient row has one writer
  // (maps on disjoint branch ranges), so that a combine can store each row once.
  bool disjoint = true;
  for (int s1 = 0; s1 < maps; ++s1)
    for (int s2 = s1 + 1; s2 < maps; ++s2)
      if (branch0[s1] < branch0[s2] + group && branch0[s2] < branch0[s1] + group) disjoint = false;
  const int ks = bwd_split(maps, npairs, sm_count());
  const SplitWorkspace sw = split_workspace(B, T, R, D, maps, group, ks);
  const int ksplit = (ks > 1 && disjoint && workspace && workspace_bytes >= sw.total) ? ks : 1;
  const int64_t n_part = (int64_t)2 * npairs * ksplit * 4;  // partials per map and kind: (CTA, softmax warp)
  p.scalar_part = nullptr;
  if (ksplit > 1 || dscale || (dweight && !delta_given)) {
    if (!workspace || workspace_bytes < 2 * n_part * maps * (int64_t)sizeof(float)) return DA_ERR_WORKSPACE;
    if (reinterpret_cast<uintptr_t>(workspace) & 15) return DA_ERR_ALIGN;
    p.scalar_part = static_cast<float*>(workspace);
  }
  p.trace = debug_trace();
  const CUtensorMapDataType tdt = dtype == DA_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUtensorMap tq, tk, tv, tdy, tq128, tk128;
  int rc = make_tmap_2d(&tq, q, tdt, 2, R, q_rows, (uint64_t)R * 2, 64, 64);
  if (rc) return rc;
  rc = make_tmap_2d(&tk, k, tdt, 2, R, k_rows, (uint64_t)R * 2, 64, 64);
  if (rc) return rc;
  // 128-row boxes of the MN-major accumulation operands (K for dQ, Q for dK)
  rc = make_tmap_2d(&tq128, q, tdt, 2, R, q_rows, (uint64_t)R * 2, 64, 128);
  if (rc) return rc;
  rc = make_tmap_2d(&tk128, k, tdt, 2, R, k_rows, (uint64_t)R * 2, 64, 128);
  if (rc) return rc;
  CUtensorMap tdy2, tvq, tdyq;
  {  // V and dY: [B*T, D] as (64-column block, row, block index); a box is 64 rows x kDpBlocks blocks for
     // the dK kernel's dP stages, 64 rows x kDpBlocksQ blocks for the dQ kernel's, 64 rows x 2 blocks for
     // the dV kernel's dY operand
    const uint64_t dims[3] = {64, (uint64_t)B * T, (uint64_t)D / 64};
    const uint64_t strides[2] = {(uint64_t)D * 2, 128};
    const uint32_t box[3] = {64, 64, kDpBlocks};
    rc = make_tmap_blocks(&tv, v, tdt, 2, 3, dims, strides, box);
    if (rc) return rc;
    rc = make_tmap_blocks(&tdy, dy, tdt, 2, 3, dims, strides, box);
    if (rc) return rc;
    const uint32_t box2[3] = {64, 64, 2};
    rc = make_tmap_blocks(&tdy2, dy, tdt, 2, 3, dims, strides, box2);
    if (rc) return rc;
    // the dQ kernel's dP stages: kDpBlocksQ blocks of each of V and dY per box (the kernel's stage layout
    // and transaction count assume exactly this box)
    const uint32_t boxq[3] = {64, 64, kDpBlocksQ};
    rc = make_tmap_blocks(&tvq, v, tdt, 2, 3, dims, strides, boxq);
    if (rc) return rc;
    rc = make_tmap_blocks(&tdyq, dy, tdt, 2, 3, dims, strides, boxq);
    if (rc) return rc;
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const bool bf16 = dtype == DA_BF16;
  const int sms = sm_count();
  // the query-parallel kernel, then the fixed-order sums of its d alpha / d gamma partials
  auto run_dq = [&](const Params& pp) -> int {
    const Layout L = make_layout(0, maps, group, R, D);
    const int cpairs = npairs * pp.ksplit;
    int r = bf16 ? launch_pair(dq_mixed_kernel<__nv_bfloat16>, L, cpairs, tq, tk, tvq, tdyq, tk128, pp, st)
                 : launch_pair(dq_mixed_kernel<__half>, L, cpairs, tq, tk, tvq, tdyq, tk128, pp, st);
    float* dw = pp.delta_given ? nullptr : pp.dweight;
    if (r || !pp.scalar_part || (!dw && !pp.dscale)) return r;
    return launch_kernel(scalar_reduce_kernel, dim3((unsigned)maps, 2, 1), dim3(256, 1, 1), 0, st, false,
                         (const float*)pp.scalar_part, (int)(2 * cpairs * 4), maps, dw, pp.dscale, pp.overwrite);
  };
  auto run_dkv = [&](const Params& pp, bool dkk) -> int {
    const Layout L = make_layout(dkk ? 1 : 2, maps, group, R, D);
    const int cpairs = npairs * pp.ksplit;
    if (dkk)
      return bf16 ? launch_pair(dkv_mixed_kernel<__nv_bfloat16, true>, L, cpairs, tq, tk, tv, tdy, tq128, pp, st)
                  : launch_pair(dkv_mixed_kernel<__half, true>, L, cpairs, tq, tk, tv, tdy, tq128, pp, st);
    return bf16 ? launch_pair(dkv_mixed_kernel<__nv_bfloat16, false>, L, cpairs, tq, tk, tv, tdy2, tq128, pp, st)
                : launch_pair(dkv_mixed_kernel<__half, false>, L, cpairs, tq, tk, tv, tdy2, tq128, pp, st);
  };
  auto grid_for = [&](int64_t n) {
    const int64_t blocks = (n + 255) / 256;
    return dim3((unsigned)(blocks < 4 * sms ? blocks : 4 * sms));
  };
  if (ksplit == 1) {
    // the query-parallel kernel runs first: without a given delta it produces it for the other two
    if (dq || dscale || !delta_given)
      if ((rc = run_dq(p))) return rc;
    if (dk && (rc = run_dkv(p, true))) return rc;
    if (dv) rc = run_dkv(p, false);
    return rc;
  }
  // Split form: every launch runs two CTA pairs per pair, each on one share of the long row, and a combine
  // adds the shares' fp32 partial rows in share order.  Without a given delta the delta sweep runs first
  // on its own (with d alpha); the dQ launch then takes the combined, exact delta.
  char* ws = static_cast<char*>(workspace);
  p.ksplit = ksplit;
  p.delta_part = reinterpret_cast<float*>(ws + sw.delta);
  SplitRows qr{q_base, q_sb, q_sbr, maps, group, T, {}}, kr{k_base, k_sb, k_sbr, maps, group, T, {}};
  SplitRows vr{0, 0, 0, 0, 1, T, {}};
  for (int s = 0; s < attn::kMaxMaps; ++s) qr.branch0[s] = kr.branch0[s] = vr.branch0[s] = p.branch0[s];
  const int64_t crows = (int64_t)B * maps * group * T;
  auto combine = [&](const float* part, int64_t rows, int cols, const SplitRows& d, void* dst) -> int {
    const dim3 grid = grid_for(rows * cols / 4);
    return bf16 ? launch_kernel(split_combine_kernel<__nv_bfloat16>, grid, dim3(256), 0, st, false, part, ksplit,
                                rows, cols, d, dst, p.overwrite)
                : launch_kernel(split_combine_kernel<__half>, grid, dim3(256), 0, st, false, part, ksplit, rows,
                                cols, d, dst, p.overwrite);
  };
  if (!delta_given) {
    Params pd = p;
    pd.dq = nullptr;
    pd.dscale = nullptr;
    if ((rc = run_dq(pd))) return rc;
    const int64_t n = (int64_t)B * maps * T;
    if ((rc = launch_kernel(delta_combine_kernel, grid_for(n), dim3(256), 0, st, false,
                            (const float*)p.delta_part, ksplit, n, delta)))
      return rc;
    p.delta_given = 1;
    p.dweight = nullptr;
  }
  if (dq || dscale) {
    Params pq = p;
    pq.part = reinterpret_cast<float*>(ws + sw.dq);
    pq.part_rows = crows;
    if ((rc = run_dq(pq))) return rc;
    if (dq && (rc = combine(pq.part, crows, R, qr, dq))) return rc;
  }
  if (dk) {
    Params pk = p;
    pk.part = reinterpret_cast<float*>(ws + sw.dk);
    pk.part_rows = crows;
    if ((rc = run_dkv(pk, true)) || (rc = combine(pk.part, crows, R, kr, dk))) return rc;
  }
  if (dv) {
    Params pv = p;
    pv.part = reinterpret_cast<float*>(ws + sw.dv);
    pv.part_rows = (int64_t)B * T;
    if ((rc = run_dkv(pv, false)) || (rc = combine(pv.part, (int64_t)B * T, D, vr, dv))) return rc;
  }
  return rc;
}

}  // namespace

extern "C" int da_attn_bwd_mixed(const void* q, int64_t q_rows, int64_t q_base, int64_t q_sb, int64_t q_sbr,
                                 const void* k, int64_t k_rows, int64_t k_base, int64_t k_sb, int64_t k_sbr,
                                 const void* v, const void* dy, int B, int T, int R, int D, int maps, int group,
                                 const int* branch0, int causal, int dtype, const float* scales,
                                 const float* weights, const float* lse, float* delta, int delta_given, float* dq,
                                 float* dk, float* dv, float* dscale, float* dweight, void* workspace,
                                 int64_t workspace_bytes, int* status, void* stream) {
  return attn_bwd_entry(q, q_rows, q_base, q_sb, q_sbr, k, k_rows, k_base, k_sb, k_sbr, v, dy, B, T, R, D, maps, group,
                        branch0, causal, dtype, scales, weights, lse, delta, delta_given, dq, dk, dv, dscale, dweight,
                        workspace, workspace_bytes, 0, status, stream);
}

extern "C" int da_attn_bwd_mixed_ow(const void* q, int64_t q_rows, int64_t q_base, int64_t q_sb, int64_t q_sbr,
                                    const void* k, int64_t k_rows, int64_t k_base, int64_t k_sb, int64_t k_sbr,
                                    const void* v, const void* dy, int B, int T, int R, int D, int maps, int group,
                                    const int* branch0, int causal, int dtype, const float* scales,
                                    const float* weights, const float* lse, float* delta, int delta_given, void* dq,
                                    void* dk, void* dv, float* dscale, float* dweight, void* workspace,
                                    int64_t workspace_bytes, int* status, void* stream) {
  return attn_bwd_entry(q, q_rows, q_base, q_sb, q_sbr, k, k_rows, k_base, k_sb, k_sbr, v, dy, B, T, R, D, maps, group,
                        branch0, causal, dtype, scales, weights, lse, delta, delta_given, static_cast<float*>(dq),
                        static_cast<float*>(dk), static_cast<float*>(dv), dscale, dweight, workspace, workspace_bytes,
                        1, status, stream);
}
