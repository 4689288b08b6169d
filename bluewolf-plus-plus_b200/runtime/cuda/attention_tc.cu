// Attention forward on sm_100a tensor cores, single pass with online softmax.
//
//   O[bh, m, :] = sum_n softmax_n(scale * q_m . k_n [n <= m if causal]) v_n
//
// One CTA owns 256 query rows of one (batch, head) as two 128-row tiles A and
// B that ping-pong: while the softmax warps of one tile turn its S into P, the
// tensor core works on the other tile.  Per 128-key block j:
//   S_X = Q_X K_j^T          tcgen05 M=128 N=128 K=16 (Q, K K-major, bf16)
//   P_X = exp2(S_X*c - m)    softmax warps, four threads per row (32 keys
//                            each, 16-lane TMEM shapes); P as bf16 pairs
//                            written back into S_X's TMEM columns
//   O_X += P_X V_j           tcgen05 M=128 N=D K=16, A = P from TMEM,
//                            B = V MN-major from smem
// S_A, S_B, O_A, O_B live in TMEM (4 x 128 columns for D = 128).  The running
// max only moves when it grows by more than 2^8 (log2 domain), so O is
// rescaled (tcgen05.ld / st) rarely; P <= 256 stays exact enough in bf16.
// The softmax arithmetic uses paired fp32 lanes (fma/add .f32x2) and 3-input
// max to halve its instruction count; items go in groups of heads whose
// K / V fit a share of L2 (read from DRAM once, shared through L2), heaviest
// first inside a group.
//
// Warp roles (576 threads): warps 0-7 softmax of tile A, warps 8-15
// softmax of tile B (warp w reads TMEM lanes 32*(w%4)..; the two warps of a
// lane quarter take 16 rows each), warp 16 TMA producer (Q once; K and V
// double-buffered, 3-D tensor maps so ragged S zero-fills per head), warp
// 17 TMEM allocator + single-thread MMA issuer.
// MMA issue order per block: PV_A(j), S_A(j+1), PV_B(j), S_B(j+1), so one
// tile's softmax always overlaps the other tile's MMAs.
//
// Every wait is bounded (BWPP_WAIT_LIMIT_NS); on expiry the kernel records
// BWPP_CUDA_ERR_TIMEOUT, unwinds, frees TMEM and returns.
#include "attention_common.cuh"

#include <algorithm>

namespace {

using namespace bwpp_attn;
// warps 0-15 softmax, 16 producer, 17 MMA.  18 warps put 5 on two of the
// SM's four register files (16K registers each), so a thread gets 96.
constexpr int THREADS = 576;
constexpr int W_PROD = 16, W_MMA = 17;
// Of every 8 score pairs, this many take exp2 on the FMA pipe (exp2_fma2),
// the rest on MUFU: one ex2 per score would keep MUFU as busy as the tensor
// core, so part of the load moves to the otherwise idle FMA pipe.
constexpr int kEmuPairsPer8 = 2;

template <int D, bool F16 = false>
struct Cfg {
  static constexpr int BOXES = D / 64;
  static constexpr int TILE = BOXES * BOX;  // Q / K / V tile bytes
  static constexpr int OFF_Q = 0;           // 2 tiles
  static constexpr int OFF_K = 2 * TILE;    // 2 stages
  static constexpr int OFF_V = 4 * TILE;    // 2 stages
  static constexpr int OFF_BAR = 6 * TILE;
  static constexpr int SMEM = OFF_BAR + 512 + 1024;
  static constexpr uint32_t TMEM_S = 0;        // S_A at 0, S_B at 128
  static constexpr uint32_t TMEM_O = 2 * BN;   // O_A at 256, O_B at 256 + D
  static constexpr uint32_t TMEM_COLS = 512;
  // split launches: per softmax warp, its O rows ([D/64][8][lane] float4)
  // and one float4 (max a, max b, sum a, sum b) per lane
  static constexpr int WARP_FLOATS = (D / 64) * 8 * 32 * 4 + 32 * 4;
  // Q, K, V and P are all bf16, or all f16 (the half ABI)
  static constexpr uint32_t IDESC_S = make_idesc_f32acc(BM, BN, 0, 0, F16 ? 1u : 0u);
  static constexpr uint32_t IDESC_PV = make_idesc_f32acc(BM, D, 0, 1, F16 ? 1u : 0u);
  static_assert(SMEM <= 232448, "shared memory budget");
};

struct Bars {
  uint64_t q_full[2], q_empty[2];
  uint64_t k_full[2], k_empty[2];
  uint64_t v_full[2], v_empty[2];
  uint64_t s_full[2], s_free[2], p_full[2], pv_done[2], o_free[2];
  uint64_t sched_full[2], sched_empty[2];
  uint64_t drain;
  int item[2];
  uint32_t tmem;
  int abort_flag;
};
static_assert(sizeof(Bars) <= 512, "barrier block");

// Work item w (in the order CTAs take them): the heads go in groups of
// `group` (causal: as many as keep their K / V in a fraction of L2; else 1),
// and inside a group the items go heaviest first across its heads: pair
// pairs - 1 of every head of the group, then pair pairs - 2, ...  The CTAs
// running together then share the group's K / V through L2, and, since the
// work counter hands items out in this order, the last items of the launch
// are the lightest (with causal items ordered head by head, a late heavy
// item left most CTAs idle at the end when there are few heads per GPU).
// Pair p is rows q0 .. q0 + 255 as tiles A and B, q0 = 2 p BM.
struct Item {
  uint32_t bh, q0;
  int nblk[2], n;
  uint32_t kb0;  // first key block (0 but in a split launch)
};

// Split tail of a non-causal launch whose last round of items would be at
// most half full: the main launch takes the whole rounds, and a second,
// split launch (the SPLIT instantiation of the kernel) runs each remaining
// item as two halves over the key blocks [0, n/2) and [n/2, n), so that
// round ends in half the time.  The two halves of an item merge through
// global memory: every softmax warp of a half counts itself in on its
// (item, warp) counter; the first to arrive stores its unnormalised O rows
// and (max, sum) to the item's slot and counts them written; the second
// waits for that (only for a half that has already arrived, so both need
// not run at the same time), merges the two in half order and stores O.
// The main launch's code is the kernel without any of this.
struct AttnSplit {
  uint32_t first;   // item index of split item 0
  uint32_t epoch;   // tag of this launch's counts
  float *partials;  // [split item][16 warps][WARP_FLOATS]
  unsigned long long *counters;  // [split item][16 warps][arrived, written]
};

template <bool SPLIT>
__device__ __forceinline__ Item decode_item(int w, uint32_t pairs, uint32_t BH, uint32_t group,
                                            uint32_t Sq, uint32_t Skv, int causal,
                                            const AttnSplit &sp) {
  Item it;
  it.kb0 = 0;
  uint32_t half = 0;
  if constexpr (SPLIT) {  // work item w: half w & 1 of item first + w / 2
    half = (uint32_t)w & 1u;
    w = (int)(sp.first + ((uint32_t)w >> 1));
  }
  const uint32_t per_group = group * pairs;
  const uint32_t g0 = (uint32_t)w / per_group * group;  // first head of w's group
  const uint32_t r = (uint32_t)w % per_group;
  const uint32_t nh = min(group, BH - g0);              // heads in that group
  it.bh = g0 + r % nh;
  it.q0 = (pairs - 1 - r / nh) * 2 * BM;
  it.nblk[0] = blocks_for(it.q0, Sq, Skv, causal);
  it.nblk[1] = blocks_for(it.q0 + BM, Sq, Skv, causal);
  it.n = max(it.nblk[0], it.nblk[1]);
  if constexpr (SPLIT) {  // non-causal: a tile with rows sees all it.n blocks
    const int h0 = it.n / 2;
    const int cnt = half ? it.n - h0 : h0;
    it.kb0 = half ? (uint32_t)h0 : 0u;
    for (int X = 0; X < 2; ++X) it.nblk[X] = it.nblk[X] > 0 ? cnt : 0;
    it.n = cnt;
  }
  return it;
}

// Where a softmax thread's two rows of O live, for split_epilogue.
struct SplitRows {
  uint32_t o_col, bh, Sq, qa, qb;
  int cpair, lane, warp;
  float scale_log2;
};

// Epilogue of one softmax warp for half (w & 1) of split item w >> 1 (see
// AttnSplit): the first half to arrive stores its unnormalised O rows and
// (max, sum) and counts them written; the second merges the two and stores
// O (and the log-sum-exp).  Weights, sums and the products' sum are rounded
// in half order, so the result does not depend on which half came first.
// False on a wait that ran out.
template <int D, bool F16>
__device__ __forceinline__ bool split_epilogue(const SplitRows &rw, const AttnIO &io,
                                               const AttnSplit &sp, uint32_t w, float la,
                                               float lb, float ma, float mb, int *status) {
  constexpr int WF = (D / 64) * 8 * 32 * 4 + 32 * 4;
  const int lane = rw.lane;
  const bool h0 = (w & 1u) == 0;
  float *slot = sp.partials + ((size_t)(w >> 1) * 16 + rw.warp) * WF;
  unsigned long long *ctr = sp.counters + ((size_t)(w >> 1) * 16 + rw.warp) * 2;
  uint32_t before = 0;
  if (lane == 0) before = epoch_arrive(ctr, sp.epoch);
  before = __shfl_sync(0xffffffffu, before, 0);
  if (before == 0) {
#pragma unroll 1
    for (int c = 0; c < D / 64; ++c) {
      uint32_t ro[32];
      tmem_ld_16x256b_x8(rw.o_col + c * 64, ro);
      tc_wait_ld(ro);
#pragma unroll
      for (int k = 0; k < 8; ++k)
        __stcg(reinterpret_cast<float4 *>(slot + ((c * 8 + k) * 32 + lane) * 4),
               make_float4(__uint_as_float(ro[4 * k]), __uint_as_float(ro[4 * k + 1]),
                           __uint_as_float(ro[4 * k + 2]), __uint_as_float(ro[4 * k + 3])));
    }
    __stcg(reinterpret_cast<float4 *>(slot + ((D / 64) * 8 * 32 + lane) * 4),
           make_float4(ma, mb, la, lb));
    __threadfence();
    __syncwarp();
    if (lane == 0) epoch_arrive(ctr + 1, sp.epoch);
    return true;
  }
  bool okw = true;
  if (lane == 0) okw = epoch_wait(ctr + 1, sp.epoch, 1, status);
  if (!__shfl_sync(0xffffffffu, okw ? 1 : 0, 0)) return false;
  __syncwarp();  // lane 0's acquire orders the whole warp's loads below
  const float4 ml = __ldcg(reinterpret_cast<const float4 *>(slot + ((D / 64) * 8 * 32 + lane) * 4));
  float wm[2], wo[2], l[2], m[2];
  const float mine_m[2] = {ma, mb}, mine_l[2] = {la, lb}, oth_m[2] = {ml.x, ml.y},
              oth_l[2] = {ml.z, ml.w};
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const float m0 = h0 ? mine_m[r] : oth_m[r], m1 = h0 ? oth_m[r] : mine_m[r];
    const float l0 = h0 ? mine_l[r] : oth_l[r], l1 = h0 ? oth_l[r] : mine_l[r];
    const float M = fmaxf(m0, m1);
    const float e0 = m0 == -INFINITY ? 0.0f : fast_exp2((m0 - M) * rw.scale_log2);
    const float e1 = m1 == -INFINITY ? 0.0f : fast_exp2((m1 - M) * rw.scale_log2);
    wm[r] = h0 ? e0 : e1;
    wo[r] = h0 ? e1 : e0;
    m[r] = M;
    l[r] = __fadd_rn(__fmul_rn(e0, l0), __fmul_rn(e1, l1));
  }
  const float inv_a = l[0] > 0.0f ? 1.0f / l[0] : 0.0f, inv_b = l[1] > 0.0f ? 1.0f / l[1] : 0.0f;
  const bool va = rw.qa < rw.Sq, vb = rw.qb < rw.Sq;
  if (io.lse && (lane & 3) == 0) {
    if (va) io.lse[(size_t)rw.bh * rw.Sq + rw.qa] = l[0] > 0.0f ? m[0] * rw.scale_log2 + __log2f(l[0]) : -INFINITY;
    if (vb) io.lse[(size_t)rw.bh * rw.Sq + rw.qb] = l[1] > 0.0f ? m[1] * rw.scale_log2 + __log2f(l[1]) : -INFINITY;
  }
#pragma unroll 1
  for (int c = 0; c < D / 64; ++c) {
    uint32_t ro[32];
    tmem_ld_16x256b_x8(rw.o_col + c * 64, ro);
    tc_wait_ld(ro);
    float v[32];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const float4 t4 = __ldcg(reinterpret_cast<const float4 *>(slot + ((c * 8 + k) * 32 + lane) * 4));
      const float ot[4] = {t4.x, t4.y, t4.z, t4.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int r = e >> 1;  // e < 2: row a, else row b
        const float pm = __fmul_rn(__uint_as_float(ro[4 * k + e]), wm[r]);
        const float po = __fmul_rn(ot[e], wo[r]);
        v[4 * k + e] = (h0 ? __fadd_rn(pm, po) : __fadd_rn(po, pm)) * (r ? inv_b : inv_a);
      }
    }
    if (io.out_f32) {
      float *oa = io.out_f32 + ((size_t)rw.bh * rw.Sq + rw.qa) * D + c * 64 + rw.cpair;
      float *ob = oa + 8 * (size_t)D;
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        if (va) __stcs(reinterpret_cast<float2 *>(oa + 8 * k), make_float2(v[4 * k], v[4 * k + 1]));
        if (vb) __stcs(reinterpret_cast<float2 *>(ob + 8 * k), make_float2(v[4 * k + 2], v[4 * k + 3]));
      }
    }
    if (io.out_bf16) {
      const size_t head_col = (size_t)(rw.bh % io.H) * D + c * 64 + rw.cpair;
      uint16_t *oa = io.out_bf16 + ((size_t)(rw.bh / io.H) * rw.Sq + rw.qa) * io.ldo + head_col;
      uint16_t *ob = oa + 8 * (size_t)io.ldo;
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        if (va) *reinterpret_cast<uint32_t *>(oa + 8 * k) = pack2_16<F16>(v[4 * k], v[4 * k + 1]);
        if (vb) *reinterpret_cast<uint32_t *>(ob + 8 * k) = pack2_16<F16>(v[4 * k + 2], v[4 * k + 3]);
      }
    }
  }
  return true;
}

// Persistent: one CTA per SM takes work items (256 query rows of one head)
// until none is left: its first item is blockIdx.x, the next ones come from
// the context's work counter (items gridDim.x, gridDim.x + 1, ... in the
// order of decode_item, so the CTAs running together share a group of heads'
// K / V in L2, and a CTA that drew a short causal item simply draws again).  The
// producer publishes each item id through a two-slot ring (sched_full /
// sched_empty); every role walks the same item sequence.  Across items the
// K / V ring keeps streaming, the next item's Q is loaded as soon as the
// last S MMAs of the current item release Q (q_empty), and the next item's
// S MMAs run while the softmax warps are still in the previous epilogue; its
// first PV waits for that epilogue to read O (o_free).  All barrier phases
// are running counters over the CTA's whole item sequence.
template <int D, bool F16, bool SPLIT>
__global__ void __launch_bounds__(THREADS, 1)
    attention_tc_kernel(const __grid_constant__ CUtensorMap tmQ,
                        const __grid_constant__ CUtensorMap tmK,
                        const __grid_constant__ CUtensorMap tmV,
                        const AttnIO io, uint32_t BH, uint32_t Sq,
                        uint32_t Skv, float scale_log2, int causal,
                        uint32_t pairs, uint32_t group, uint32_t n_items, const AttnSplit sp,
                        int *sched, int *status) {
  using C = Cfg<D, F16>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t *smem = smem_raw + ((1024u - (raw & 1023u)) & 1023u);
  Bars *bar = reinterpret_cast<Bars *>(smem + C::OFF_BAR);
  volatile int *abort_flag = &bar->abort_flag;
  const int total = (int)n_items;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < 2; ++s) {
      mbar_init(&bar->q_full[s], 1);
      mbar_init(&bar->q_empty[s], 1);
      mbar_init(&bar->k_full[s], 1);
      mbar_init(&bar->k_empty[s], 1);
      mbar_init(&bar->v_full[s], 1);
      mbar_init(&bar->v_empty[s], 1);
      mbar_init(&bar->s_full[s], 1);
      mbar_init(&bar->s_free[s], 8);
      mbar_init(&bar->p_full[s], 8);
      mbar_init(&bar->pv_done[s], 1);
      mbar_init(&bar->o_free[s], 8);
      mbar_init(&bar->sched_full[s], 1);
      mbar_init(&bar->sched_empty[s], 17);  // MMA thread + 16 softmax warps
    }
    mbar_init(&bar->drain, 1);
    bar->abort_flag = 0;
    fence_mbar_init();
    prefetch_tmap(&tmQ);
    prefetch_tmap(&tmK);
    prefetch_tmap(&tmV);
  }
  if (warp == W_MMA) {
    tmem_alloc(&bar->tmem, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bar->tmem;

  if (warp == W_PROD) {
    // ----------------------------------------------------------- producer
    if (lane == 0) {
      uint32_t kc = 0, vc = 0;  // K / V blocks loaded so far
      bool ok = true;
      int w = (int)blockIdx.x;
      for (uint32_t seq = 0; ok && !*abort_flag; ++seq) {
        const int slot = seq & 1;
        if (!mbar_wait(&bar->sched_empty[slot], ((seq >> 1) & 1) ^ 1, status)) { ok = false; break; }
        bar->item[slot] = w < total ? w : -1;
        mbar_arrive(&bar->sched_full[slot]);
        if (w >= total) break;
        const Item it = decode_item<SPLIT>(w, pairs, BH, group, Sq, Skv, causal, sp);
        // K(0) first (its slot frees with the previous item's last S MMAs),
        // then both Q tiles.  Every item has at least one block (its first
        // row is below Sq and Skv >= 1).
        {
          const int s = kc & 1;
          if (!mbar_wait(&bar->k_empty[s], ((kc >> 1) & 1) ^ 1, status)) { ok = false; break; }
          mbar_arrive_expect_tx(&bar->k_full[s], C::TILE);
          load_rows<C::BOXES>(smem + C::OFF_K + s * C::TILE, &tmK, &bar->k_full[s], io, it.bh, Skv,
                              it.kb0 * BN);
          ++kc;
        }
        for (int X = 0; X < 2 && ok; ++X) {
          if (!mbar_wait(&bar->q_empty[X], (seq & 1) ^ 1, status)) { ok = false; break; }
          mbar_arrive_expect_tx(&bar->q_full[X], C::TILE);
          load_rows<C::BOXES>(smem + C::OFF_Q + X * C::TILE, &tmQ, &bar->q_full[X], io, it.bh, Sq,
                              it.q0 + X * BM);
        }
        for (int j = 0; j < it.n && ok && !*abort_flag; ++j) {
          if (j + 1 < it.n) {
            const int s = kc & 1;
            if (!mbar_wait(&bar->k_empty[s], ((kc >> 1) & 1) ^ 1, status)) { ok = false; break; }
            mbar_arrive_expect_tx(&bar->k_full[s], C::TILE);
            load_rows<C::BOXES>(smem + C::OFF_K + s * C::TILE, &tmK, &bar->k_full[s], io, it.bh,
                                Skv, (it.kb0 + j + 1) * BN);
            ++kc;
          }
          const int vs = vc & 1;
          if (!mbar_wait(&bar->v_empty[vs], ((vc >> 1) & 1) ^ 1, status)) { ok = false; break; }
          mbar_arrive_expect_tx(&bar->v_full[vs], C::TILE);
          load_rows<C::BOXES>(smem + C::OFF_V + vs * C::TILE, &tmV, &bar->v_full[vs], io, it.bh, Skv,
                              (it.kb0 + j) * BN);
          ++vc;
        }
        w = (int)gridDim.x + atomicAdd(sched, 1);
      }
      if (!ok) *abort_flag = 1;
    }
  } else if (warp == W_MMA) {
    // -------------------------------------------------------- MMA issuer
    if (lane == 0) {
      // Every smem descriptor is a base built once plus a byte offset known
      // at compile time per k step (the start-address field is the low 14
      // bits, addresses stay below 256 KB, so the add never carries out of
      // it): a group of 8 MMAs then costs the tensor core's time, not the
      // issuing thread's, which rebuilding descriptors per MMA made it.
      const uint64_t dq = make_smem_desc(smem_u32(smem + C::OFF_Q), 16, 1024, BWPP_SWIZZLE_128B);
      const uint64_t dk = make_smem_desc(smem_u32(smem + C::OFF_K), 16, 1024, BWPP_SWIZZLE_128B);
      const uint64_t dv = make_smem_desc(smem_u32(smem + C::OFF_V), BOX, 1024, BWPP_SWIZZLE_128B);
      // S_X = Q_X K^T into TMEM columns X * 128 (K in slot kslot)
      auto issue_s = [&](int X, int kslot) {
        const uint64_t qd = desc_add(dq, (uint32_t)X * C::TILE);
        const uint64_t kd = desc_add(dk, (uint32_t)kslot * C::TILE);
        const uint32_t d_tmem = tmem + C::TMEM_S + X * BN;
#pragma unroll
        for (int ks = 0; ks < D / 16; ++ks) {
          const uint32_t off = (ks >> 2) * BOX + (ks & 3) * 32;
          tc_mma_f16_ss(d_tmem, desc_add(qd, off), desc_add(kd, off), C::IDESC_S, ks > 0 ? 1u : 0u);
        }
        tc_commit(&bar->s_full[X]);
      };
      // O_X (+)= P_X V with P_X read from TMEM (16-bit pairs in key order
      // in the first 64 columns of S_X: 16 keys = 8 columns per MMA) and V
      // from smem slot vslot
      auto issue_pv = [&](int X, int vslot, bool first) {
        const uint64_t vd = desc_add(dv, (uint32_t)vslot * C::TILE);
        const uint32_t pt = tmem + C::TMEM_S + X * BN;
        const uint32_t d_tmem = tmem + C::TMEM_O + X * D;
#pragma unroll
        for (int ks = 0; ks < BN / 16; ++ks)
          tc_mma_f16_ts(d_tmem, pt + ks * 8, desc_add(vd, ks * 2048), C::IDESC_PV,
                        (!first || ks > 0) ? 1u : 0u);
        tc_commit(&bar->pv_done[X]);
      };
      uint32_t kc = 0, vc = 0;          // K / V blocks consumed
      uint32_t sc[2] = {0, 0};          // S MMAs issued per tile
      uint32_t pc[2] = {0, 0};          // P blocks consumed per tile
      bool ok = true;
      for (uint32_t seq = 0; ok && !*abort_flag; ++seq) {
        const int slot = seq & 1;
        if (!mbar_wait(&bar->sched_full[slot], (seq >> 1) & 1, status)) { ok = false; break; }
        const int w = bar->item[slot];
        mbar_arrive(&bar->sched_empty[slot]);
        if (w < 0) break;
        const Item it = decode_item<SPLIT>(w, pairs, BH, group, Sq, Skv, causal, sp);
        {
          // block 0: S_A(0), S_B(0)
          ok = mbar_wait(&bar->k_full[kc & 1], (kc >> 1) & 1, status);
          for (int X = 0; X < 2 && ok; ++X) ok = mbar_wait(&bar->q_full[X], seq & 1, status);
          for (int X = 0; X < 2 && ok; ++X) {
            if (it.nblk[X] > 0) {
              if (sc[X] > 0) ok = mbar_wait(&bar->s_free[X], (sc[X] - 1) & 1, status);
              if (!ok) break;
              tc_fence_after();
              issue_s(X, kc & 1);
              ++sc[X];
            }
            // Q_X is free once this item's last S_X MMA completes, so the
            // next item's Q loads during this item's last block
            if (it.nblk[X] <= 1) tc_commit(&bar->q_empty[X]);
          }
          if (!ok) break;
          tc_commit(&bar->k_empty[kc & 1]);
          ++kc;
        }
        for (int j = 0; j < it.n && ok && !*abort_flag; ++j) {
          bool v_ready = false, k_ready = false;
          for (int X = 0; X < 2 && ok; ++X) {
            if (j < it.nblk[X]) {
              ok = mbar_wait(&bar->p_full[X], pc[X] & 1, status);
              ++pc[X];
              // the first PV of an item overwrites O_X: the previous item's
              // epilogue must have read it
              if (ok && j == 0 && seq > 0) ok = mbar_wait(&bar->o_free[X], (seq - 1) & 1, status);
              if (ok && !v_ready) v_ready = ok = mbar_wait(&bar->v_full[vc & 1], (vc >> 1) & 1, status);
              if (!ok) break;
              tc_fence_after();
              issue_pv(X, vc & 1, j == 0);
            }
            if (X == 1) tc_commit(&bar->v_empty[vc & 1]);  // V free after PV_B(j)
            if (j + 1 < it.nblk[X]) {
              if (!k_ready) k_ready = ok = mbar_wait(&bar->k_full[kc & 1], (kc >> 1) & 1, status);
              if (ok) ok = mbar_wait(&bar->s_free[X], (sc[X] - 1) & 1, status);
              if (!ok) break;
              tc_fence_after();
              issue_s(X, kc & 1);
              ++sc[X];
              if (j + 2 == it.nblk[X]) tc_commit(&bar->q_empty[X]);
            }
          }
          ++vc;
          if (ok && j + 1 < it.n) {
            tc_commit(&bar->k_empty[kc & 1]);
            ++kc;
          }
        }
        if (!ok) break;
        // a tile with no block in this item (tile B past Sq) still takes
        // the previous item's epilogue hand-off, keeping the phases aligned
        for (int X = 0; X < 2 && ok; ++X)
          if (it.nblk[X] == 0 && seq > 0) ok = mbar_wait(&bar->o_free[X], (seq - 1) & 1, status);
      }
      if (!ok) *abort_flag = 1;
      tc_commit(&bar->drain);
      mbar_wait(&bar->drain, 0, status);
    }
  } else if (warp < W_PROD) {
    // --------------------------------------------------- softmax + epilogue
    // Eight warps per tile, two per TMEM lane quarter: warp (q, h) owns the
    // 16 rows 32q + 16h .. + 15 and reads them with the 16-lane shapes.
    // Thread t holds rows ra = base + t/4 and rb = ra + 8 and, of every
    // 8-column group k, columns 8k + 2(t%4) and + 1: a row is spread over
    // the 4 threads t/4 alike, so its max and sum are two shuffles and the
    // warps share nothing.  P goes back as 16-bit pairs with 16x128b, which
    // puts pair (8k + 2(t%4)) / 2 = 4k + t%4 of each row at that column:
    // the packed P in key order in S_X's first 64 columns.
    const int X = warp >> 3;                                  // query tile
    const int quarter = warp & 3;                             // TMEM lane quarter
    const int lane0 = quarter * 32 + ((warp >> 2) & 1) * 16;  // first row of this warp
    const int ra = lane0 + (lane >> 2);                       // rows of this thread (in the tile)
    const int cpair = 2 * (lane & 3);  // column offset within each 8-column group
    const uint32_t lane_base = (uint32_t)lane0 << 16;
    const uint32_t s_col = tmem + lane_base + C::TMEM_S + X * BN;
    const uint32_t o_col = tmem + lane_base + C::TMEM_O + X * D;
    auto quad_max = [](float v) {
      v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 1));
      return fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 2));
    };
    auto quad_sum = [](float v) {
      v += __shfl_xor_sync(0xffffffffu, v, 1);
      return v + __shfl_xor_sync(0xffffffffu, v, 2);
    };
    bool ok = true;
    uint32_t sc = 0;   // S_X blocks consumed
    uint32_t pvc = 0;  // PV_X MMAs before this item
    for (uint32_t seq = 0; ok; ++seq) {
      const int slot = seq & 1;
      if (!mbar_wait(&bar->sched_full[slot], (seq >> 1) & 1, status)) { ok = false; break; }
      const int w = bar->item[slot];
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar->sched_empty[slot]);
      if (w < 0) break;
      const Item it = decode_item<SPLIT>(w, pairs, BH, group, Sq, Skv, causal, sp);
      const uint32_t bh = it.bh;
      const uint32_t qa = it.q0 + X * BM + ra, qb = qa + 8;  // query indices
      // last visible key of each row, counted from the item's first key
      // block (a split item's second half starts at it.kb0 and always holds
      // a visible key, so the difference stays non-negative)
      const uint32_t lim_a = (causal && qa < Skv - 1 ? qa : Skv - 1) - it.kb0 * BN;
      const uint32_t lim_b = (causal && qb < Skv - 1 ? qb : Skv - 1) - it.kb0 * BN;
      const int nb = it.nblk[X];
      float m_a = -INFINITY, m_b = -INFINITY;  // reference maxima (scaled units)
      float l_a = 0.0f, l_b = 0.0f;            // this thread's share of the row sums
      for (int j = 0; j < nb && ok; ++j) {
        if (*abort_flag || !mbar_wait(&bar->s_full[X], sc & 1, status)) {
          ok = false;
          break;
        }
        ++sc;
        tc_fence_after();
        // r[32h + 4k + e]: columns 64h + 8k + cpair + (e & 1); e < 2 row
        // ra, e >= 2 row rb
        uint32_t r[64];
        tmem_ld_16x256b_x8(s_col, *reinterpret_cast<uint32_t(*)[32]>(&r[0]));
        tmem_ld_16x256b_x8(s_col + 64, *reinterpret_cast<uint32_t(*)[32]>(&r[32]));
        tc_wait_ld(*reinterpret_cast<uint32_t(*)[32]>(&r[0]));
        tc_wait_ld(*reinterpret_cast<uint32_t(*)[32]>(&r[32]));
        const uint32_t n0 = (uint32_t)j * BN;
        if (n0 + BN - 1 > (lim_a < lim_b ? lim_a : lim_b)) {
          // visible iff n0 + column <= lim
          const int rel_a = (int)lim_a - (int)n0 - cpair, rel_b = (int)lim_b - (int)n0 - cpair;
#pragma unroll
          for (int v = 0; v < 64; ++v) {
            const int col = 8 * (v >> 2) + (v & 1);  // column - cpair
            if (col > ((v & 2) ? rel_b : rel_a)) r[v] = __float_as_uint(-INFINITY);
          }
        }
        float mxa, mxb;
        {
          float a4[4], b4[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            a4[i] = __uint_as_float(r[4 * i]);
            b4[i] = __uint_as_float(r[4 * i + 2]);
          }
#pragma unroll
          for (int v = 0; v < 64; v += 4) {
            const int i = (v >> 2) & 3;
            a4[i] = max3(a4[i], __uint_as_float(r[v]), __uint_as_float(r[v + 1]));
            b4[i] = max3(b4[i], __uint_as_float(r[v + 2]), __uint_as_float(r[v + 3]));
          }
          mxa = quad_max(fmaxf(fmaxf(a4[0], a4[1]), fmaxf(a4[2], a4[3])));
          mxb = quad_max(fmaxf(fmaxf(b4[0], b4[1]), fmaxf(b4[2], b4[3])));
        }
        // the reference max only moves when it grows by more than 2^8
        // (log2 domain), so O is rescaled rarely
        const float na = fmaxf(m_a, mxa), nb_ = fmaxf(m_b, mxb);
        const bool mva = (na - m_a) * scale_log2 > 8.0f, mvb = (nb_ - m_b) * scale_log2 > 8.0f;
        const float ua = mva ? na : m_a, ub = mvb ? nb_ : m_b;
        const float alpha_a = mva ? fast_exp2((m_a - na) * scale_log2) : 1.0f;
        const float alpha_b = mvb ? fast_exp2((m_b - nb_) * scale_log2) : 1.0f;
        // P = exp2(S*c - m) as 16-bit pairs; the row sums add the fp32 values
        {
          const uint64_t sc2 = f2pack(scale_log2, scale_log2);
          const uint64_t nba = f2pack(-ua * scale_log2, -ua * scale_log2);
          const uint64_t nbb = f2pack(-ub * scale_log2, -ub * scale_log2);
          uint64_t acc_a = f2pack(0.0f, 0.0f), acc_b = f2pack(0.0f, 0.0f);
#pragma unroll
          for (int hf = 0; hf < 2; ++hf) {
            uint32_t pk[16];
#pragma unroll
            for (int k = 0; k < 8; ++k) {
              const int v = hf * 32 + 4 * k;
              float y0, y1, y2, y3, p0, p1, p2, p3;
              f2unpack(f2fma(f2pack(__uint_as_float(r[v]), __uint_as_float(r[v + 1])), sc2, nba), y0, y1);
              f2unpack(f2fma(f2pack(__uint_as_float(r[v + 2]), __uint_as_float(r[v + 3])), sc2, nbb), y2, y3);
              // of every 8 pairs, kEmuPairsPer8 take the FMA pipe
              if ((2 * (k & 3)) >= 8 - kEmuPairsPer8) {
                exp2_fma2(y0, y1, p0, p1);
                exp2_fma2(y2, y3, p2, p3);
              } else {
                p0 = fast_exp2(y0);  // MUFU
                p1 = fast_exp2(y1);
                p2 = fast_exp2(y2);
                p3 = fast_exp2(y3);
              }
              pk[2 * k] = pack2_16<F16>(p0, p1);
              pk[2 * k + 1] = pack2_16<F16>(p2, p3);
              acc_a = f2add(acc_a, f2pack(p0, p1));
              acc_b = f2add(acc_b, f2pack(p2, p3));
            }
            tmem_st_16x128b_x8(s_col + hf * 32, pk);
          }
          float a0, a1, b0, b1;
          f2unpack(acc_a, a0, a1);
          f2unpack(acc_b, b0, b1);
          l_a = l_a * alpha_a + (a0 + a1);
          l_b = l_b * alpha_b + (b0 + b1);
          m_a = ua;
          m_b = ub;
        }
        // Rescale O's rows whose max moved (after the exponentials, so S no
        // longer occupies registers).  PV_X(j-1) is complete: the commit
        // that signalled S_X(j) was issued after it.
        if (j > 0 && __any_sync(0xffffffffu, mva || mvb)) {
#pragma unroll 1
          for (int c = 0; c < D / 64; ++c) {
            uint32_t ro[32];
            tmem_ld_16x256b_x8(o_col + c * 64, ro);
            tc_wait_ld(ro);
#pragma unroll
            for (int v = 0; v < 32; ++v)
              ro[v] = __float_as_uint(__uint_as_float(ro[v]) * ((v & 2) ? alpha_b : alpha_a));
            tmem_st_16x256b_x8(o_col + c * 64, ro);
          }
        }
        tc_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&bar->s_free[X]);  // S_X may be overwritten
          mbar_arrive(&bar->p_full[X]);  // P_X ready for PV_X(j)
        }
      }
      if (!ok) break;
      // epilogue: O / l -> global, then hand O_X back to the MMA warp
      if constexpr (SPLIT) {
        if (nb > 0) {
          pvc += (uint32_t)nb;
          if (!mbar_wait(&bar->pv_done[X], (pvc - 1) & 1, status)) { ok = false; break; }
          tc_fence_after();
          const SplitRows rw{o_col, bh, Sq, qa, qb, cpair, lane, warp, scale_log2};
          if (!split_epilogue<D, F16>(rw, io, sp, (uint32_t)w, quad_sum(l_a), quad_sum(l_b), m_a,
                                      m_b, status)) {
            ok = false;
            break;
          }
        }
      } else if (nb > 0) {
        pvc += (uint32_t)nb;
        if (!mbar_wait(&bar->pv_done[X], (pvc - 1) & 1, status)) { ok = false; break; }
        tc_fence_after();
        const float la = quad_sum(l_a), lb = quad_sum(l_b);
        const float inv_a = la > 0.0f ? 1.0f / la : 0.0f, inv_b = lb > 0.0f ? 1.0f / lb : 0.0f;
        const bool va = qa < Sq, vb = qb < Sq;
        if (io.lse && (lane & 3) == 0) {
          if (va) io.lse[(size_t)bh * Sq + qa] = la > 0.0f ? m_a * scale_log2 + __log2f(la) : -INFINITY;
          if (vb) io.lse[(size_t)bh * Sq + qb] = lb > 0.0f ? m_b * scale_log2 + __log2f(lb) : -INFINITY;
        }
        // Each store instruction writes 8 rows x 4 threads x one column
        // pair: 8 whole 32-byte sectors for fp32.
#pragma unroll 1
        for (int c = 0; c < D / 64; ++c) {
          uint32_t ro[32];
          tmem_ld_16x256b_x8(o_col + c * 64, ro);
          tc_wait_ld(ro);
          if (io.out_f32) {
            float *oa = io.out_f32 + ((size_t)bh * Sq + qa) * D + c * 64 + cpair;
            float *ob = oa + 8 * (size_t)D;
#pragma unroll
            for (int k = 0; k < 8; ++k) {
              if (va)
                __stcs(reinterpret_cast<float2 *>(oa + 8 * k),
                       make_float2(__uint_as_float(ro[4 * k]) * inv_a, __uint_as_float(ro[4 * k + 1]) * inv_a));
              if (vb)
                __stcs(reinterpret_cast<float2 *>(ob + 8 * k),
                       make_float2(__uint_as_float(ro[4 * k + 2]) * inv_b, __uint_as_float(ro[4 * k + 3]) * inv_b));
            }
          }
          if (io.out_bf16) {
            const size_t head_col = (size_t)(bh % io.H) * D + c * 64 + cpair;
            uint16_t *oa = io.out_bf16 + ((size_t)(bh / io.H) * Sq + qa) * io.ldo + head_col;
            uint16_t *ob = oa + 8 * (size_t)io.ldo;
#pragma unroll
            for (int k = 0; k < 8; ++k) {
              if (va)
                *reinterpret_cast<uint32_t *>(oa + 8 * k) =
                    pack2_16<F16>(__uint_as_float(ro[4 * k]) * inv_a, __uint_as_float(ro[4 * k + 1]) * inv_a);
              if (vb)
                *reinterpret_cast<uint32_t *>(ob + 8 * k) =
                    pack2_16<F16>(__uint_as_float(ro[4 * k + 2]) * inv_b, __uint_as_float(ro[4 * k + 3]) * inv_b);
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar->o_free[X]);
    }
    if (!ok) *abort_flag = 1;
  }

  tc_fence_before();
  __syncthreads();
  if (warp == W_MMA) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

// head-major: dims {D, S, BH}; token-major (ld > 0): dims {D, H, B*S}, row pitch ld
int make_tmap_3d(BwppCudaCtx *ctx, CUtensorMap *map, const void *base, uint32_t D,
                 uint32_t S, uint32_t BH, uint32_t H, uint32_t ld, bool f16 = false) {
  bwpp_encode_tiled_fn enc = bwpp_get_encode_tiled();
  if (!enc) return bwpp_set_error(ctx, BWPP_CUDA_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[3], strides[2];
  cuuint32_t box[3];
  if (ld == 0) {
    dims[0] = D; dims[1] = S; dims[2] = BH;
    strides[0] = (cuuint64_t)D * 2; strides[1] = (cuuint64_t)S * D * 2;
    box[0] = 64; box[1] = 128; box[2] = 1;
  } else {
    dims[0] = D; dims[1] = H; dims[2] = (cuuint64_t)(BH / H) * S;
    strides[0] = (cuuint64_t)D * 2; strides[1] = (cuuint64_t)ld * 2;
    box[0] = 64; box[1] = 1; box[2] = 128;
  }
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(map, f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3,
                   const_cast<void *>(base), dims,
                   strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return bwpp_set_error(ctx, BWPP_CUDA_ERR_CUDA, "attention tensor map failed (%d)", (int)r);
  return BWPP_CUDA_OK;
}

bool g_attr_set[8][64] = {};

template <int D, bool F16, bool SPLIT>
int set_smem_attr(BwppCudaCtx *ctx) {
  const int di = (D == 128 ? 1 : 0) + (F16 ? 2 : 0) + (SPLIT ? 4 : 0);
  if (ctx->device < 64 && !g_attr_set[di][ctx->device]) {
    const int rc = bwpp_check_cuda(ctx,
                                   cudaFuncSetAttribute(attention_tc_kernel<D, F16, SPLIT>,
                                                        cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                        Cfg<D, F16>::SMEM),
                                   "attention smem attribute");
    if (rc) return rc;
    g_attr_set[di][ctx->device] = true;
  }
  return BWPP_CUDA_OK;
}

template <int D, bool F16 = false>
int launch(BwppCudaCtx *ctx, const uint16_t *q, const uint16_t *k, const uint16_t *v,
           uint32_t ld_in, uint32_t BH, uint32_t H, uint32_t Sq, uint32_t Skv, float scale,
           int causal, const AttnIO &io) {
  CUtensorMap tq, tk, tv;
  int rc = make_tmap_3d(ctx, &tq, q, D, Sq, BH, H, ld_in, F16);
  if (!rc) rc = make_tmap_3d(ctx, &tk, k, D, Skv, BH, H, ld_in, F16);
  if (!rc) rc = make_tmap_3d(ctx, &tv, v, D, Skv, BH, H, ld_in, F16);
  if (!rc) rc = set_smem_attr<D, F16, false>(ctx);
  if (rc) return rc;
  const uint32_t pairs = (Sq + 2 * BM - 1) / (2 * BM);
  const uint64_t items = (uint64_t)pairs * BH;
  if (items > 0x7fffffffull)
    return bwpp_set_error(ctx, BWPP_CUDA_ERR_UNSUPPORTED, "attention: too many work items");
  // persistent: one CTA per SM (at most one per item); the work counter
  // hands out the items after the first gridDim.x
  const uint64_t grid = items < (uint64_t)ctx->num_sms ? items : (uint64_t)ctx->num_sms;
  // heads per item group: their K / V (2 Skv D 16-bit values each) within
  // 32 MB.  Non-causal items are all alike, so there the order stays head by
  // head (group 1): the CTAs of a head then read each K / V block together,
  // 1.2% faster than the grouped order (which took causal at 32 heads per
  // GPU from 808 to 1001 TFLOP/s).
  const uint64_t kv_head = 4ull * Skv * D;
  const uint32_t group =
      causal ? (uint32_t)std::max<uint64_t>(1, std::min<uint64_t>(BH, (32ull << 20) / kv_head))
             : 1u;
  // Non-causal items are alike: a last round at most half full runs as a
  // second, split launch (AttnSplit) after the whole rounds
  AttnSplit sp{};
  uint64_t whole = items;
  {
    const uint64_t rem = items % grid;
    const uint32_t nkv = (Skv + BN - 1) / BN;
    float *parts = nullptr;
    size_t part_floats = 0, ncounters = 0;
    unsigned long long *counters = nullptr;
    uint32_t epoch = 0;
    if (!causal && grid == (uint64_t)ctx->num_sms && rem > 0 && 2 * rem <= grid && nkv >= 2 &&
        set_smem_attr<D, F16, true>(ctx) == BWPP_CUDA_OK &&
        bwpp_split_scratch(ctx, &parts, &part_floats, &counters, &ncounters, &epoch) &&
        rem * 16 * (uint64_t)Cfg<D, F16>::WARP_FLOATS <= part_floats && rem * 16 * 2 <= ncounters) {
      whole = items - rem;
      sp.first = (uint32_t)whole;
      sp.epoch = epoch;
      sp.partials = parts;
      sp.counters = counters;
    }
  }
  rc = bwpp_check_cuda(ctx, cudaMemsetAsync(ctx->sched_counter, 0, sizeof(int), ctx->stream),
                       "attention work counter");
  if (rc) return rc;
  attention_tc_kernel<D, F16, false><<<(unsigned)grid, THREADS, Cfg<D, F16>::SMEM, ctx->stream>>>(
      tq, tk, tv, io, BH, Sq, Skv, scale * 1.4426950408889634f, causal, pairs, group,
      (uint32_t)whole, sp, ctx->sched_counter, ctx->status_word);
  BWPP_LAUNCH_CHECK(ctx, "attention tcgen05");
  if (whole < items) {
    const uint32_t halves = (uint32_t)(2 * (items - whole));
    rc = bwpp_check_cuda(ctx, cudaMemsetAsync(ctx->sched_counter, 0, sizeof(int), ctx->stream),
                         "attention work counter");
    if (rc) return rc;
    const unsigned g2 = halves < (uint32_t)ctx->num_sms ? halves : (unsigned)ctx->num_sms;
    attention_tc_kernel<D, F16, true><<<g2, THREADS, Cfg<D, F16>::SMEM, ctx->stream>>>(
        tq, tk, tv, io, BH, Sq, Skv, scale * 1.4426950408889634f, causal, pairs, group, halves, sp,
        ctx->sched_counter, ctx->status_word);
    BWPP_LAUNCH_CHECK(ctx, "attention tcgen05 split tail");
  }
  return BWPP_CUDA_OK;
}

}  // namespace

// Contiguous [BH, S, D] bf16 inputs with D in {64, 128}: tensor-core path.
// Returns BWPP_CUDA_ERR_UNSUPPORTED for anything else (the caller then uses
// the CUDA-core kernel).
int bwpp_attention_tc_launch(BwppCudaCtx *ctx, const uint16_t *q,
                             const uint16_t *k, const uint16_t *v, float *o,
                             uint32_t BH, uint32_t Sq, uint32_t Skv, uint32_t D,
                             float scale, int causal) {
  auto al = [](const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  // the lazy running max assumes a positive softmax scale
  if (!al(q) || !al(k) || !al(v) || !al(o) || Skv == 0 || !(scale > 0.0f))
    return BWPP_CUDA_ERR_UNSUPPORTED;
  AttnIO io{o, nullptr, 0, nullptr, 0, 1};
  if (D == 128) return launch<128>(ctx, q, k, v, 0, BH, 1, Sq, Skv, scale, causal, io);
  if (D == 64) return launch<64>(ctx, q, k, v, 0, BH, 1, Sq, Skv, scale, causal, io);
  return BWPP_CUDA_ERR_UNSUPPORTED;
}

// The half ABI: contiguous [BH, S, D] f16 inputs, D in {64, 128}, f16
// head-major output [BH, Sq, D].  Returns BWPP_CUDA_ERR_UNSUPPORTED for
// anything else.
int bwpp_attention_tc_launch_f16(BwppCudaCtx *ctx, const uint16_t *q, const uint16_t *k,
                                 const uint16_t *v, uint16_t *o, uint32_t BH, uint32_t Sq,
                                 uint32_t Skv, uint32_t D, float scale, int causal) {
  auto al = [](const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  if (!al(q) || !al(k) || !al(v) || !al(o) || Skv == 0 || !(scale > 0.0f))
    return BWPP_CUDA_ERR_UNSUPPORTED;
  // head-major 16-bit output: row bh * Sq + m (H = 1 in the output map), pitch D
  AttnIO io{nullptr, o, D, nullptr, 0, 1};
  if (D == 128) return launch<128, true>(ctx, q, k, v, 0, BH, 1, Sq, Skv, scale, causal, io);
  if (D == 64) return launch<64, true>(ctx, q, k, v, 0, BH, 1, Sq, Skv, scale, causal, io);
  return BWPP_CUDA_ERR_UNSUPPORTED;
}

// Training-step form: token-major bf16 inputs (row pitch ld_in, head h at
// column h*D), bf16 token-major output (pitch ldo) and the per-query base-2
// log-sum-exp [B*H, S] the backward pass needs.  Sq == Skv == S.
int bwpp_attention_fwd_train(BwppCudaCtx *ctx, const uint16_t *q, const uint16_t *k,
                             const uint16_t *v, uint32_t ld_in, uint32_t B, uint32_t H,
                             uint32_t S, uint32_t D, float scale, int causal, uint16_t *o,
                             uint32_t ldo, float *lse) {
  if (D != 128 || !(scale > 0.0f) || S == 0 || (ld_in % 8) || (ldo % 8))
    return bwpp_set_error(ctx, BWPP_CUDA_ERR_UNSUPPORTED, "attention train: D=128 only");
  AttnIO io{nullptr, o, ldo, lse, 1, H};
  return launch<128>(ctx, q, k, v, ld_in, B * H, H, S, S, scale, causal, io);
}
