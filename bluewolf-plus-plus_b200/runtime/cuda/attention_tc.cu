// Attention forward on sm_100a tensor cores, single pass with online softmax.
//
//   O[bh, m, :] = sum_n softmax_n(scale * q_m . k_n [n <= m if causal]) v_n
//
// One CTA owns 256 query rows of one (batch, head) as two 128-row tiles A and
// B that ping-pong: while the softmax warps of one tile turn its S into P, the
// tensor core works on the other tile.  Per 128-key block j:
//   S_X = Q_X K_j^T          tcgen05 M=128 N=128 K=16 (Q, K K-major, bf16)
//   P_X = exp2(S_X*c - m)    softmax warps, two threads per row (64 keys
//                            each); P as bf16 pairs written back into S_X's
//                            TMEM columns
//   O_X += P_X V_j           tcgen05 M=128 N=D K=16, A = P from TMEM,
//                            B = V MN-major from smem
// S_A, S_B, O_A, O_B live in TMEM (4 x 128 columns for D = 128).  The running
// max only moves when it grows by more than 2^8 (log2 domain), so O is
// rescaled (tcgen05.ld / st) rarely; P <= 256 stays exact enough in bf16.
// The softmax arithmetic uses paired fp32 lanes (fma/add .f32x2) and 3-input
// max to halve its instruction count; CTAs are ordered head-major so one
// head's K / V is read from DRAM once and shared through L2.
//
// Warp roles (576 threads): warps 0-7 softmax of tile A, warps 8-15
// softmax of tile B (warp w reads TMEM lanes 32*(w%4)..; two warps per lane
// quarter split the keys and O columns), warp 16 TMA producer (Q once; K
// and V double-buffered, 3-D tensor maps so ragged S zero-fills per head),
// warp 17 TMEM allocator + single-thread MMA issuer.
// MMA issue order per block: PV_A(j), S_A(j+1), PV_B(j), S_B(j+1), so one
// tile's softmax always overlaps the other tile's MMAs.
//
// Every wait is bounded (BWPP_WAIT_LIMIT_NS); on expiry the kernel records
// BWPP_CUDA_ERR_TIMEOUT, unwinds, frees TMEM and returns.
#include "attention_common.cuh"

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
  // epilogue staging: 32 rows x 128 B per softmax warp
  static constexpr int OFF_STAGE = 6 * TILE;
  static constexpr int STAGE_WARP = 32 * 64;
  static constexpr int OFF_BAR = OFF_STAGE + 16 * STAGE_WARP;
  static constexpr int SMEM = OFF_BAR + 512 + 1024;
  static constexpr uint32_t TMEM_S = 0;        // S_A at 0, S_B at 128
  static constexpr uint32_t TMEM_O = 2 * BN;   // O_A at 256, O_B at 256 + D
  static constexpr uint32_t TMEM_COLS = 512;
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
  uint64_t pair[8];  // the two halves of a tile's lane quarter: one phase per exchange
  uint64_t drain;
  int item[2];
  uint32_t tmem;
  int abort_flag;
};
static_assert(sizeof(Bars) <= 512, "barrier block");

// Work item w (in the order CTAs take them): head bh = w / pairs, query
// pair pairs - 1 - w % pairs of that head (the heaviest causal pair first),
// i.e. rows q0 .. q0 + 255 as tiles A and B.
struct Item {
  uint32_t bh, q0;
  int nblk[2], n;
};

__device__ __forceinline__ Item decode_item(int w, uint32_t pairs, uint32_t Sq, uint32_t Skv,
                                            int causal) {
  Item it;
  it.bh = (uint32_t)w / pairs;
  it.q0 = (pairs - 1 - (uint32_t)w % pairs) * 2 * BM;
  it.nblk[0] = blocks_for(it.q0, Sq, Skv, causal);
  it.nblk[1] = blocks_for(it.q0 + BM, Sq, Skv, causal);
  it.n = max(it.nblk[0], it.nblk[1]);
  return it;
}

// Persistent: one CTA per SM takes work items (256 query rows of one head)
// until none is left: its first item is blockIdx.x, the next ones come from
// the context's work counter (items gridDim.x, gridDim.x + 1, ... in
// head-major order, so the CTAs running together share a few heads' K / V in
// L2, and a CTA that drew a short causal item simply draws again).  The
// producer publishes each item id through a two-slot ring (sched_full /
// sched_empty); every role walks the same item sequence.  Across items the
// K / V ring keeps streaming, the next item's Q is loaded as soon as the
// last S MMAs of the current item release Q (q_empty), and the next item's
// S MMAs run while the softmax warps are still in the previous epilogue; its
// first PV waits for that epilogue to read O (o_free).  All barrier phases
// are running counters over the CTA's whole item sequence.
template <int D, bool F16>
__global__ void __launch_bounds__(THREADS, 1)
    attention_tc_kernel(const __grid_constant__ CUtensorMap tmQ,
                        const __grid_constant__ CUtensorMap tmK,
                        const __grid_constant__ CUtensorMap tmV,
                        const AttnIO io, uint32_t BH, uint32_t Sq,
                        uint32_t Skv, float scale_log2, int causal,
                        uint32_t pairs, int *sched, int *status) {
  using C = Cfg<D, F16>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t *smem = smem_raw + ((1024u - (raw & 1023u)) & 1023u);
  Bars *bar = reinterpret_cast<Bars *>(smem + C::OFF_BAR);
  volatile int *abort_flag = &bar->abort_flag;
  const int total = (int)(pairs * BH);

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
    for (int p = 0; p < 8; ++p) mbar_init(&bar->pair[p], 2);
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
        const Item it = decode_item(w, pairs, Sq, Skv, causal);
        // K(0) first (its slot frees with the previous item's last S MMAs),
        // then both Q tiles.  Every item has at least one block (its first
        // row is below Sq and Skv >= 1).
        {
          const int s = kc & 1;
          if (!mbar_wait(&bar->k_empty[s], ((kc >> 1) & 1) ^ 1, status)) { ok = false; break; }
          mbar_arrive_expect_tx(&bar->k_full[s], C::TILE);
          load_rows<C::BOXES>(smem + C::OFF_K + s * C::TILE, &tmK, &bar->k_full[s], io, it.bh, Skv, 0);
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
                                Skv, (j + 1) * BN);
            ++kc;
          }
          const int vs = vc & 1;
          if (!mbar_wait(&bar->v_empty[vs], ((vc >> 1) & 1) ^ 1, status)) { ok = false; break; }
          mbar_arrive_expect_tx(&bar->v_full[vs], C::TILE);
          load_rows<C::BOXES>(smem + C::OFF_V + vs * C::TILE, &tmV, &bar->v_full[vs], io, it.bh, Skv,
                              j * BN);
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
      // O_X (+)= P_X V with P_X read from TMEM (16-bit pairs: keys
      // [64h, 64h + 64) in S_X columns [64h, 64h + 32), 16 keys = 8 columns
      // per MMA) and V from smem slot vslot
      auto issue_pv = [&](int X, int vslot, bool first) {
        const uint64_t vd = desc_add(dv, (uint32_t)vslot * C::TILE);
        const uint32_t pt = tmem + C::TMEM_S + X * BN;
        const uint32_t d_tmem = tmem + C::TMEM_O + X * D;
#pragma unroll
        for (int ks = 0; ks < BN / 16; ++ks)
          tc_mma_f16_ts(d_tmem, pt + (ks >> 2) * 64 + (ks & 3) * 8, desc_add(vd, ks * 2048), C::IDESC_PV,
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
        const Item it = decode_item(w, pairs, Sq, Skv, causal);
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
    // Two warps share each 32-row lane quarter of a tile: half h takes keys
    // [64h, 64h + 64) of every block (and writes their P into the first 32
    // of its own 64 S columns) and O columns [h D/2, (h+1) D/2).  The halves
    // agree on the row's reference max through shared memory (one
    // mbarrier-paced exchange per block); their row sums meet once, in the
    // epilogue.
    const int sw = warp;                  // softmax warp 0..15
    const int X = sw >> 3;                // query tile
    const int h = (sw >> 2) & 1;          // key / O-column half
    const int quarter = warp & 3;         // TMEM lanes 32*quarter ..
    const int row = quarter * 32 + lane;
    uint64_t *pair_bar = &bar->pair[X * 4 + quarter];
    const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
    const uint32_t s_col = tmem + lane_base + C::TMEM_S + X * BN + h * 64;
    const uint32_t o_col = tmem + lane_base + C::TMEM_O + X * D + h * (D / 2);
    // per-warp 2 KB: epilogue staging, and (outside the epilogue) two
    // 32-float exchange slots the partner half reads
    uint8_t *stage_raw = smem + C::OFF_STAGE + sw * C::STAGE_WARP;
    const float *peer_xch =
        reinterpret_cast<const float *>(smem + C::OFF_STAGE + (sw ^ 4) * C::STAGE_WARP);
    bool ok = true;
    uint32_t xc = 0;  // exchanges so far (slot and phase parity = xc & 1)
    // Max or sum of v over the two halves of this row.  Slots are
    // double-buffered: a warp rewrites a slot two exchanges later, and the
    // exchange in between completes only after the partner arrived for it,
    // i.e. after it read the slot.  The wait is bounded like every other:
    // on expiry ok turns false and the warp unwinds.
    auto pair_sync = [&]() {
      __syncwarp();
      if (lane == 0) mbar_arrive(pair_bar);
      const bool done = mbar_wait(pair_bar, xc & 1, status);
      ++xc;
      return done;
    };
    auto pair_combine = [&](float v, bool sum) {
      reinterpret_cast<float *>(stage_raw)[(xc & 1) * 32 + lane] = v;
      const int slot = (int)(xc & 1) * 32;
      if (!pair_sync()) ok = false;
      const float o = peer_xch[slot + lane];
      return sum ? v + o : fmaxf(v, o);
    };
    uint32_t sc = 0;   // S_X blocks consumed
    uint32_t pvc = 0;  // PV_X MMAs before this item
    for (uint32_t seq = 0; ok; ++seq) {
      const int slot = seq & 1;
      if (!mbar_wait(&bar->sched_full[slot], (seq >> 1) & 1, status)) { ok = false; break; }
      const int w = bar->item[slot];
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar->sched_empty[slot]);
      if (w < 0) break;
      const Item it = decode_item(w, pairs, Sq, Skv, causal);
      const uint32_t bh = it.bh;
      const uint32_t m_row = it.q0 + X * BM + row;  // query index
      const int nb = it.nblk[X];
      float m_run = -INFINITY, l_run = 0.0f;
      for (int j = 0; j < nb && ok; ++j) {
        if (*abort_flag || !mbar_wait(&bar->s_full[X], sc & 1, status)) {
          ok = false;
          break;
        }
        ++sc;
        tc_fence_after();
        uint32_t r[64];
        tmem_ld_32x32b_x32(s_col, *reinterpret_cast<uint32_t(*)[32]>(&r[0]));
        tmem_ld_32x32b_x32(s_col + 32, *reinterpret_cast<uint32_t(*)[32]>(&r[32]));
        tc_wait_ld(*reinterpret_cast<uint32_t(*)[32]>(&r[0]));
        tc_wait_ld(*reinterpret_cast<uint32_t(*)[32]>(&r[32]));
        // keys n0 + i; blocks that need no mask take a branch-free path,
        // masked ones compare each key with one limit
        const uint32_t n0 = (uint32_t)j * BN + h * 64;
        uint32_t lim = Skv - 1;                       // last visible key
        if (causal && m_row < lim) lim = m_row;
        if (n0 + 63 > lim) {
          const int lim_rel = (int)lim - (int)n0;     // visible iff index <= lim_rel
#pragma unroll
          for (int i = 0; i < 64; ++i)
            if (i > lim_rel) r[i] = __float_as_uint(-INFINITY);
        }
        auto block_max = [&]() {
          float m8[8];
#pragma unroll
          for (int k = 0; k < 8; ++k) m8[k] = max3(__uint_as_float(r[k]), __uint_as_float(r[8 + k]),
                                                   __uint_as_float(r[16 + k]));
#pragma unroll
          for (int i = 24; i < 64; i += 16)
#pragma unroll
            for (int k = 0; k < 8; ++k)
              m8[k] = max3(m8[k], __uint_as_float(r[i + k]), __uint_as_float(r[i + 8 + k]));
          return fmaxf(fmaxf(max3(m8[0], m8[1], m8[2]), max3(m8[3], m8[4], m8[5])),
                       fmaxf(m8[6], m8[7]));
        };
        // the row's max over both halves; the reference max only moves when
        // it grows by more than 2^8 (log2 domain), so O is rescaled rarely
        const float m_new = fmaxf(m_run, pair_combine(block_max(), false));
        if (!ok) break;
        const bool move = (m_new - m_run) * scale_log2 > 8.0f;
        const float m_use = move ? m_new : m_run;
        const float alpha = move ? fast_exp2((m_run - m_new) * scale_log2) : 1.0f;
        // P = exp2(S*c - m) as 16-bit pairs into this half's first 32 S
        // columns (already read); the row sum adds the fp32 values
        {
          const uint64_t sc2 = f2pack(scale_log2, scale_log2);
          const float mb = m_use * scale_log2;
          const uint64_t nb2 = f2pack(-mb, -mb);
          uint64_t acc2[2] = {f2pack(0.0f, 0.0f), f2pack(0.0f, 0.0f)};
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            uint32_t pk[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const int e = c * 16 + 2 * i;
              float y0, y1, p0, p1;
              f2unpack(f2fma(f2pack(__uint_as_float(r[e]), __uint_as_float(r[e + 1])), sc2, nb2), y0, y1);
              if ((i & 7) >= 8 - kEmuPairsPer8) {
                exp2_fma2(y0, y1, p0, p1);  // FMA pipe
              } else {
                p0 = fast_exp2(y0);  // MUFU
                p1 = fast_exp2(y1);
              }
              pk[i] = pack2_16<F16>(p0, p1);
              acc2[i & 1] = f2add(acc2[i & 1], f2pack(p0, p1));
            }
            tmem_st_32x32b_x8(s_col + c * 8, pk);
          }
          float a, b, c2, d;
          f2unpack(acc2[0], a, b);
          f2unpack(acc2[1], c2, d);
          l_run = l_run * alpha + ((a + b) + (c2 + d));
          m_run = m_use;
        }
        // Rescale this half's O columns when a row's max moved (after the
        // exponentials, so S no longer occupies registers).  PV_X(j-1) is
        // complete: the commit that signalled S_X(j) was issued after it.
        if (j > 0 && __any_sync(0xffffffffu, move)) {
#pragma unroll 1
          for (int c = 0; c < D / 32; ++c) {
            uint32_t ro[16];
            tmem_ld_32x32b_x16(o_col + c * 16, ro);
            tc_wait_ld16(ro);
#pragma unroll
            for (int i = 0; i < 16; ++i) ro[i] = __float_as_uint(__uint_as_float(ro[i]) * alpha);
            tmem_st_32x32b_x16(o_col + c * 16, ro);
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
      if (nb > 0) {
        pvc += (uint32_t)nb;
        if (!mbar_wait(&bar->pv_done[X], (pvc - 1) & 1, status)) { ok = false; break; }
        tc_fence_after();
        const float l_tot = pair_combine(l_run, true);
        // the partner has read this warp's slot before staging overwrites it
        if (!ok || !pair_sync()) { ok = false; break; }
        const float inv = l_tot > 0.0f ? 1.0f / l_tot : 0.0f;
        if (h == 0 && m_row < Sq && io.lse)
          io.lse[(size_t)bh * Sq + m_row] =
              l_tot > 0.0f ? m_run * scale_log2 + __log2f(l_tot) : -INFINITY;
        // O leaves through shared memory: each thread stages a 64-byte
        // piece of its row (16-byte parts XOR-swizzled by row so the
        // row-per-thread writes and the 8-rows-per-instruction reads both
        // hit distinct banks); every store instruction then writes 8 rows x
        // 64 contiguous bytes instead of 32 scattered 16-byte pieces.
        uint4 *stage = reinterpret_cast<uint4 *>(stage_raw);
        const uint32_t row0 = it.q0 + X * BM + quarter * 32;  // this warp's first row
        const int part = lane & 3;
        auto put = [&](int i, uint4 v) { stage[lane * 4 + (i ^ ((lane >> 1) & 3))] = v; };
        auto flush = [&](auto &&row_ptr) {
          __syncwarp();
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const int rr = 8 * k + (lane >> 2);
            const uint4 val = stage[rr * 4 + (part ^ ((rr >> 1) & 3))];
            if (row0 + rr < Sq) *(row_ptr(row0 + rr) + part) = val;
          }
          __syncwarp();
        };
        const uint32_t col0 = h * (D / 2);  // first O column of this half
        if (io.out_f32) {
#pragma unroll 1
          for (int c = 0; c < D / 64; ++c) {
            uint32_t r[32];
            tmem_ld_32x32b_x32(o_col + c * 32, r);
            tc_wait_ld(r);
#pragma unroll
            for (int half16 = 0; half16 < 2; ++half16) {
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                const int e = half16 * 16 + 4 * i;
                put(i, make_uint4(__float_as_uint(__uint_as_float(r[e]) * inv),
                                  __float_as_uint(__uint_as_float(r[e + 1]) * inv),
                                  __float_as_uint(__uint_as_float(r[e + 2]) * inv),
                                  __float_as_uint(__uint_as_float(r[e + 3]) * inv)));
              }
              flush([&](uint32_t m) {
                return reinterpret_cast<uint4 *>(io.out_f32 + ((size_t)bh * Sq + m) * D + col0 +
                                                 c * 32 + half16 * 16);
              });
            }
          }
        }
        if (io.out_bf16) {
#pragma unroll 1
          for (int c = 0; c < D / 64; ++c) {
            uint32_t r[32];
            tmem_ld_32x32b_x32(o_col + c * 32, r);
            tc_wait_ld(r);
#pragma unroll
            for (int i = 0; i < 4; ++i)
              put(i, make_uint4(
                  pack2_16<F16>(__uint_as_float(r[8 * i]) * inv, __uint_as_float(r[8 * i + 1]) * inv),
                  pack2_16<F16>(__uint_as_float(r[8 * i + 2]) * inv, __uint_as_float(r[8 * i + 3]) * inv),
                  pack2_16<F16>(__uint_as_float(r[8 * i + 4]) * inv, __uint_as_float(r[8 * i + 5]) * inv),
                  pack2_16<F16>(__uint_as_float(r[8 * i + 6]) * inv, __uint_as_float(r[8 * i + 7]) * inv)));
            flush([&](uint32_t m) {
              return reinterpret_cast<uint4 *>(io.out_bf16 + ((size_t)(bh / io.H) * Sq + m) * io.ldo +
                                               (size_t)(bh % io.H) * D + col0 + c * 32);
            });
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

bool g_attr_set[4][64] = {};

template <int D, bool F16 = false>
int launch(BwppCudaCtx *ctx, const uint16_t *q, const uint16_t *k, const uint16_t *v,
           uint32_t ld_in, uint32_t BH, uint32_t H, uint32_t Sq, uint32_t Skv, float scale,
           int causal, const AttnIO &io) {
  CUtensorMap tq, tk, tv;
  int rc = make_tmap_3d(ctx, &tq, q, D, Sq, BH, H, ld_in, F16);
  if (!rc) rc = make_tmap_3d(ctx, &tk, k, D, Skv, BH, H, ld_in, F16);
  if (!rc) rc = make_tmap_3d(ctx, &tv, v, D, Skv, BH, H, ld_in, F16);
  if (rc) return rc;
  const int di = (D == 128 ? 1 : 0) + (F16 ? 2 : 0);
  if (ctx->device < 64 && !g_attr_set[di][ctx->device]) {
    rc = bwpp_check_cuda(ctx,
                         cudaFuncSetAttribute(attention_tc_kernel<D, F16>,
                                              cudaFuncAttributeMaxDynamicSharedMemorySize,
                                              Cfg<D, F16>::SMEM),
                         "attention smem attribute");
    if (rc) return rc;
    g_attr_set[di][ctx->device] = true;
  }
  const uint32_t pairs = (Sq + 2 * BM - 1) / (2 * BM);
  const uint64_t items = (uint64_t)pairs * BH;
  if (items > 0x7fffffffull)
    return bwpp_set_error(ctx, BWPP_CUDA_ERR_UNSUPPORTED, "attention: too many work items");
  // persistent: one CTA per SM (at most one per item); the work counter
  // hands out the items after the first gridDim.x
  const uint64_t grid = items < (uint64_t)ctx->num_sms ? items : (uint64_t)ctx->num_sms;
  rc = bwpp_check_cuda(ctx, cudaMemsetAsync(ctx->sched_counter, 0, sizeof(int), ctx->stream),
                       "attention work counter");
  if (rc) return rc;
  attention_tc_kernel<D, F16><<<(unsigned)grid, THREADS, Cfg<D, F16>::SMEM, ctx->stream>>>(
      tq, tk, tv, io, BH, Sq, Skv, scale * 1.4426950408889634f, causal, pairs,
      ctx->sched_counter, ctx->status_word);
  BWPP_LAUNCH_CHECK(ctx, "attention tcgen05");
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
