// Attention backward on sm_100a tensor cores (training step of the tiny_model
// config).  With s = scale * q.k, P = softmax(s) recomputed from the forward's
// base-2 log-sum-exp (P = exp2(q.k * scale*log2e - lse2)), dO the upstream
// gradient and delta = rowsum(dO * O):
//   dP = dO V^T,  dS = P * (dP - delta),
//   dQ = scale * dS K,  dK = scale * dS^T Q,  dV = P^T dO
// Two persistent kernels (one CTA per SM), no atomics:
//   bwd_dq_kernel    items (head, 128 query rows); loops over 128-key blocks:
//                    S = Q K^T and dP = dO V^T into TMEM, the softmax warps
//                    (one query row per thread) form dS -> smem bf16,
//                    dQ += dS K accumulates in TMEM.
//   bwd_dkdv_kernel  items (head, 128 keys) from a work counter; loops over
//                    128-row query tiles: S^T = K Q^T and dP^T = V dO^T into
//                    TMEM, the softmax warps (one key per thread) form P^T and
//                    dS^T as bf16 in TMEM, dV += P^T dO and dK += dS^T Q
//                    accumulate in TMEM.
// Warps: 0 TMA producer, 1 TMEM allocator + MMA issuer, 2-9 softmax (two
// per TMEM lane quarter, each taking half of a block's 128 columns: with one
// warp per quarter the exp2 / dS / pack work left the tensor core idle most
// of the time).  All waits are bounded (BWPP_WAIT_LIMIT_NS) as in the
// forward kernel.
// Operands reuse the forward's smem layouts: a 128-row tile is two 64-column
// 128-byte-swizzle boxes; read K-major for S-type products and MN-major when
// it is the B of dQ / dK / dV.
#include "attention_common.cuh"

#include <type_traits>

namespace {

using namespace bwpp_attn;

constexpr int D = 128;
constexpr int TILE = 2 * BOX;  // 128 rows x 128 bf16
constexpr int SM_WARPS = 8;  // softmax warps: two per TMEM lane quarter, half the columns each
constexpr int THREADS = 64 + 32 * SM_WARPS;
constexpr uint32_t IDESC_KK = make_idesc_bf16_f32(128, 128, 0, 0);  // S-type
constexpr uint32_t IDESC_KM = make_idesc_bf16_f32(128, D, 0, 1);    // dQ / dK / dV

struct BwdIO {
  uint16_t *d0, *d1;  // dq kernel: dQ; dkdv kernel: dK (d0), dV (d1)
  uint32_t ldd;       // token-major pitch of the outputs
  const float *lse;   // [B*H, Sq]
  const float *delta; // [B*H, Sq]
  AttnIO in;          // input layout (tok / H)
  int tma_out;        // dkdv kernel: dK / dV leave through the tmDK / tmDV maps
};

// The issue loops below build each descriptor's low word once and step it by
// (offset >> 4): the issuing thread shares its SM sub-partition with two busy
// softmax warps, so every instruction it saves shortens the MMA stream.
// (SBO 1024 and the 128-byte swizzle for both K- and MN-major boxes; the
// LBO, 16 resp. BOX bytes, sits in the low word)
constexpr uint32_t HI_SW = smem_desc_hi(1024, BWPP_SWIZZLE_128B);

__device__ __forceinline__ void mma_kk(uint32_t d, uint32_t a, uint32_t b) {
  // D(128 x 128) = A(128 x D) B(128 x D)^T, both K-major
  const uint32_t alo = smem_desc_lo(a, 16), blo = smem_desc_lo(b, 16);
#pragma unroll
  for (int ks = 0; ks < D / 16; ++ks) {
    const uint32_t off = ((ks >> 2) * BOX + (ks & 3) * 32) >> 4;
    tc_mma_f16_ss_w(d, alo + off, HI_SW, blo + off, HI_SW, IDESC_KK, ks > 0 ? 1u : 0u);
  }
}

__device__ __forceinline__ void mma_km(uint32_t d, uint32_t a, uint32_t b, bool acc) {
  // D(128 x D) += A(128 x 128, K-major) B(128 x D, MN-major)
  const uint32_t alo = smem_desc_lo(a, 16), blo = smem_desc_lo(b, BOX);
#pragma unroll
  for (int ks = 0; ks < 128 / 16; ++ks) {
    const uint32_t aoff = ((ks >> 2) * BOX + (ks & 3) * 32) >> 4;
    tc_mma_f16_ss_w(d, alo + aoff, HI_SW, blo + ((ks * 2048) >> 4), HI_SW, IDESC_KM,
                    (acc || ks > 0) ? 1u : 0u);
  }
}

// Writes a row of 128 fp32 TMEM values (x scale) as bf16 to global memory.
__device__ __forceinline__ void store_row_bf16(uint32_t taddr, uint16_t *dst, float scale,
                                               bool valid, int half) {
#pragma unroll 1
  for (int c = half * (D / 64); c < (half + 1) * (D / 64); ++c) {
    uint32_t r[32];
    tmem_ld_32x32b_x32(taddr + c * 32, r);
    tc_wait_ld(r);
    if (valid) {
#pragma unroll
      for (int i = 0; i < 4; ++i)
        *reinterpret_cast<uint4 *>(dst + c * 32 + 8 * i) = make_uint4(
            pack_bf16(__uint_as_float(r[8 * i]) * scale, __uint_as_float(r[8 * i + 1]) * scale),
            pack_bf16(__uint_as_float(r[8 * i + 2]) * scale, __uint_as_float(r[8 * i + 3]) * scale),
            pack_bf16(__uint_as_float(r[8 * i + 4]) * scale, __uint_as_float(r[8 * i + 5]) * scale),
            pack_bf16(__uint_as_float(r[8 * i + 6]) * scale, __uint_as_float(r[8 * i + 7]) * scale));
    }
  }
}

// Converts this thread's 64 fp32 TMEM columns at taddr (x scale) to bf16 and
// writes them as row `row` of the 64-column box `half` of a 128-byte-swizzle
// tile (both 32-column loads in flight before one wait).
__device__ __forceinline__ void stage_row_bf16(uint32_t taddr, uint8_t *tile, int row, int half,
                                               float scale) {
  uint32_t r[2][32];
  tmem_ld_32x32b_x32(taddr, r[0]);
  tmem_ld_32x32b_x32(taddr + 32, r[1]);
  tc_wait_ld(r[0]);
  tc_wait_ld(r[1]);
#pragma unroll
  for (int cc = 0; cc < 2; ++cc) {
    uint32_t pk[16];
#pragma unroll
    for (int i = 0; i < 16; ++i)
      pk[i] = pack_bf16(__uint_as_float(r[cc][2 * i]) * scale, __uint_as_float(r[cc][2 * i + 1]) * scale);
    store_swizzled_chunk(tile, row, half * 2 + cc, pk);
  }
}

// ---------------------------------------------------------------------------
// dQ
// ---------------------------------------------------------------------------
// K in a ring of three slots (K(j) is read by S(j) and, a block later, by
// dQ(j)); V in one slot (V(j) is read by dP(j) alone, and V(j+1) loads while
// dQ(j) runs).
constexpr int K_SLOTS = 3;
constexpr int Q_OFF_Q = 0, Q_OFF_DO = TILE, Q_OFF_K = 2 * TILE, Q_OFF_V = (2 + K_SLOTS) * TILE,
              Q_OFF_DS = (3 + K_SLOTS) * TILE, Q_OFF_BAR = (4 + K_SLOTS) * TILE;
constexpr int Q_SMEM = Q_OFF_BAR + 256 + 1024;
static_assert(Q_SMEM <= 232448, "dq smem");

// Pipeline of bwd_dq_kernel, per key block j (K in a ring of three, V in one
// slot):
//   MMA:     S(j+1) once S(j) is read | dP(j+1) once dS(j) is in smem (dP(j)
//            was read for it) | dQ(j)
//   softmax: S(j) into registers -> s_read; P(j) = exp2(...);
//            dS(j) = P (dP(j) - delta) -> smem -> ds_full
// so S(j+1) runs on the tensor core while the softmax works on block j, and
// dP(j+1) is ready when dQ(j) has read dS(j) and the smem tile is free again.
// Persistent: one CTA per SM walks the (head, 128-row tile) items in rounds
// (q_pick: a round is gridDim.x consecutive items of a few heads, every other
// round taken in reverse so heavy and light tiles even out).  Block-level
// barrier phases follow a block counter that
// runs on across items.  The two dQ accumulators (TMEM columns 256, 384)
// alternate between items, so an item's dQ store overlaps the next item's
// MMAs; Q / dO are released after an item's last S / dP MMA, so the next
// item's loads overlap its tail.
struct QBars {
  uint64_t qd_full, qd_empty, k_full[K_SLOTS], k_empty[K_SLOTS], v_full, v_empty, s_full, dp_full,
      s_read, ds_full, dq_done,
      acc_free[2], drain, out_staged, ds_free;
  uint32_t tmem;
  int abort_flag;
};
static_assert(sizeof(QBars) <= 256, "dq barriers");

struct QItem {
  uint32_t bh, q0;
  int n;
};

// Item i: head i / qtiles, its tiles heaviest (last) first.
__device__ __forceinline__ QItem q_item(uint32_t i, uint32_t BH, uint32_t qtiles, uint32_t Sq,
                                        uint32_t Skv, int causal) {
  QItem it;
  it.bh = i / qtiles;
  it.q0 = (qtiles - 1 - i % qtiles) * BM;
  it.n = blocks_for(it.q0, Sq, Skv, causal);
  return it;
}

// The item CTA c takes in its round j: rounds of gridDim.x consecutive items
// (a few heads, whose K / V the CTAs of a round share in L2), every other
// round walked backwards so that the heavy and light positions of a head's
// tiles even out over each CTA's rounds.  Past the last item: >= items.
__device__ __forceinline__ uint32_t q_pick(uint32_t rnd) {
  return rnd * gridDim.x + ((rnd & 1) ? gridDim.x - 1 - blockIdx.x : blockIdx.x);
}

__global__ void __launch_bounds__(THREADS, 1)
    bwd_dq_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                  const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmDO,
                  const __grid_constant__ CUtensorMap tmDQ, const BwdIO io, uint32_t BH, uint32_t Sq, uint32_t Skv, float scale,
                  float scale_log2, int causal, uint32_t qtiles, int *status) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t *smem = smem_raw + ((1024u - (raw & 1023u)) & 1023u);
  QBars *bar = reinterpret_cast<QBars *>(smem + Q_OFF_BAR);
  volatile int *abort_flag = &bar->abort_flag;
  const uint32_t items = BH * qtiles;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    mbar_init(&bar->qd_full, 1);
    mbar_init(&bar->qd_empty, 1);
    for (int s = 0; s < K_SLOTS; ++s) {
      mbar_init(&bar->k_full[s], 1);
      mbar_init(&bar->k_empty[s], 1);
    }
    mbar_init(&bar->v_full, 1);
    mbar_init(&bar->v_empty, 1);
    for (int s = 0; s < 2; ++s) mbar_init(&bar->acc_free[s], SM_WARPS);
    mbar_init(&bar->out_staged, 32 * SM_WARPS);
    mbar_init(&bar->ds_free, 1);
    mbar_init(&bar->s_full, 1);
    mbar_init(&bar->dp_full, 1);
    mbar_init(&bar->s_read, SM_WARPS);
    mbar_init(&bar->ds_full, SM_WARPS);
    mbar_init(&bar->dq_done, 1);
    mbar_init(&bar->drain, 1);
    bar->abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(&bar->tmem, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bar->tmem;  // S at 0, dP at 128, dQ at 256 / 384 (by item parity)

  if (warp == 0) {
    if (lane == 0) {
      uint32_t kvc = 0;  // K / V blocks loaded
      int k = 0;         // items with work, in every role
      for (uint32_t rnd = 0; rnd * gridDim.x < items && !*abort_flag; ++rnd) {
        const uint32_t i = q_pick(rnd);
        if (i >= items) continue;
        const QItem it = q_item(i, BH, qtiles, Sq, Skv, causal);
        if (it.n == 0) continue;
        if (!mbar_wait(&bar->qd_empty, (k++ & 1) ^ 1, status)) {
          *abort_flag = 1;
          break;
        }
        mbar_arrive_expect_tx(&bar->qd_full, 2 * TILE);
        load_rows<2>(smem + Q_OFF_Q, &tmQ, &bar->qd_full, io.in, it.bh, Sq, it.q0);
        load_rows<2>(smem + Q_OFF_DO, &tmDO, &bar->qd_full, io.in, it.bh, Sq, it.q0);
        for (int j = 0; j < it.n && !*abort_flag; ++j, ++kvc) {
          // K(j) waits for dQ(j-3) to release its slot, V(j) for dP(j-1):
          // in that order they come free
          const int s = (int)(kvc % K_SLOTS);
          if (!mbar_wait(&bar->k_empty[s], ((kvc / K_SLOTS) & 1) ^ 1, status)) {
            *abort_flag = 1;
            break;
          }
          mbar_arrive_expect_tx(&bar->k_full[s], TILE);
          load_rows<2>(smem + Q_OFF_K + s * TILE, &tmK, &bar->k_full[s], io.in, it.bh, Skv, j * BN);
          if (!mbar_wait(&bar->v_empty, (kvc & 1) ^ 1, status)) {
            *abort_flag = 1;
            break;
          }
          mbar_arrive_expect_tx(&bar->v_full, TILE);
          load_rows<2>(smem + Q_OFF_V, &tmV, &bar->v_full, io.in, it.bh, Skv, j * BN);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t qa = smem_u32(smem + Q_OFF_Q), da = smem_u32(smem + Q_OFF_DO);
      const uint32_t dsa = smem_u32(smem + Q_OFF_DS);
      auto ka = [&](uint32_t c) { return smem_u32(smem + Q_OFF_K + (c % K_SLOTS) * TILE); };
      const uint32_t va = smem_u32(smem + Q_OFF_V);
      auto kfull = [&](uint32_t c) { return &bar->k_full[c % K_SLOTS]; };
      auto kpar = [&](uint32_t c) { return (c / K_SLOTS) & 1; };
      uint32_t g = 0;  // key blocks of all earlier items (the K / V stage counter too)
      bool ok = true;
      int k = -1;
      for (uint32_t rnd = 0; rnd * gridDim.x < items && ok && !*abort_flag; ++rnd) {
        const uint32_t i = q_pick(rnd);
        if (i >= items) continue;
        const QItem it = q_item(i, BH, qtiles, Sq, Skv, causal);
        if (it.n == 0) continue;
        ++k;
        const uint32_t acc = tmem + 256 + (uint32_t)(k & 1) * 128;
        // block 0: S and dP (the previous item's last S / dP were read before
        // its last dS was published, which its last dQ waited for)
        ok = mbar_wait(&bar->qd_full, k & 1, status) &&
             mbar_wait(kfull(g), kpar(g), status) &&
             (k < 2 || mbar_wait(&bar->acc_free[k & 1], ((k >> 1) - 1) & 1, status));
        if (!ok) break;
        tc_fence_after();
        mma_kk(tmem + 0, qa, ka(g));  // S  = Q  K_0^T
        tc_commit(&bar->s_full);
        ok = mbar_wait(&bar->v_full, g & 1, status);
        if (!ok) break;
        tc_fence_after();
        mma_kk(tmem + 128, da, va);  // dP = dO V_0^T
        tc_commit(&bar->dp_full);
        tc_commit(&bar->v_empty);
        if (it.n == 1) tc_commit(&bar->qd_empty);  // Q / dO: last S / dP issued
        for (int j = 0; j < it.n && ok && !*abort_flag; ++j) {
          const uint32_t gj = g + (uint32_t)j;
          if (j + 1 < it.n) {
            ok = mbar_wait(kfull(gj + 1), kpar(gj + 1), status) &&
                 mbar_wait(&bar->s_read, gj & 1, status);
            if (!ok) break;
            tc_fence_after();
            mma_kk(tmem + 0, qa, ka(gj + 1));  // S(j+1), over the S(j) just read
            tc_commit(&bar->s_full);
          }
          ok = mbar_wait(&bar->ds_full, gj & 1, status);
          if (!ok) break;
          tc_fence_after();
          // dP(j+1) first (over the dP(j) read for dS(j)): the softmax needs it
          // for dS(j+1) as soon as dQ(j) has read dS(j)
          if (j + 1 < it.n) {
            ok = mbar_wait(&bar->v_full, (gj + 1) & 1, status);
            if (!ok) break;
            tc_fence_after();
            mma_kk(tmem + 128, da, va);
            tc_commit(&bar->dp_full);
            tc_commit(&bar->v_empty);
            if (j + 2 == it.n) tc_commit(&bar->qd_empty);
          }
          mma_km(acc, dsa, ka(gj), j > 0);  // dQ += dS(j) K_j
          tc_commit(&bar->dq_done);
          tc_commit(&bar->k_empty[gj % K_SLOTS]);
        }
        g += (uint32_t)it.n;
      }
      if (!ok) *abort_flag = 1;
      tc_commit(&bar->drain);
      mbar_wait(&bar->drain, 0, status);
    }
  } else {
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;  // which 64 columns of each block
    const int row = quarter * 32 + lane;
    const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
    uint8_t *ds_tile = smem + Q_OFF_DS;
    bool ok = true;
    uint32_t g = 0;
    int k = -1;
    for (uint32_t rnd = 0; rnd * gridDim.x < items && ok; ++rnd) {
      const uint32_t i = q_pick(rnd);
      if (i >= items) continue;
      const QItem it = q_item(i, BH, qtiles, Sq, Skv, causal);
      if (it.n == 0) continue;
      ++k;
      const uint32_t bh = it.bh, m = it.q0 + row;
      const bool valid = m < Sq;
      const float lse = valid ? io.lse[(size_t)bh * Sq + m] : INFINITY;
      const float dl = valid ? io.delta[(size_t)bh * Sq + m] : 0.0f;
      const uint32_t acc = tmem + 256 + (uint32_t)(k & 1) * 128;
      for (int j = 0; j < it.n && ok; ++j) {
        const uint32_t gj = g + (uint32_t)j;
        if (*abort_flag || !mbar_wait(&bar->s_full, gj & 1, status)) {
          *abort_flag = 1;
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t n0 = (uint32_t)j * BN;
        uint32_t lim = Skv - 1;
        if (causal && m < lim) lim = m;
        const int lim_rel = (int)lim - (int)n0;
        // P for this warp's 64 columns, kept in registers (both 32-column
        // loads in flight before one wait).  Of every 8 column pairs, 2 take
        // exp2 on the FMA pipe; blocks below the diagonal skip the mask.
        float p[BN / 2];
        {
          uint32_t rs[2][32];
          tmem_ld_32x32b_x32(tmem + lane_base + half * 64, rs[0]);
          tmem_ld_32x32b_x32(tmem + lane_base + half * 64 + 32, rs[1]);
          tc_wait_ld(rs[0]);
          tc_wait_ld(rs[1]);
          // S(j) is in registers: S(j+1) may now overwrite it, and runs
          // while this block's exp2 and dS work goes on
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&bar->s_read);
          const uint64_t sc2 = f2pack(scale_log2, scale_log2), nl2 = f2pack(-lse, -lse);
          auto pq = [&](auto masked) {
#pragma unroll
            for (int cc = 0; cc < 2; ++cc)
#pragma unroll
              for (int g = 0; g < 8; ++g) {
                const uint32_t *r = &rs[cc][4 * g];
                float y[4], e[4];
                f2unpack(f2fma(f2pack(__uint_as_float(r[0]), __uint_as_float(r[1])), sc2, nl2),
                         y[0], y[1]);
                f2unpack(f2fma(f2pack(__uint_as_float(r[2]), __uint_as_float(r[3])), sc2, nl2),
                         y[2], y[3]);
                if ((g & 3) == 3) {
                  exp2_fma2(y[0], y[1], e[0], e[1]);
                  exp2_fma2(y[2], y[3], e[2], e[3]);
                } else {
#pragma unroll
                  for (int k = 0; k < 4; ++k) e[k] = fast_exp2(y[k]);
                }
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                  if constexpr (decltype(masked)::value) {
                    if ((half * 2 + cc) * 32 + 4 * g + k > lim_rel) e[k] = 0.0f;
                  }
                  p[cc * 32 + 4 * g + k] = e[k];
                }
              }
          };
          if (__all_sync(0xffffffffu, lim_rel >= BN - 1))
            pq(std::false_type{});
          else
            pq(std::true_type{});
        }
        // dS smem is free once the dQ MMA of the previous block is done and,
        // in an item's first block, once the previous item's dQ tile staged
        // there has been read by its TMA store
        if (!mbar_wait(&bar->dp_full, gj & 1, status) ||
            (gj > 0 && !mbar_wait(&bar->dq_done, (gj - 1) & 1, status)) ||
            (io.tma_out && j == 0 && k > 0 && !mbar_wait(&bar->ds_free, (k - 1) & 1, status))) {
          *abort_flag = 1;
          ok = false;
          break;
        }
        tc_fence_after();
        {
          uint32_t rp[2][32];
          tmem_ld_32x32b_x32(tmem + lane_base + 128 + half * 64, rp[0]);
          tmem_ld_32x32b_x32(tmem + lane_base + 128 + half * 64 + 32, rp[1]);
          tc_wait_ld(rp[0]);
          tc_wait_ld(rp[1]);
          const uint64_t nd2 = f2pack(-dl, -dl);
#pragma unroll
          for (int cc = 0; cc < 2; ++cc) {
            uint32_t pk[16];
#pragma unroll
            for (int e = 0; e < 16; ++e) {
              // dS = P (dP - delta), a masked P being 0
              float t0, t1;
              f2unpack(f2mul(f2pack(p[cc * 32 + 2 * e], p[cc * 32 + 2 * e + 1]),
                             f2add(f2pack(__uint_as_float(rp[cc][2 * e]),
                                          __uint_as_float(rp[cc][2 * e + 1])),
                                   nd2)),
                       t0, t1);
              pk[e] = pack_bf16(t0, t1);
            }
            store_swizzled_chunk(ds_tile, row, half * 2 + cc, pk);
          }
        }
        fence_proxy_async_smem();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bar->ds_full);  // also: dP(j) has been read
      }
      if (!ok) break;
      g += (uint32_t)it.n;
      // this item's dQ: all its MMAs are done when its last dq_done arrives
      if (!mbar_wait(&bar->dq_done, (g - 1) & 1, status)) {
        *abort_flag = 1;
        ok = false;
        break;
      }
      tc_fence_after();
      if (io.tma_out) {
        // dQ (x scale, bf16) staged in the dS tile, whose last reader dQ(n-1)
        // is done, and sent with two TMA stores (rows past Sq clipped by the
        // map); the issuing thread releases the tile when they have read it
        stage_row_bf16(acc + lane_base + half * 64, ds_tile, row, half, scale);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bar->acc_free[k & 1]);
        fence_proxy_async_smem();
        mbar_arrive(&bar->out_staged);
        if (threadIdx.x == 64) {
          if (mbar_wait(&bar->out_staged, k & 1, status)) {
            const int32_t hh = (int32_t)(bh % io.in.H), bb = (int32_t)(bh / io.in.H);
            tma_store_4d(&tmDQ, ds_tile, 0, hh, (int32_t)it.q0, bb);
            tma_store_4d(&tmDQ, ds_tile + BOX, 64, hh, (int32_t)it.q0, bb);
            tma_store_commit();
            tma_store_wait_read<0>();  // smem read; the writes finish on their own
          } else {
            *abort_flag = 1;
          }
          mbar_arrive(&bar->ds_free);
        }
      } else {
        uint16_t *dst = io.d0 + ((size_t)(bh / io.in.H) * Sq + m) * io.ldd +
                        (size_t)(bh % io.in.H) * D;
        store_row_bf16(acc + lane_base, dst, scale, valid, half);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bar->acc_free[k & 1]);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ---------------------------------------------------------------------------
// dK, dV
// ---------------------------------------------------------------------------
// Q / dO double-buffered in smem; P^T and dS^T never touch smem: the softmax
// writes them as bf16 pairs into TMEM over the S^T / dP^T columns they were
// computed from (half h of the 128 queries: columns 64h .. 64h+31 of S^T,
// resp. 128 + 64h .. of dP^T, inside the range that warp itself read), and
// the dV / dK MMAs take them as the A operand from TMEM.  MMA order per query
// tile i:  S^T(i), dP^T(i) | dV(i), in two halves as each half of P^T(i) is
// stored | S^T(i+1) (over P^T(i), after dV(i) in issue order) | dK(i) once
// dS^T(i) is stored | dP^T(i+1) (over dS^T(i)), so the exp2 work of tile i+1
// overlaps dK(i).
constexpr int K_OFF_K = 0, K_OFF_V = TILE, K_OFF_Q = 2 * TILE, K_OFF_DO = 4 * TILE,
              K_OFF_LSE = 6 * TILE, K_OFF_BAR = K_OFF_LSE + 2 * 2 * 128 * 4;
constexpr int K_SMEM = K_OFF_BAR + 256 + 1024;
static_assert(K_SMEM <= 232448, "dkdv smem");

struct KBars {
  uint64_t kv_full, kv_empty, q_full[2], q_empty[2], do_full[2], do_empty[2], s_full, dp_full,
      pt_half[2], dst_full, staged, acc_full, acc_free, out_staged[2], sched_full[2],
      sched_empty[2], drain;
  int item[2];
  uint32_t tmem;
  int abort_flag;
};
static_assert(sizeof(KBars) <= 256, "dkdv barriers");

// Work item w: 128 keys (k0) of head bh, seen by query tiles i0 .. qtiles-1.
// Items go in groups of hg heads (about one item per SM), so the CTAs running
// together share a few heads' Q / dO in L2; inside a group the heaviest key
// blocks come first (causal: key block 0 is seen by every query tile), so the
// CTAs that draw from the work counter last get the short items.
struct KItem {
  uint32_t bh, k0, i0;
  int n;  // query tiles
};
__device__ __forceinline__ KItem k_item(uint32_t w, uint32_t BH, uint32_t kblocks,
                                        uint32_t qtiles, uint32_t hg, int causal) {
  const uint32_t per = hg * kblocks, grp = w / per, r = w % per;
  const uint32_t h0 = grp * hg, hn = min(hg, BH - h0);
  KItem it;
  it.bh = h0 + r % hn;
  it.k0 = (r / hn) * BN;
  it.i0 = causal ? min(it.k0 / BM, qtiles) : 0;  // first query tile that sees k0
  it.n = (int)(qtiles - it.i0);
  return it;
}

// D(128 x D) (+)= A(128 x 128 queries, bf16 pairs in TMEM at the half-split
// columns a0 + [0, 32) and a0 + [64, 96)) B(128 queries x D, MN-major smem)
// The K steps of mma_tm in two parts: part 0 covers queries 0-31 and 64-95
// (the first 32-query part each softmax half forms), part 1 the others.
__device__ __forceinline__ void mma_tm_part(uint32_t d, uint32_t a0, uint32_t b, bool acc,
                                            int part) {
  const uint32_t blo = smem_desc_lo(b, BOX);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int ks = (i >> 1) * 4 + part * 2 + (i & 1);  // part 0: 0, 1, 4, 5; part 1: 2, 3, 6, 7
    const uint32_t acol = a0 + (ks >> 2) * 64 + (ks & 3) * 8;
    tc_mma_f16_ts_w(d, acol, blo + ((ks * 2048) >> 4), HI_SW, IDESC_KM, (acc || i > 0) ? 1u : 0u);
  }
}

__device__ __forceinline__ void mma_tm(uint32_t d, uint32_t a0, uint32_t b, bool acc) {
  const uint32_t blo = smem_desc_lo(b, BOX);
#pragma unroll
  for (int ks = 0; ks < 128 / 16; ++ks) {
    const uint32_t acol = a0 + (ks >> 2) * 64 + (ks & 3) * 8;
    tc_mma_f16_ts_w(d, acol, blo + ((ks * 2048) >> 4), HI_SW, IDESC_KM, (acc || ks > 0) ? 1u : 0u);
  }
}

// Persistent: one CTA per SM takes items until none is left: its first item is
// blockIdx.x, the next come from the context's work counter.  The producer
// publishes each item through a two-slot ring (sched_full / sched_empty);
// every role walks the same sequence, and all barrier phases count tiles (g)
// or items (k) over the CTA's whole sequence.  Across items: the next item's
// K / V load as soon as the last S^T / dP^T MMAs of the current one are done
// (kv_empty), its first Q / dO into the free slots, and its S^T(0) / dP^T(0)
// MMAs run while the softmax warps drain the current dV / dK (acc_full); its
// first dV MMA waits for that drain (acc_free).  The drain stages the bf16
// tiles in the last tile's Q / dO slots; the producer thread stores them with
// TMA before it loads into those slots again.
__global__ void __launch_bounds__(THREADS, 1)
    bwd_dkdv_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmDO,
                    const __grid_constant__ CUtensorMap tmDK, const __grid_constant__ CUtensorMap tmDV,
                    const BwdIO io, uint32_t BH, uint32_t Sq, uint32_t Skv, float scale,
                    float scale_log2, int causal, uint32_t kblocks, uint32_t hg, int *sched,
                    int *status) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t *smem = smem_raw + ((1024u - (raw & 1023u)) & 1023u);
  KBars *bar = reinterpret_cast<KBars *>(smem + K_OFF_BAR);
  volatile int *abort_flag = &bar->abort_flag;
  float *lse_s = reinterpret_cast<float *>(smem + K_OFF_LSE);  // [2][128]
  float *del_s = lse_s + 2 * 128;                              // [2][128]
  const uint32_t qtiles = (Sq + BM - 1) / BM;
  const int total = (int)(BH * kblocks);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    mbar_init(&bar->kv_full, 1);
    mbar_init(&bar->kv_empty, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&bar->q_full[s], 1);
      mbar_init(&bar->q_empty[s], 1);
      mbar_init(&bar->do_full[s], 1);
      mbar_init(&bar->do_empty[s], 1);
      mbar_init(&bar->sched_full[s], 1);
      mbar_init(&bar->sched_empty[s], 1 + SM_WARPS);  // MMA thread + softmax warps
    }
    mbar_init(&bar->s_full, 1);
    mbar_init(&bar->dp_full, 1);
    mbar_init(&bar->pt_half[0], SM_WARPS);
    mbar_init(&bar->pt_half[1], SM_WARPS);
    mbar_init(&bar->dst_full, SM_WARPS);
    mbar_init(&bar->staged, 32 * SM_WARPS);
    mbar_init(&bar->acc_full, 1);
    mbar_init(&bar->acc_free, SM_WARPS);
    mbar_init(&bar->out_staged[0], 32 * SM_WARPS);  // by item parity
    mbar_init(&bar->out_staged[1], 32 * SM_WARPS);
    mbar_init(&bar->drain, 1);
    bar->abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(&bar->tmem, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bar->tmem;  // S^T 0, dP^T 128, dV 256, dK 384

  if (warp == 0) {
    // ------------------------------------------------- scheduler + producer
    if (lane == 0) {
      bool ok = true;
      uint32_t g = 0, k = 0;  // tiles / items (with query tiles) loaded so far
      int w = (int)blockIdx.x;
      // The drain of an item leaves its bf16 dV / dK tiles in its last tile's
      // dO / Q slot; this thread stores them (oldest first) before it loads
      // into that slot again, or before it exits, so no softmax warp waits on
      // a store.  At most two drains are pending: slots alternate by tile.
      struct Pend {
        uint32_t k, bh, k0;
        int sl;
      } pq[2] = {};
      int np = 0;
      auto flush_one = [&]() {
        const Pend e = pq[0];
        pq[0] = pq[1];
        --np;
        const bool staged = mbar_wait(&bar->out_staged[e.k & 1], (e.k >> 1) & 1, status);
        if (staged && io.tma_out) {
          const int32_t hh = (int32_t)(e.bh % io.in.H), bb = (int32_t)(e.bh / io.in.H);
          for (int box = 0; box < 2; ++box) {
            tma_store_4d(&tmDV, smem + K_OFF_DO + e.sl * TILE + box * BOX, box * 64, hh,
                         (int32_t)e.k0, bb);
            tma_store_4d(&tmDK, smem + K_OFF_Q + e.sl * TILE + box * BOX, box * 64, hh,
                         (int32_t)e.k0, bb);
          }
          tma_store_commit();
          tma_store_wait_read<0>();  // smem read; the writes finish on their own
        }
        mbar_arrive(&bar->q_empty[e.sl]);  // the slots of that item's last tile, free again
        mbar_arrive(&bar->do_empty[e.sl]);
        return staged;
      };
      for (uint32_t seq = 0; ok && !*abort_flag; ++seq) {
        const int slot = seq & 1;
        if (!mbar_wait(&bar->sched_empty[slot], ((seq >> 1) & 1) ^ 1, status)) {
          ok = false;
          break;
        }
        bar->item[slot] = w < total ? w : -1;
        mbar_arrive(&bar->sched_full[slot]);
        if (w >= total) break;
        const KItem it = k_item((uint32_t)w, BH, kblocks, qtiles, hg, causal);
        if (it.n > 0) {
          if (k > 0 && !mbar_wait(&bar->kv_empty, (k - 1) & 1, status)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&bar->kv_full, 2 * TILE);
          load_rows<2>(smem + K_OFF_K, &tmK, &bar->kv_full, io.in, it.bh, Skv, it.k0);
          load_rows<2>(smem + K_OFF_V, &tmV, &bar->kv_full, io.in, it.bh, Skv, it.k0);
          // Q and dO have their own slots: dO(t) is free once dV(t) is
          // done, Q(t) only after dK(t), so each load starts as early as it can
          for (int t = 0; t < it.n; ++t, ++g) {
            const int s = g & 1;
            const uint32_t par = ((g >> 1) & 1) ^ 1;
            const uint32_t qs = (it.i0 + t) * BM;
            while (ok && np > 0 && (pq[0].sl == s || (np == 2 && pq[1].sl == s))) ok = flush_one();
            if (!ok) break;
            if (!mbar_wait(&bar->q_empty[s], par, status)) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(&bar->q_full[s], TILE);
            load_rows<2>(smem + K_OFF_Q + s * TILE, &tmQ, &bar->q_full[s], io.in, it.bh, Sq, qs);
            if (!mbar_wait(&bar->do_empty[s], par, status)) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(&bar->do_full[s], TILE);
            load_rows<2>(smem + K_OFF_DO + s * TILE, &tmDO, &bar->do_full[s], io.in, it.bh, Sq, qs);
          }
          if (ok && np == 2) ok = flush_one();
          pq[np++] = Pend{k, it.bh, it.k0, (int)((g - 1) & 1)};
          ++k;
        }
        w = (int)gridDim.x + atomicAdd(sched, 1);
      }
      while (ok && np > 0) ok = flush_one();
      if (!ok) *abort_flag = 1;
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA
    if (lane == 0) {
      bool ok = true;
      uint32_t g = 0, k = 0;
      const uint32_t ka = smem_u32(smem + K_OFF_K), va = smem_u32(smem + K_OFF_V);
      auto qa = [&](uint32_t gg) { return smem_u32(smem + K_OFF_Q + (gg & 1) * TILE); };
      auto da = [&](uint32_t gg) { return smem_u32(smem + K_OFF_DO + (gg & 1) * TILE); };
      for (uint32_t seq = 0; ok; ++seq) {
        const int slot = seq & 1;
        if (!mbar_wait(&bar->sched_full[slot], (seq >> 1) & 1, status)) {
          ok = false;
          break;
        }
        const int w = bar->item[slot];
        mbar_arrive(&bar->sched_empty[slot]);
        if (w < 0) break;
        const int n = k_item((uint32_t)w, BH, kblocks, qtiles, hg, causal).n;
        if (n == 0) continue;
        const uint32_t g0 = g;
        ok = mbar_wait(&bar->kv_full, k & 1, status) &&
             mbar_wait(&bar->q_full[g0 & 1], (g0 >> 1) & 1, status);
        if (!ok) break;
        tc_fence_after();
        mma_kk(tmem + 0, ka, qa(g0));  // S^T(0)  = K  Q_0^T
        tc_commit(&bar->s_full);
        ok = mbar_wait(&bar->do_full[g0 & 1], (g0 >> 1) & 1, status);
        if (!ok) break;
        tc_fence_after();
        mma_kk(tmem + 128, va, da(g0));  // dP^T(0) = V dO_0^T
        tc_commit(&bar->dp_full);
        if (n == 1) tc_commit(&bar->kv_empty);  // K / V read for the last time
        for (int t = 0; t < n && ok && !*abort_flag; ++t) {
          const uint32_t gg = g0 + t;
          ok = mbar_wait(&bar->pt_half[0], gg & 1, status);
          // the first dV of an item overwrites the accumulator the previous
          // item's drain reads
          if (ok && t == 0 && k > 0) ok = mbar_wait(&bar->acc_free, (k - 1) & 1, status);
          if (!ok) break;
          tc_fence_after();
          mma_tm_part(tmem + 256, tmem + 0, da(gg), t > 0, 0);  // dV += P^T(t) dO_t: queries
          ok = mbar_wait(&bar->pt_half[1], gg & 1, status);     // 0-31, 64-95, then the rest
          if (!ok) break;
          tc_fence_after();
          mma_tm_part(tmem + 256, tmem + 0, da(gg), true, 1);
          if (t + 1 < n) {
            tc_commit(&bar->do_empty[gg & 1]);  // the last tile's slot: released by the drain
            ok = mbar_wait(&bar->q_full[(gg + 1) & 1], ((gg + 1) >> 1) & 1, status);
            if (!ok) break;
            tc_fence_after();
            mma_kk(tmem + 0, ka, qa(gg + 1));  // S^T(t+1), after dV(t) read P^T(t)
            tc_commit(&bar->s_full);
          }
          ok = mbar_wait(&bar->dst_full, gg & 1, status);
          if (!ok) break;
          tc_fence_after();
          mma_tm(tmem + 384, tmem + 128, qa(gg), t > 0);  // dK += dS^T(t) Q_t
          tc_commit(t + 1 < n ? &bar->q_empty[gg & 1] : &bar->acc_full);
          if (t + 1 < n) {
            ok = mbar_wait(&bar->do_full[(gg + 1) & 1], ((gg + 1) >> 1) & 1, status);
            if (!ok) break;
            tc_fence_after();
            mma_kk(tmem + 128, va, da(gg + 1));  // dP^T(t+1), after dK(t) read dS^T(t)
            tc_commit(&bar->dp_full);
            if (t + 2 == n) tc_commit(&bar->kv_empty);
          }
        }
        g += (uint32_t)n;
        ++k;
      }
      if (!ok) *abort_flag = 1;
      tc_commit(&bar->drain);
      mbar_wait(&bar->drain, 0, status);
    }
  } else {
    // -------------------------------------------------------------- softmax
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;     // which 64 query columns of each tile
    const int row = quarter * 32 + lane;  // key within the block
    const int tid = (threadIdx.x - 64) & 127;  // both halves stage the same 128 values
    const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
    bool ok = true;
    uint32_t gt = 0, k = 0;  // tiles / items done (the inner loops use g for column groups)
    for (uint32_t seq = 0; ok; ++seq) {
      const int slot = seq & 1;
      if (!mbar_wait(&bar->sched_full[slot], (seq >> 1) & 1, status)) {
        ok = false;
        break;
      }
      const int w = bar->item[slot];
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar->sched_empty[slot]);
      if (w < 0) break;
      const KItem itm = k_item((uint32_t)w, BH, kblocks, qtiles, hg, causal);
      const uint32_t bh = itm.bh, k0 = itm.k0, i0 = itm.i0;
      const int n = itm.n;
      const uint32_t key = k0 + row;
      const bool valid = key < Skv;
      uint16_t *dk_dst = io.d0 + ((size_t)(bh / io.in.H) * Skv + key) * io.ldd + (size_t)(bh % io.in.H) * D;
      uint16_t *dv_dst = io.d1 + ((size_t)(bh / io.in.H) * Skv + key) * io.ldd + (size_t)(bh % io.in.H) * D;
      if (n == 0) {
        // no query sees these keys: zero gradients
        if (valid)
          for (int c = half * (D / 2); c < (half + 1) * (D / 2); c += 8) {
            *reinterpret_cast<uint4 *>(dk_dst + c) = make_uint4(0, 0, 0, 0);
            *reinterpret_cast<uint4 *>(dv_dst + c) = make_uint4(0, 0, 0, 0);
          }
        continue;
      }
      // -lse / -delta of one query per thread, loaded a tile ahead so the
      // global loads' latency hides behind the current tile
      float nl = -INFINITY, nd = 0.0f;
      auto fetch = [&](int t) {
        const uint32_t q = (i0 + t) * BM + tid;
        nl = q < Sq ? -io.lse[(size_t)bh * Sq + q] : -INFINITY;
        nd = q < Sq ? -io.delta[(size_t)bh * Sq + q] : 0.0f;
      };
      fetch(0);
      for (int t = 0; t < n && ok; ++t) {
        const uint32_t gg = gt + t;
        const uint32_t qs = (i0 + t) * BM;
        // stage this tile's -lse / -delta in buffer gg & 1; every thread
        // passed phase gg-1 only after all had finished tile gg-2, so the
        // buffer is free.  Bounded wait, like every other.
        lse_s[(gg & 1) * 128 + tid] = nl;
        del_s[(gg & 1) * 128 + tid] = nd;
        mbar_arrive(&bar->staged);
        if (t + 1 < n) fetch(t + 1);
        if (*abort_flag || !mbar_wait(&bar->staged, gg & 1, status) ||
            !mbar_wait(&bar->s_full, gg & 1, status)) {
          *abort_flag = 1;
          ok = false;
          break;
        }
        tc_fence_after();
        // query q = qs + col is visible to this key iff q >= key (causal),
        // q < Sq and key < Skv
        int first_rel = causal ? (int)key - (int)qs : 0;  // first visible col
        if (first_rel < 0) first_rel = 0;
        const int last_rel = key < Skv ? (int)min(Sq - 1 - qs, (uint32_t)127) : -1;
        const float *nls = lse_s + (gg & 1) * 128;  // -lse per query
        const float *ndd = del_s + (gg & 1) * 128;  // -delta per query
        // P^T for this warp's 64 queries: registers, and bf16 pairs into TMEM.
        // Of every 8 column pairs, 2 take exp2 on the FMA pipe (exp2_fma2) to
        // share the load with MUFU.  Tiles off the diagonal skip the mask.
        float p[64];
        {
          uint32_t rs[2][32];  // both 32-column loads in flight before one wait
          tmem_ld_32x32b_x32(tmem + lane_base + half * 64, rs[0]);
          tmem_ld_32x32b_x32(tmem + lane_base + half * 64 + 32, rs[1]);
          tc_wait_ld(rs[0]);
          tc_wait_ld(rs[1]);
          const uint64_t sc2 = f2pack(scale_log2, scale_log2);
          auto pt = [&](auto masked) {
  #pragma unroll
            for (int cc = 0; cc < 2; ++cc) {
              const int c = half * 2 + cc;
              const float4 *l4 = reinterpret_cast<const float4 *>(nls + c * 32);
              uint32_t pk[16];
  #pragma unroll
              for (int g = 0; g < 8; ++g) {
                const float4 l = l4[g];
                const uint32_t *r = &rs[cc][4 * g];
                float y[4], e[4];
                f2unpack(f2fma(f2pack(__uint_as_float(r[0]), __uint_as_float(r[1])), sc2,
                               f2pack(l.x, l.y)),
                         y[0], y[1]);
                f2unpack(f2fma(f2pack(__uint_as_float(r[2]), __uint_as_float(r[3])), sc2,
                               f2pack(l.z, l.w)),
                         y[2], y[3]);
                if ((g & 3) == 3) {
                  exp2_fma2(y[0], y[1], e[0], e[1]);
                  exp2_fma2(y[2], y[3], e[2], e[3]);
                } else {
  #pragma unroll
                  for (int k = 0; k < 4; ++k) e[k] = fast_exp2(y[k]);
                }
                if constexpr (decltype(masked)::value) {
  #pragma unroll
                  for (int k = 0; k < 4; ++k) {
                    const int col = c * 32 + 4 * g + k;
                    if (col < first_rel || col > last_rel) e[k] = 0.0f;
                  }
                }
  #pragma unroll
                for (int k = 0; k < 4; ++k) p[cc * 32 + 4 * g + k] = e[k];
                pk[2 * g] = pack_bf16(e[0], e[1]);
                pk[2 * g + 1] = pack_bf16(e[2], e[3]);
              }
              tmem_st_32x32b_x16(tmem + lane_base + half * 64 + cc * 16, pk);
              // each 32-query part of P^T is signalled on its own, so the
              // dV MMAs over it start while the next part is formed
              tc_wait_st();
              tc_fence_before();
              __syncwarp();
              if (lane == 0) mbar_arrive(&bar->pt_half[cc]);  // cc 1: S^T(t) has been read
            }
          };
          if (__all_sync(0xffffffffu, first_rel == 0 && last_rel == 127))
            pt(std::false_type{});
          else
            pt(std::true_type{});
        }
        if (!mbar_wait(&bar->dp_full, gg & 1, status)) {
          *abort_flag = 1;
          ok = false;
          break;
        }
        tc_fence_after();
        {
          uint32_t rp[2][32];
          tmem_ld_32x32b_x32(tmem + lane_base + 128 + half * 64, rp[0]);
          tmem_ld_32x32b_x32(tmem + lane_base + 128 + half * 64 + 32, rp[1]);
          tc_wait_ld(rp[0]);
          tc_wait_ld(rp[1]);
  #pragma unroll
          for (int cc = 0; cc < 2; ++cc) {
            const int c = half * 2 + cc;
            const float4 *d4 = reinterpret_cast<const float4 *>(ndd + c * 32);
            uint32_t dk[16];
  #pragma unroll
            for (int g = 0; g < 8; ++g) {
              // dS^T = P^T (dP^T - delta), a masked P^T being 0
              const float4 d = d4[g];
              const uint32_t *r = &rp[cc][4 * g];
              const float *pp = &p[cc * 32 + 4 * g];
              float t0, t1, t2, t3;
              f2unpack(f2mul(f2pack(pp[0], pp[1]),
                             f2add(f2pack(__uint_as_float(r[0]), __uint_as_float(r[1])),
                                   f2pack(d.x, d.y))),
                       t0, t1);
              f2unpack(f2mul(f2pack(pp[2], pp[3]),
                             f2add(f2pack(__uint_as_float(r[2]), __uint_as_float(r[3])),
                                   f2pack(d.z, d.w))),
                       t2, t3);
              dk[2 * g] = pack_bf16(t0, t1);
              dk[2 * g + 1] = pack_bf16(t2, t3);
            }
            tmem_st_32x32b_x16(tmem + lane_base + 128 + half * 64 + cc * 16, dk);
          }
        }
        tc_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bar->dst_full);  // also: dP^T(t) has been read
      }
      if (!ok) break;
      // drain: every MMA of the item, dK(n-1) last, is done at acc_full
      const int sl = (int)((gt + n - 1) & 1);
      const bool done = mbar_wait(&bar->acc_full, k & 1, status);
      if (done)
        tc_fence_after();
      else
        *abort_flag = 1;
      if (io.tma_out) {
        // stage dV / dK as bf16 in the last tile's dO / Q slot, laid out like
        // the loaded tiles (two 64-column boxes, 128-byte swizzle); the
        // producer thread sends them with four TMA stores (whole rows leave
        // as bulk writes, rows past Skv are clipped by the map) before it
        // reuses the slot
        uint8_t *sv = smem + K_OFF_DO + sl * TILE, *sk = smem + K_OFF_Q + sl * TILE;
        if (done) {
          stage_row_bf16(tmem + lane_base + 256 + half * 64, sv, row, half, 1.0f);
          stage_row_bf16(tmem + lane_base + 384 + half * 64, sk, row, half, scale);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bar->acc_free);  // dV / dK read out of TMEM
        fence_proxy_async_smem();
      } else {
        if (done) {
          store_row_bf16(tmem + lane_base + 256, dv_dst, 1.0f, valid, half);
          store_row_bf16(tmem + lane_base + 384, dk_dst, scale, valid, half);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bar->acc_free);
      }
      mbar_arrive(&bar->out_staged[k & 1]);  // every softmax thread, done or not
      if (!done) {
        ok = false;
        break;
      }
      gt += (uint32_t)n;
      ++k;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

int make_map(BwppCudaCtx *ctx, CUtensorMap *map, const void *base, uint32_t S, uint32_t BH,
             uint32_t H, uint32_t ld) {
  bwpp_encode_tiled_fn enc = bwpp_get_encode_tiled();
  if (!enc) return bwpp_set_error(ctx, BWPP_CUDA_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[3] = {D, H, (cuuint64_t)(BH / H) * S};
  cuuint64_t strides[2] = {(cuuint64_t)D * 2, (cuuint64_t)ld * 2};
  cuuint32_t box[3] = {64, 1, 128};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void *>(base), dims,
                   strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return bwpp_set_error(ctx, BWPP_CUDA_ERR_CUDA, "attention bwd tensor map failed (%d)", (int)r);
  return BWPP_CUDA_OK;
}

// dK / dV as a TMA store target: token-major rows b*S + s, head h at column
// h*128, pitch ld; 4-D {D, H, S, B} so a box never crosses into the next
// sequence (rows past S are clipped).  Returns false where TMA cannot take
// the layout (base or pitch not 16-byte aligned); the kernel then stores rows
// directly.
bool make_out_map(CUtensorMap *map, const void *base, uint32_t S, uint32_t B, uint32_t H,
                  uint32_t ld) {
  bwpp_encode_tiled_fn enc = bwpp_get_encode_tiled();
  if (!enc || (reinterpret_cast<uintptr_t>(base) & 15u) || (ld % 8)) return false;
  cuuint64_t dims[4] = {D, H, S, B};
  cuuint64_t strides[3] = {(cuuint64_t)D * 2, (cuuint64_t)ld * 2, (cuuint64_t)S * ld * 2};
  cuuint32_t box[4] = {64, 1, 128, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void *>(base), dims, strides,
             box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool g_attr[64] = {};

}  // namespace

// Token-major bf16 inputs (q/k/v with pitch ld_in, dO with pitch ld_do, head h
// at column h*128), lse / delta [B*H, S]; writes dQ, dK, dV token-major bf16
// with pitch ldd.  Sq == Skv == S, head dim 128.
int bwpp_attention_bwd_train(BwppCudaCtx *ctx, const uint16_t *q, const uint16_t *k,
                             const uint16_t *v, uint32_t ld_in, const uint16_t *dout,
                             uint32_t ld_do, const float *lse, const float *delta,
                             uint32_t B, uint32_t H, uint32_t S, float scale, int causal,
                             uint16_t *dq, uint16_t *dk, uint16_t *dv, uint32_t ldd) {
  // 16-byte rows: the tensor maps and the 128-bit stores need aligned
  // pitches and output bases
  if (S == 0 || !(scale > 0.0f) || (ld_in % 8) || (ld_do % 8) || (ldd % 8) ||
      ((reinterpret_cast<uintptr_t>(dq) | reinterpret_cast<uintptr_t>(dk) |
        reinterpret_cast<uintptr_t>(dv)) & 15u))
    return bwpp_set_error(ctx, BWPP_CUDA_ERR_UNSUPPORTED, "attention bwd: layout");
  const uint32_t BH = B * H;
  CUtensorMap tq, tk, tv, tdo;
  int rc = make_map(ctx, &tq, q, S, BH, H, ld_in);
  if (!rc) rc = make_map(ctx, &tk, k, S, BH, H, ld_in);
  if (!rc) rc = make_map(ctx, &tv, v, S, BH, H, ld_in);
  if (!rc) rc = make_map(ctx, &tdo, dout, S, BH, H, ld_do);
  if (rc) return rc;
  if (ctx->device < 64 && !g_attr[ctx->device]) {
    rc = bwpp_check_cuda(ctx,
                         cudaFuncSetAttribute(bwd_dq_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                              Q_SMEM),
                         "bwd dq smem");
    if (!rc)
      rc = bwpp_check_cuda(ctx,
                           cudaFuncSetAttribute(bwd_dkdv_kernel,
                                                cudaFuncAttributeMaxDynamicSharedMemorySize, K_SMEM),
                           "bwd dkdv smem");
    if (rc) return rc;
    g_attr[ctx->device] = true;
  }
  const float sl2 = scale * 1.4426950408889634f;
  const uint32_t tiles = (S + 127) / 128;
  BwdIO io{dq, nullptr, ldd, lse, delta, AttnIO{nullptr, nullptr, 0, nullptr, 1, H}, 0};
  CUtensorMap tdq;
  io.tma_out = make_out_map(&tdq, dq, S, B, H, ldd);
  if (!io.tma_out) tdq = tq;  // unused
  const uint32_t dq_grid = min((uint32_t)ctx->num_sms, tiles * BH);  // persistent
  bwd_dq_kernel<<<dq_grid, THREADS, Q_SMEM, ctx->stream>>>(tq, tk, tv, tdo, tdq, io, BH, S, S, scale,
                                                           sl2, causal, tiles, ctx->status_word);
  BWPP_LAUNCH_CHECK(ctx, "attention bwd dq");
  BwdIO io2{dk, dv, ldd, lse, delta, AttnIO{nullptr, nullptr, 0, nullptr, 1, H}, 0};
  CUtensorMap tdk, tdv;
  io2.tma_out = make_out_map(&tdk, dk, S, B, H, ldd) && make_out_map(&tdv, dv, S, B, H, ldd);
  if (!io2.tma_out) tdk = tdv = tq;  // unused
  // persistent: one CTA per SM (at most one per item); the work counter
  // hands out items gridDim.x, gridDim.x + 1, ...
  const uint32_t kv_items = tiles * BH;
  const uint32_t kv_grid = min((uint32_t)ctx->num_sms, kv_items);
  const uint32_t hg = max(1u, (uint32_t)ctx->num_sms / tiles);  // heads per item group
  rc = bwpp_check_cuda(ctx, cudaMemsetAsync(ctx->sched_counter, 0, sizeof(int), ctx->stream),
                       "attention bwd work counter");
  if (rc) return rc;
  bwd_dkdv_kernel<<<kv_grid, THREADS, K_SMEM, ctx->stream>>>(tq, tk, tv, tdo, tdk, tdv, io2, BH, S, S,
                                                             scale, sl2, causal, tiles, hg,
                                                             ctx->sched_counter, ctx->status_word);
  BWPP_LAUNCH_CHECK(ctx, "attention bwd dkdv");
  return BWPP_CUDA_OK;
}

int bwpp_attention_fwd_train(BwppCudaCtx *ctx, const uint16_t *q, const uint16_t *k,
                             const uint16_t *v, uint32_t ld_in, uint32_t B, uint32_t H,
                             uint32_t S, uint32_t D, float scale, int causal, uint16_t *o,
                             uint32_t ldo, float *lse);
int bwpp_attn_delta(BwppCudaCtx *ctx, const uint16_t *dO, const uint16_t *O, float *delta,
                    uint32_t B, uint32_t S, uint32_t H, uint32_t Dh);

extern "C" {

int bwpp_cuda_attention_fwd_lse_bf16(BwppCudaCtx *ctx, const uint16_t *q, const uint16_t *k,
                                     const uint16_t *v, uint32_t ld_qkv, uint32_t B, uint32_t H,
                                     uint32_t S, float scale, int causal, uint16_t *o,
                                     uint32_t ldo, float *lse) {
  int rc = bwpp_ctx_enter(ctx);
  if (rc) return rc;
  if (!q || !k || !v || !o || !lse || ld_qkv < H * D || ldo < H * D)
    return bwpp_set_error(ctx, BWPP_CUDA_ERR_ARG, "attention fwd_lse: bad args");
  if (B == 0 || H == 0 || S == 0) return BWPP_CUDA_OK;
  return bwpp_attention_fwd_train(ctx, q, k, v, ld_qkv, B, H, S, D, scale, causal, o, ldo, lse);
}

int bwpp_cuda_attention_bwd_bf16(BwppCudaCtx *ctx, const uint16_t *q, const uint16_t *k,
                                 const uint16_t *v, uint32_t ld_qkv, const uint16_t *o,
                                 uint32_t ldo, const uint16_t *dout, uint32_t ld_do,
                                 const float *lse, uint32_t B, uint32_t H, uint32_t S,
                                 float scale, int causal, uint16_t *dq, uint16_t *dk,
                                 uint16_t *dv, uint32_t ldd) {
  int rc = bwpp_ctx_enter(ctx);
  if (rc) return rc;
  if (!q || !k || !v || !o || !dout || !lse || !dq || !dk || !dv || ld_qkv < H * D ||
      ldo < H * D || ld_do < H * D || ldd < H * D)
    return bwpp_set_error(ctx, BWPP_CUDA_ERR_ARG, "attention bwd: bad args");
  if (B == 0 || H == 0 || S == 0) return BWPP_CUDA_OK;
  if (ldo != H * D)
    return bwpp_set_error(ctx, BWPP_CUDA_ERR_UNSUPPORTED, "attention bwd: O must be dense");
  float *delta = (float *)bwpp_ctx_workspace(ctx, sizeof(float) * (size_t)B * H * S);
  if (!delta) return BWPP_CUDA_ERR_NOMEM;
  if (ld_do != H * D)
    return bwpp_set_error(ctx, BWPP_CUDA_ERR_UNSUPPORTED, "attention bwd: dO must be dense");
  rc = bwpp_attn_delta(ctx, dout, o, delta, B, S, H, D);
  if (rc) return rc;
  return bwpp_attention_bwd_train(ctx, q, k, v, ld_qkv, dout, ld_do, lse, delta, B, H, S, scale,
                                  causal, dq, dk, dv, ldd);
}

}  // extern "C"
