// Fused matmul (+bias, +SiLU, +residual) on sm_100a tensor cores.
//
// C[M,N] = epilogue(A[M,K] * B[K,N]), A and B bf16, fp32 accumulation.
// epilogue: +bias[N], then SiLU, then +residual[M,N] (fp32), each optional
// (bias before SiLU as in runtime/cpu/bwpp_cpu_ref.c:26-31 and
// compiler/codegen_metal.c:426-431); C is written as fp32 or bf16.
// Operand layouts (template): A K-major (a[m*lda+k]) or MN-major (a[k*lda+m]),
// B MN-major (b[k*ldb+n], the reference's row-major B) or K-major
// (b[n*ldb+k], i.e. a transposed weight).  The MN-major forms let the
// autodiff products (dX = dY W^T, dW = X^T dY) run without transposes.
//
// Persistent, warp-specialised kernel (320 threads per CTA), in two forms:
//   CTA pair (cluster of 2, tcgen05 cta_group::2), used when M > 128: the
//     pair computes a 256 x 256 tile; each CTA loads 128 rows of A and 128
//     columns of B per K step (32 KB, 6-stage ring) into its own shared
//     memory, so operand traffic per SM is 2/3 of the single-CTA form.  The
//     TMA bytes of both CTAs count on rank 0's "full" barrier; rank 0's single
//     MMA thread issues M=256 N=256 K=16 MMAs and commits to the barriers of
//     both CTAs; each CTA's epilogue drains its own 128 TMEM lanes and
//     arrives on rank 0's "accumulator empty" barrier.
//   single CTA: 128 x 256 tiles, 48 KB per K step, 4-stage ring.
// Roles:
//   warp 0       TMA producer, 128-byte swizzle
//   warp 1       TMEM allocator + single-thread tcgen05.mma issuer; commits
//                free the smem stage / publish the accumulator
//   warps 2..9   epilogue, two warps per TMEM lane quarter taking alternate
//                32-column chunks: tcgen05.ld 32 lanes x 32 columns, +bias
//                (held in registers per tile, shuffled out), SiLU, +residual,
//                swizzled smem staging, TMA store.  One warp per quarter left
//                the SiLU latency-bound (12 us per fp32 tile, 7.6 us now).
//                The arithmetic runs as paired fp32 operations (add / mul
//                .f32x2): the MMA thread shares a sub-partition with two
//                epilogue warps, and their issue slots slow its MMA stream
//                (a variant with more epilogue instructions ran 2% slower).
// Two 256-column fp32 accumulators in TMEM (512 columns): the epilogue of
// tile i overlaps the main loop of tile i+1.  Tiles are rasterised in groups
// of 8 M-blocks so CTAs running together share B panels in L2.
// The main loop is bound by operand traffic from L2 into shared memory:
// a CTA loads 32 KB per 64-deep K step of a pair tile at about 80 GB/s per
// SM (~400 ns) against ~340 ns of MMA at the 1.5 GHz the part runs at under
// this load (ncu: tensor pipe 82% active), so the tile shape, not the MMA
// issue rate, sets the kernel's speed.
// The wave tail is cut into K parts that run in one round (see GemmWork).
//
// Every wait is bounded (BWPP_WAIT_LIMIT_NS); an expired wait records
// BWPP_CUDA_ERR_TIMEOUT, all roles unwind, TMEM is freed and the kernel ends.
//
// Shapes the TMA path cannot describe (row pitch not a multiple of 16 bytes,
// unaligned pointers, K == 0) run on a CUDA-core kernel instead.
#include <stdlib.h>

#include "bwpp_cuda_internal.cuh"

namespace {

constexpr int BM = 128, BN = 256, BK = 64;  // BM: rows per CTA; BN: accumulator width
constexpr int A_STAGE = BM * BK * 2;        // 16 KB
constexpr int B_SUB = 64 * BK * 2;          // 8 KB: 64 MN-columns x 64 K-rows
constexpr int EPI_WARPS = 8;   // two per TMEM lane quarter
constexpr int EPI_COLS = 32;                // columns per TMEM load / store
constexpr int EPI_BUF = 32 * EPI_COLS * 4;  // 4 KB: 32 rows x 128 B
constexpr int THREADS = 64 + 32 * EPI_WARPS;
constexpr uint32_t TMEM_COLS = 2 * BN;
constexpr uint32_t GROUP_M = 8;

// PAIR: a cluster of two CTAs computes a 256 x 256 tile with cta_group::2
// MMAs; each CTA loads 128 rows of A and 128 columns of B per K step (32 KB,
// six stages).  Single CTA: 128 x 256 tiles, 128 rows of A and 256 columns of
// B per K step (48 KB, four stages).
template <bool PAIR>
struct GemmCfg {
  static constexpr int BN_LOAD = PAIR ? 128 : 256;  // B columns this CTA loads
  static constexpr int STAGES = PAIR ? 6 : 4;
  static constexpr int B_STAGE = BN_LOAD * BK * 2;
  static constexpr int OFF_B = STAGES * A_STAGE;
  static constexpr int OFF_C = OFF_B + STAGES * B_STAGE;
  static constexpr int OFF_BAR = OFF_C + EPI_WARPS * EPI_BUF;  // one staging buffer per warp
  static constexpr int SMEM_ALLOC = OFF_BAR + 256 + 1024;  // + slack for 1024-B alignment
  static constexpr uint32_t TILE_M = PAIR ? 2 * BM : BM;
  static_assert(SMEM_ALLOC <= 232448, "exceeds the 227 KB opt-in limit");
  static_assert((2 * STAGES + 5) * 8 + 8 <= 256, "barrier block");
};

struct GemmEpi {
  const float *bias;      // [N] or nullptr
  const void *residual;   // [M, ldr] added last, or nullptr: fp32, or 16-bit per res16
  uint32_t ldr;
  int silu;
  int out_bf16;           // 16-bit output (bf16, or f16 when out_f16)
  int out_f16;
  int res16;              // residual element type: 0 fp32, 1 bf16, 2 f16
  // SwiGLU backward (glu != nullptr): the product is d(a) for a = silu(gate)
  // * up; glu holds [gate | up] bf16 rows (gate column f, up column glu_F + f,
  // pitch ldglu).  C receives d(gate) (bf16), glu_up_out d(up) (same pitch).
  const uint16_t *glu;
  uint16_t *glu_up_out;
  uint32_t ldglu, glu_F;
  // 1: the residual operand multiplies instead of adding (the gate of a
  // SwiGLU: silu(A B + bias) * R)
  int res_mul;
  };

// Work of a launch, handed out round-robin to `workers` workers (CTA pairs,
// or CTAs): worker w takes items w, w + workers, w + 2 workers, ...
// Items [0, items) are tiles in rasterised order.  Items below split_begin
// are whole tiles; from split_begin on, each remaining tile is cut into two N
// halves (MMA N = BN / 2), so a short last wave spreads over twice as many
// workers.  Item i >= split_begin is half (i - split_begin) % 2 of tile
// split_begin + (i - split_begin) / 2.
// Split tail (sk_parts > 1): the sk_tiles tiles after the full waves are cut
// into sk_parts K ranges, and items [items, items + sk_tiles * sk_parts)
// hold them part-major (all tiles' part 0, then all tiles' part 1, ...);
// sk_tiles * sk_parts <= workers, so the whole tail is normally one round,
// each part its worker's last item.  The tile's output is shared out like a
// reduce-scatter: an epilogue warp's chunks fall into sk_parts classes
// (chunk k is in class k % sk_parts), and each class is finished by the part
// that reaches it last.  A part visits the classes in the order part + 1,
// part + 2, ..., part (its "own" class last).  At each class it counts
// itself in (an epoch-tagged arrival counter); if others are still to come,
// it writes its fp32 partials of that class to its slot of `partials` and
// counts them written; the last to arrive instead owns the class: once the
// written count shows every other part's partials, it adds them (in part
// order) to its own accumulator and runs the epilogue on those chunks.
// A part waits only for parts that have already arrived, so they are
// running and finish their writes on their own: the split tail needs no
// two CTAs resident at the same time (kernels of other streams may hold
// SMs), and when all parts run together each ends up owning its own class.
struct GemmWork {
  uint32_t split_begin;
  uint32_t items;
  uint32_t workers;
  uint32_t sk_tile0;   // first split tile (= items)
  uint32_t sk_tiles;   // 0: no split tail
  uint32_t sk_parts;
  uint32_t split_first;  // 1: the split parts are every worker's first item, so
                         // their hand-off overlaps the whole tiles after them
  uint32_t epoch;      // tag of this launch's counts (counter high word)
  float *partials;     // [slot][TILE_M][BN] fp32, in TMEM chunk order
  unsigned long long *counters;  // [slot][2 CTAs][EPI_WARPS][arrived, written]
};

// One work item: a tile (or tile half) and the K blocks [kb0, kb1) of it.
struct GemmItem {
  uint32_t mb, nb, n_off, wn, kb0, kb1;
  uint32_t role;       // 0 whole tile (or half), 3 split part
  uint32_t part;       // split part: its K range index
  uint32_t slot;       // split part: slot of part 0 of its tile (part p: slot + p;
                       // class c's counters: slot + c)
};

__device__ __forceinline__ void tile_coords(uint32_t t, uint32_t tiles_m,
                                            uint32_t tiles_n, uint32_t &mb,
                                            uint32_t &nb) {
  const uint32_t per_group = GROUP_M * tiles_n;
  const uint32_t g = t / per_group;
  const uint32_t first_m = g * GROUP_M;
  const uint32_t gm = min(GROUP_M, tiles_m - first_m);
  const uint32_t r = t - g * per_group;
  mb = first_m + r % gm;
  nb = r / gm;
}

// The item with round-robin index `it`; false past the last item.
__device__ __forceinline__ bool get_item(const GemmWork &w, uint32_t tiles_m, uint32_t tiles_n,
                                         uint32_t num_kb, uint32_t it, GemmItem &x) {
  const uint32_t nsplit = w.sk_tiles * w.sk_parts;
  // split parts come first (split_first) or after the whole tiles
  const bool split = w.split_first ? it < nsplit : it >= w.items;
  if (!split) {
    const uint32_t wi = w.split_first ? it - nsplit : it;
    if (wi >= w.items) return false;
    uint32_t t = wi, half = 0;
    x.wn = BN;
    if (wi >= w.split_begin) {
      t = w.split_begin + (wi - w.split_begin) / 2;
      half = (wi - w.split_begin) & 1;
      x.wn = BN / 2;
    }
    tile_coords(t, tiles_m, tiles_n, x.mb, x.nb);
    x.n_off = half * (BN / 2);
    x.kb0 = 0;
    x.kb1 = num_kb;
    x.role = 0;
    x.part = 0;
    x.slot = 0;
    return true;
  }
  const uint32_t j = w.split_first ? it : it - w.items;
  if (j >= nsplit) return false;
  const uint32_t part = j / w.sk_tiles, tr = j - part * w.sk_tiles;
  tile_coords(w.sk_tile0 + tr, tiles_m, tiles_n, x.mb, x.nb);
  x.n_off = 0;
  x.wn = BN;
  x.kb0 = part * num_kb / w.sk_parts;
  x.kb1 = (part + 1) * num_kb / w.sk_parts;
  x.role = 3;
  x.part = part;
  x.slot = tr * w.sk_parts;
  return true;
}

template <bool A_MN, bool B_MN, bool PAIR>
__global__ void __launch_bounds__(THREADS, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA,
                   const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmC, const GemmEpi epi,
                   uint32_t M, uint32_t N, uint32_t K, uint32_t ab_f16, const GemmWork work,
                   int *status) {
  using Cfg = GemmCfg<PAIR>;
  constexpr int STAGES = Cfg::STAGES;
  // A and B both bf16, or both f16 (the half ABI)
  const uint32_t IDESC =
      make_idesc_f32acc(Cfg::TILE_M, BN, A_MN ? 1u : 0u, B_MN ? 1u : 0u, ab_f16);
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t *smem = smem_raw + ((1024u - (raw & 1023u)) & 1023u);
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + Cfg::OFF_BAR);
  uint64_t *empty = full + STAGES;
  uint64_t *tfull = empty + STAGES;
  uint64_t *tempty = tfull + 2;
  uint64_t *drain = tempty + 2;
  uint32_t *tmem_holder = reinterpret_cast<uint32_t *>(drain + 1);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // rank 0 of a pair issues the MMAs and owns the barriers both CTAs feed
  const uint32_t rank = PAIR ? cluster_ctarank() : 0u;
  const uint32_t worker = PAIR ? cluster_id_x() : blockIdx.x;
  const uint32_t tiles_m = (M + Cfg::TILE_M - 1) / Cfg::TILE_M, tiles_n = (N + BN - 1) / BN;
  const uint32_t num_kb = (K + BK - 1) / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], PAIR ? 2 * EPI_WARPS : EPI_WARPS);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
    prefetch_tmap(&tmC);
  }
  if (warp == 1) {
    if constexpr (PAIR) {
      tmem_alloc_pair(tmem_holder, TMEM_COLS);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(tmem_holder, TMEM_COLS);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  if constexpr (PAIR) cluster_sync_all(); else __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      uint32_t stage = 0, phase = 0;
      GemmItem x;
      for (uint32_t it = worker;
           !*abort_flag && get_item(work, tiles_m, tiles_n, num_kb, it, x); it += work.workers) {
        // In a pair each CTA holds wn / 2 of the MMA's columns.
        const int32_t row0 = (int32_t)(x.mb * Cfg::TILE_M + rank * BM);
        const int32_t col0 = (int32_t)(x.nb * BN + x.n_off + rank * (PAIR ? x.wn / 2 : 0));
        const uint32_t b_boxes = (PAIR ? x.wn / 2 : x.wn) / 64;
        for (uint32_t kb = x.kb0; kb < x.kb1; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, status)) {
            *abort_flag = 1;
            break;
          }
          // the pair's bytes all count on rank 0's barrier; a half tile
          // loads half of this CTA's B columns
          if (rank == 0)
            mbar_arrive_expect_tx(&full[stage],
                                  (PAIR ? 2 : 1) * (A_STAGE + (b_boxes * 64) * BK * 2));
          uint32_t fbar = 0;
          if constexpr (PAIR) fbar = cluster_addr(&full[stage], 0);
          auto load = [&](void *dst, const CUtensorMap *map, int32_t x, int32_t y) {
            if constexpr (PAIR) tma_load_2d_pair(dst, map, fbar, x, y);
            else tma_load_2d(dst, map, &full[stage], x, y);
          };
          uint8_t *sa = smem + stage * A_STAGE;
          uint8_t *sb = smem + Cfg::OFF_B + stage * Cfg::B_STAGE;
          const int32_t k0 = (int32_t)(kb * BK);
          if (!A_MN) {
            load(sa, &tmA, k0, row0);  // [128 rows of M] x [64 K]: one 16 KB box
          } else {
#pragma unroll
            for (int j = 0; j < BM / 64; ++j)  // [64 K rows] x [64 M] boxes
              load(sa + j * B_SUB, &tmA, row0 + j * 64, k0);
          }
          // B in boxes of 64 columns: MN-major [64 K rows] x [64 N], K-major
          // [64 N rows] x [64 K] (stacked boxes form one swizzled panel)
          for (uint32_t j = 0; j < b_boxes; ++j) {
            if (B_MN) load(sb + j * B_SUB, &tmB, col0 + (int32_t)j * 64, k0);
            else load(sb + j * B_SUB, &tmB, k0, col0 + (int32_t)j * 64);
          }
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------- MMA issuer
    if (lane == 0 && rank == 0) {
      // commit: arrive on this CTA's barrier and, for a pair, the peer's copy
      auto commit = [&](uint64_t *bar) {
        if constexpr (PAIR) {
          tc_commit_pair(smem_u32(bar));
          tc_commit_pair(cluster_addr(bar, 1));
        } else {
          tc_commit(bar);
        }
      };
      uint32_t stage = 0, phase = 0, acc = 0, acc_phase = 0;
      GemmItem x;
      for (uint32_t it = worker;
           !*abort_flag && get_item(work, tiles_m, tiles_n, num_kb, it, x); it += work.workers) {
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1, status)) {
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        const uint32_t idesc = x.wn == BN ? IDESC
            : make_idesc_f32acc(Cfg::TILE_M, BN / 2, A_MN ? 1u : 0u, B_MN ? 1u : 0u, ab_f16);
        bool ok = true;
        for (uint32_t kb = x.kb0; kb < x.kb1; ++kb) {
          if (!mbar_wait(&full[stage], phase, status)) {
            *abort_flag = 1;
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = smem_u32(smem + stage * A_STAGE);
          const uint32_t b0 = smem_u32(smem + Cfg::OFF_B + stage * Cfg::B_STAGE);
#pragma unroll
          for (int ks = 0; ks < BK / 16; ++ks) {
            // K-major, 128-B swizzle: a K step of 16 bf16 is 32 bytes inside
            // the swizzle atom; 8-row groups 1 KB apart (SBO).
            // MN-major, 128-B swizzle: 64-element MN atoms 8 KB apart (LBO),
            // 8-row K groups 1 KB apart (SBO); a K step of 16 rows is 2 KB.
            const uint64_t ad = A_MN ? make_smem_desc(a0 + ks * 2048, B_SUB, 1024, BWPP_SWIZZLE_128B)
                                     : make_smem_desc(a0 + ks * 32, 16, 1024, BWPP_SWIZZLE_128B);
            const uint64_t bd = B_MN ? make_smem_desc(b0 + ks * 2048, B_SUB, 1024, BWPP_SWIZZLE_128B)
                                     : make_smem_desc(b0 + ks * 32, 16, 1024, BWPP_SWIZZLE_128B);
            const uint32_t accum = (kb != x.kb0 || ks != 0) ? 1u : 0u;
            if constexpr (PAIR) tc_mma_f16_ss_pair(d_tmem, ad, bd, idesc, accum);
            else tc_mma_f16_ss(d_tmem, ad, bd, idesc, accum);
          }
          commit(&empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        commit(&tfull[acc]);
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1;
      }
      // every MMA issued by this thread has finished before TMEM is freed
      if constexpr (PAIR) tc_commit_pair(smem_u32(drain)); else tc_commit(drain);
      mbar_wait(drain, 0, status);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const int ew = warp - 2;
    const int sub = ew >> 2;  // the two warps of a quarter take alternate chunks
    uint8_t *stage_c = smem + Cfg::OFF_C + ew * EPI_BUF;
    uint32_t acc = 0, acc_phase = 0;
    const int out16 = epi.out_bf16;
    const int cw = out16 ? 64 : 32;  // chunk: 32 rows x 128 bytes of output
    const int per = out16 ? 2 : 1;   // 32-column accumulator parts per chunk
    const uint32_t tq = (uint32_t)(q * 32) << 16;  // TMEM lane base of this warp
    // accumulator column of this warp's i-th 32-column part (chunks sub,
    // sub + 2, ...)
    auto part_col = [&](int i) { return (uint32_t)((sub + 2 * (i / per)) * cw + (i % per) * 32); };
    // partial slots: [slot][CTA rank][32-column chunk][float4 index][row];
    // one warp's 32 rows of one float4 index are 512 contiguous bytes
    auto slot_rows = [&](uint32_t sl) {
      return work.partials + (size_t)sl * Cfg::TILE_M * BN + (size_t)rank * BM * BN +
             (size_t)(q * 32 + lane) * 4;
    };
    // class counters of a split tile: [slot][CTA rank][epilogue warp][arrived, written]
    auto counter_of = [&](uint32_t sl) {
      return work.counters + ((size_t)(sl * 2 + rank) * EPI_WARPS + ew) * 2;
    };
    GemmItem x;
    for (uint32_t it = worker;
         !*abort_flag && get_item(work, tiles_m, tiles_n, num_kb, it, x); it += work.workers) {
      const uint32_t mb = x.mb, nb = x.nb, n_off = x.n_off, wn = x.wn;
      // This item's bias, loaded before the accumulator is ready: lane l
      // holds columns 8l .. 8l+7 of the item, handed out by shuffles.
      float breg[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      if (epi.bias) {
        const uint32_t bc = nb * BN + n_off + (uint32_t)lane * 8;
        if (bc + 8 <= N) {
          const float4 b0 = __ldg(reinterpret_cast<const float4 *>(epi.bias + bc));
          const float4 b1 = __ldg(reinterpret_cast<const float4 *>(epi.bias + bc) + 1);
          breg[0] = b0.x; breg[1] = b0.y; breg[2] = b0.z; breg[3] = b0.w;
          breg[4] = b1.x; breg[5] = b1.y; breg[6] = b1.z; breg[7] = b1.w;
        } else {
#pragma unroll
          for (int i = 0; i < 8; ++i) breg[i] = bc + i < N ? __ldg(epi.bias + bc + i) : 0.f;
        }
      }
      if (!mbar_wait(&tfull[acc], acc_phase, status)) {
        *abort_flag = 1;
        break;
      }
      tc_fence_after();
      // chunks with columns below N; this warp takes chunks sub, sub + 2, ...
      const uint32_t first_col = nb * BN + n_off;
      const int nchunks = (int)min(wn / cw, (N - first_col + cw - 1) / cw);
      const int my_chunks = nchunks > sub ? (nchunks - sub + 1) / 2 : 0;
      // split part: this warp's chunk k is in class k % parts; the part that
      // reaches a class last finishes it (see GemmWork)
      const bool split = x.role == 3;
      const int parts = split ? (int)work.sk_parts : 1;
      const int me = split ? (int)x.part : 0;
      const uint32_t n_contrib = split ? (uint32_t)parts - 1 : 0;
      auto class_chunks = [&](int c) {
        return my_chunks > c ? (my_chunks - c + parts - 1) / parts : 0;
      };
      uint32_t owned = split ? 0u : 1u;  // bit c: this part finishes class c
      if (split) {
        float *dst = slot_rows(x.slot + x.part);
        // Classes whose partials this part has stored but not yet counted
        // written: one fence, then lane c counts class c (the counters'
        // round trips to L2, slow while other tiles' main loops run, overlap).
        uint32_t unsignalled = 0;
        auto signal_written = [&]() {
          if (!__any_sync(0xffffffffu, unsignalled != 0)) return;
          __threadfence();
          __syncwarp();
          if (lane < parts && (unsignalled >> lane & 1u))
            epoch_arrive(counter_of(x.slot + lane) + 1, work.epoch);
          __syncwarp();
          unsignalled = 0;
        };
        for (int i = 1; i <= parts; ++i) {
          const int c = (me + i) % parts;  // this part's own class last
          if (class_chunks(c) == 0) continue;
          // before the own class, let the owners of the others go on
          if (i == parts) signal_written();
          unsigned long long *ctr = counter_of(x.slot + c);
          uint32_t before = 0;
          if (lane == 0) before = epoch_arrive(ctr, work.epoch);
          before = __shfl_sync(0xffffffffu, before, 0);
          if (before == (uint32_t)parts - 1) {  // every other part is in: finish it here
            owned |= 1u << c;
            continue;
          }
          // others still to come: this part's partial sums of class c to its
          // slot (counted written by signal_written, every lane's stores first)
          unsignalled |= 1u << c;
          for (int k = c; k < my_chunks; k += parts) {
            for (int h = 0; h < per; ++h) {
              const uint32_t cc = part_col(k * per + h);
              uint32_t w[32];
              tmem_ld_32x32b_x32(tmem_base + tq + acc * BN + cc, w);
              tc_wait_ld(w);
#pragma unroll
              for (int j = 0; j < 8; ++j)
                __stcg(reinterpret_cast<float4 *>(dst + (size_t)(cc / 32) * BM * 32 + j * BM * 4),
                       make_float4(__uint_as_float(w[4 * j]), __uint_as_float(w[4 * j + 1]),
                                   __uint_as_float(w[4 * j + 2]), __uint_as_float(w[4 * j + 3])));
            }
          }
        }
        signal_written();
      }
      // the other parts' slots, in part order
      auto contrib_slot = [&](uint32_t c) { return x.slot + (c < (uint32_t)me ? c : c + 1); };
      // Partials are staged through shared memory with per-thread async
      // copies, `depth` parts ahead, so many loads are in flight.  The
      // operand ring is free once this item's MMAs are done, as a split part
      // is always its worker's last item (checked; else plain loads).  Each
      // warp takes an eighth of the ring: `depth` x n_contrib blocks of 4 KB
      // ([float4 index][lane] x 16 B, each lane reads back its own).
      constexpr uint32_t RING_SHARE = Cfg::OFF_C / EPI_WARPS;
      int depth = 0;
      if (n_contrib) {
        GemmItem later;
        const int fit = (int)(RING_SHARE / (4096u * n_contrib));
        if (!get_item(work, tiles_m, tiles_n, num_kb, it + work.workers, later) && fit >= 1) {
          depth = fit < 8 ? fit : 8;
          fence_proxy_async_smem();  // the ring was last used by TMA and the tensor core
        }
      }
      const uint32_t pbuf = smem_u32(smem) + (uint32_t)ew * RING_SHARE;
      bool item_ok = true;
      for (int cls = 0; cls < parts && item_ok; ++cls) {
        if (!(owned >> cls & 1u)) continue;
        const int own_chunks = class_chunks(cls);
        const int own_parts = own_chunks * per;
        // accumulator column of this warp's t-th 32-column part of class cls
        auto own_col = [&](int t) { return part_col((cls + (t / per) * parts) * per + t % per); };
        int issued = 0;
        auto issue = [&](int t) {
          const uint32_t base = pbuf + (uint32_t)((t % depth) * n_contrib) * 4096u + lane * 16u;
          const uint32_t pc = own_col(t) / 32;
          for (uint32_t c = 0; c < n_contrib; ++c) {
            const float *src = slot_rows(contrib_slot(c)) + (size_t)pc * BM * 32;
#pragma unroll
            for (int j = 0; j < 8; ++j) cp_async_16(base + c * 4096u + j * 512u, src + j * BM * 4);
          }
          cp_async_commit();
          ++issued;
        };
        if (n_contrib) {
          // the other parts have all arrived, so they are running: wait for
          // their partials of this class to be written
          bool ok = true;
          if (lane == 0) ok = epoch_wait(counter_of(x.slot + cls) + 1, work.epoch, n_contrib, status);
          if (!__shfl_sync(0xffffffffu, ok ? 1 : 0, 0)) {
            item_ok = false;
            break;
          }
          __syncwarp();  // lane 0's acquire orders the whole warp's loads below
          if (depth)
            for (int t = 0; t < depth && t < own_parts; ++t) issue(t);
        }
        const uint32_t row0 = mb * Cfg::TILE_M + rank * BM + q * 32;
        const uint32_t my_row = row0 + lane;
        for (int ko = 0; ko < own_chunks; ++ko) {
          const int k = cls + ko * parts;  // this warp's chunk index
          const uint32_t col0 = first_col + (uint32_t)(sub + 2 * k) * cw;
          uint32_t outw[32];
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            if (h == 1 && !out16) break;
            const int t = ko * per + h;           // this warp's owned-part index
            const uint32_t cs = col0 + h * 32;    // first column of this 32-wide part
            const uint32_t cc = cs - first_col;   // accumulator column
            uint32_t r[32];
            tmem_ld_32x32b_x32(tmem_base + tq + acc * BN + cc, r);
            tc_wait_ld(r);
            float v[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
            if (n_contrib) {
              const int pc = (int)(cc / 32);
              // The tile's sum is the left fold p0 + p1 + ... in part order,
              // this part's own accumulator taking its place, so the result
              // does not depend on which part finished the class.
              auto fold = [&](auto contrib) {
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                  float4 sum = me == 0 ? make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2],
                                                     v[4 * j + 3])
                                       : contrib(0u, j);
#pragma unroll 1
                  for (int pq = 1; pq < parts; ++pq) {
                    const float4 t4 = pq == me ? make_float4(v[4 * j], v[4 * j + 1],
                                                             v[4 * j + 2], v[4 * j + 3])
                                               : contrib((uint32_t)(pq < me ? pq : pq - 1), j);
                    sum.x += t4.x;
                    sum.y += t4.y;
                    sum.z += t4.z;
                    sum.w += t4.w;
                  }
                  v[4 * j] = sum.x;
                  v[4 * j + 1] = sum.y;
                  v[4 * j + 2] = sum.z;
                  v[4 * j + 3] = sum.w;
                }
              };
              if (depth) {
                cp_async_wait_pending(issued - (t + 1));
                const uint8_t *blk = smem + (size_t)ew * RING_SHARE +
                                     (size_t)((t % depth) * n_contrib) * 4096u + lane * 16u;
                fold([&](uint32_t c, int j) {
                  return *reinterpret_cast<const float4 *>(blk + c * 4096u + j * 512u);
                });
                if (t + depth < own_parts) issue(t + depth);  // into the block just read
              } else if (n_contrib <= 2) {
                // Straight from L2, each load a round trip that the next
                // tile's running main loop makes slow: both contributors'
                // float4s of half the part are requested before any is
                // added (two round trips per part).  Same left fold in part
                // order: (a + b) + c.
                const float *src0 = slot_rows(contrib_slot(0)) + (size_t)pc * BM * 32;
                const float *src1 = slot_rows(contrib_slot(n_contrib > 1 ? 1u : 0u)) + (size_t)pc * BM * 32;
#pragma unroll
                for (int hh = 0; hh < 2; ++hh) {
                  float4 pre[2][4];
#pragma unroll
                  for (int j = 0; j < 4; ++j) {
                    pre[0][j] = __ldcg(reinterpret_cast<const float4 *>(src0 + (4 * hh + j) * BM * 4));
                    if (n_contrib > 1)
                      pre[1][j] = __ldcg(reinterpret_cast<const float4 *>(src1 + (4 * hh + j) * BM * 4));
                  }
#pragma unroll
                  for (int jj = 0; jj < 4; ++jj) {
                    const int j = 4 * hh + jj;
                    const float4 own = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
                    const float4 a = me == 0 ? own : pre[0][jj];
                    const float4 b = me == 0 ? pre[0][jj] : (me == 1 ? own : pre[1][jj]);
                    float4 s = make_float4(a.x + b.x, a.y + b.y, a.z + b.z, a.w + b.w);
                    if (parts == 3) {
                      const float4 c3 = me == 2 ? own : pre[1][jj];
                      s = make_float4(s.x + c3.x, s.y + c3.y, s.z + c3.z, s.w + c3.w);
                    }
                    v[4 * j] = s.x;
                    v[4 * j + 1] = s.y;
                    v[4 * j + 2] = s.z;
                    v[4 * j + 3] = s.w;
                  }
                }
              } else {
                fold([&](uint32_t c, int j) {
                  const float *src = slot_rows(contrib_slot(c)) + (size_t)pc * BM * 32;
                  return __ldcg(reinterpret_cast<const float4 *>(src + j * BM * 4));
                });
              }
            }
            if (epi.bias) {
              // paired adds: one issue slot for two columns (the issuing
              // thread of the MMAs shares its sub-partition with epilogue warps)
#pragma unroll
              for (int j = 0; j < 32; j += 2)
                f2unpack(f2add(f2pack(v[j], v[j + 1]),
                               f2pack(__shfl_sync(0xffffffffu, breg[j & 7], (int)(cc >> 3) + (j >> 3)),
                                      __shfl_sync(0xffffffffu, breg[(j + 1) & 7],
                                                  (int)(cc >> 3) + ((j + 1) >> 3)))),
                         v[j], v[j + 1]);
            }
            if (epi.glu && my_row < M) {
              // SwiGLU backward: with s = sigmoid(gate), d(gate) = v up s (1 +
              // gate (1 - s)) replaces v; d(up) = v gate s is stored here
              const uint16_t *gr = epi.glu + (size_t)my_row * epi.ldglu + cs;
              const uint16_t *ur = gr + epi.glu_F;
              uint16_t *dur = epi.glu_up_out + (size_t)my_row * epi.ldglu + cs;
              if (cs + 32 <= N) {
                uint32_t gw[16], uw[16], dw[16];
#pragma unroll
                for (int k4 = 0; k4 < 4; ++k4) {
                  const uint4 tg = *reinterpret_cast<const uint4 *>(gr + 8 * k4);
                  const uint4 tu = *reinterpret_cast<const uint4 *>(ur + 8 * k4);
                  gw[4 * k4] = tg.x; gw[4 * k4 + 1] = tg.y; gw[4 * k4 + 2] = tg.z; gw[4 * k4 + 3] = tg.w;
                  uw[4 * k4] = tu.x; uw[4 * k4 + 1] = tu.y; uw[4 * k4 + 2] = tu.z; uw[4 * k4 + 3] = tu.w;
                }
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                  float du[2];
#pragma unroll
                  for (int e = 0; e < 2; ++e) {
                    const float g = load16<false>((uint16_t)(gw[i] >> (16 * e)));
                    const float u = load16<false>((uint16_t)(uw[i] >> (16 * e)));
                    const float sg = __fdividef(1.0f, 1.0f + __expf(-g));
                    const float d = v[2 * i + e];
                    v[2 * i + e] = d * u * sg * (1.0f + g * (1.0f - sg));
                    du[e] = d * g * sg;
                  }
                  dw[i] = pack2_16<false>(du[0], du[1]);
                }
#pragma unroll
                for (int k4 = 0; k4 < 4; ++k4)
                  *reinterpret_cast<uint4 *>(dur + 8 * k4) =
                      make_uint4(dw[4 * k4], dw[4 * k4 + 1], dw[4 * k4 + 2], dw[4 * k4 + 3]);
              } else {
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                  if (cs + j >= N) continue;
                  const float g = load16<false>(gr[j]), u = load16<false>(ur[j]);
                  const float sg = __fdividef(1.0f, 1.0f + __expf(-g));
                  const float d = v[j];
                  v[j] = d * u * sg * (1.0f + g * (1.0f - sg));
                  dur[j] = (uint16_t)(pack2_16<false>(d * g * sg, 0.0f) & 0xFFFFu);
                }
              }
            }
            if (epi.silu) {
#pragma unroll
              for (int j = 0; j < 32; j += 2)
                f2unpack(bwpp_silu_f2(f2pack(v[j], v[j + 1])), v[j], v[j + 1]);
            }
            if (epi.residual && my_row < M && epi.res16) {
              // 16-bit residual (read before this chunk is stored: may alias C)
              const uint16_t *rr =
                  static_cast<const uint16_t *>(epi.residual) + (size_t)my_row * epi.ldr + cs;
              const bool f16 = epi.res16 == 2;
              if (cs + 32 <= N && (epi.ldr & 7) == 0 &&
                  (reinterpret_cast<uintptr_t>(epi.residual) & 15) == 0) {
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                  const uint4 t = *reinterpret_cast<const uint4 *>(rr + 8 * j);
                  const uint32_t w[4] = {t.x, t.y, t.z, t.w};
#pragma unroll
                  for (int e = 0; e < 4; ++e) {
                    const uint16_t lo = (uint16_t)(w[e] & 0xFFFFu), hi = (uint16_t)(w[e] >> 16);
                    const float r0 = f16 ? load16<true>(lo) : load16<false>(lo);
                    const float r1 = f16 ? load16<true>(hi) : load16<false>(hi);
                    const uint64_t vv = f2pack(v[8 * j + 2 * e], v[8 * j + 2 * e + 1]);
                    const uint64_t rr2 = f2pack(r0, r1);
                    f2unpack(epi.res_mul ? f2mul(vv, rr2) : f2add(vv, rr2), v[8 * j + 2 * e],
                             v[8 * j + 2 * e + 1]);
                  }
                }
              } else {
#pragma unroll
                for (int j = 0; j < 32; ++j)
                  if (cs + j < N) {
                    const float r = f16 ? load16<true>(rr[j]) : load16<false>(rr[j]);
                    v[j] = epi.res_mul ? v[j] * r : v[j] + r;
                  }
              }
            } else if (epi.residual && my_row < M) {
              const float *rr = static_cast<const float *>(epi.residual) + (size_t)my_row * epi.ldr + cs;
              if (cs + 32 <= N && (epi.ldr & 3) == 0 &&
                  (reinterpret_cast<uintptr_t>(epi.residual) & 15) == 0) {
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                  const float4 t = *reinterpret_cast<const float4 *>(rr + 4 * j);
                  const uint64_t v01 = f2pack(v[4 * j], v[4 * j + 1]), t01 = f2pack(t.x, t.y);
                  const uint64_t v23 = f2pack(v[4 * j + 2], v[4 * j + 3]), t23 = f2pack(t.z, t.w);
                  f2unpack(epi.res_mul ? f2mul(v01, t01) : f2add(v01, t01), v[4 * j], v[4 * j + 1]);
                  f2unpack(epi.res_mul ? f2mul(v23, t23) : f2add(v23, t23), v[4 * j + 2], v[4 * j + 3]);
                }
              } else {
#pragma unroll
                for (int j = 0; j < 32; ++j)
                  if (cs + j < N) v[j] = epi.res_mul ? v[j] * rr[j] : v[j] + rr[j];
              }
            }
            if (out16) {
#pragma unroll
              for (int j = 0; j < 16; ++j)
                outw[h * 16 + j] = epi.out_f16 ? pack2_16<true>(v[2 * j], v[2 * j + 1])
                                               : pack2_16<false>(v[2 * j], v[2 * j + 1]);
            } else {
#pragma unroll
              for (int j = 0; j < 32; ++j) outw[j] = __float_as_uint(v[j]);
            }
          }
          // the previous store from this warp's buffer has finished reading it
          if (lane == 0) tma_store_wait_read<0>();
          __syncwarp();
          uint8_t *sc = stage_c;
#pragma unroll
          for (int j = 0; j < 8; ++j)
            *reinterpret_cast<uint4 *>(sc + lane * 128 + ((j ^ (lane & 7)) << 4)) =
                make_uint4(outw[4 * j], outw[4 * j + 1], outw[4 * j + 2], outw[4 * j + 3]);
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0 && row0 < M) {
            tma_store_2d(&tmC, sc, (int32_t)col0, (int32_t)row0);
            tma_store_commit();
          }
        }
        if (depth) cp_async_wait_pending(0);  // the ring is reused by the next class
      }  // classes
      if (!item_ok) {
        *abort_flag = 1;
        break;
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if constexpr (PAIR) mbar_arrive_cluster(cluster_addr(&tempty[acc], 0));
        else mbar_arrive(&tempty[acc]);
      }
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1;
    }
    if (lane == 0) tma_store_wait_all<0>();
  }

  // Neither CTA of a pair leaves (or frees TMEM) while the other may still
  // touch its barriers: every wait above is bounded, so both arrive here.
  tc_fence_before();
  if constexpr (PAIR) cluster_sync_all(); else __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    if constexpr (PAIR) tmem_dealloc_pair(tmem_base, TMEM_COLS);
    else tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------
// CUDA-core fallback for shapes TMA cannot describe (and K == 0)
// ---------------------------------------------------------------------------
constexpr int ST = 16;

__global__ void gemm_simt_kernel(const uint16_t *__restrict__ a,
                                 const uint16_t *__restrict__ b, void *c,
                                 uint32_t M, uint32_t N, uint32_t K, uint32_t lda,
                                 uint32_t ldb, uint32_t ldc, int a_mn, int b_mn,
                                 const GemmEpi epi, int ab_f16) {
  __shared__ float As[ST][ST + 1], Bs[ST][ST + 1];
  const uint32_t row = blockIdx.y * ST + threadIdx.y;
  const uint32_t col = blockIdx.x * ST + threadIdx.x;
  auto bf = [ab_f16](uint16_t h) { return ab_f16 ? load16<true>(h) : load16<false>(h); };
  float acc = 0.0f;
  for (uint32_t k0 = 0; k0 < K; k0 += ST) {
    const uint32_t ka = k0 + threadIdx.x, kb = k0 + threadIdx.y;
    As[threadIdx.y][threadIdx.x] =
        (row < M && ka < K) ? bf(a_mn ? a[(size_t)ka * lda + row] : a[(size_t)row * lda + ka]) : 0.0f;
    Bs[threadIdx.y][threadIdx.x] =
        (kb < K && col < N) ? bf(b_mn ? b[(size_t)kb * ldb + col] : b[(size_t)col * ldb + kb]) : 0.0f;
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < ST; ++kk) acc += As[threadIdx.y][kk] * Bs[kk][threadIdx.x];
    __syncthreads();
  }
  if (row < M && col < N) {
    if (epi.bias) acc += epi.bias[col];
    if (epi.silu) acc = acc / (1.0f + expf(-acc));
    if (epi.residual) {
      const size_t ri = (size_t)row * epi.ldr + col;
      const uint16_t *r16 = static_cast<const uint16_t *>(epi.residual);
      const float r = epi.res16 == 0 ? static_cast<const float *>(epi.residual)[ri]
                      : epi.res16 == 2 ? load16<true>(r16[ri]) : load16<false>(r16[ri]);
      acc = epi.res_mul ? acc * r : acc + r;
    }
    if (epi.out_bf16) {
      const uint32_t w = epi.out_f16 ? pack2_16<true>(acc, 0.0f) : pack2_16<false>(acc, 0.0f);
      reinterpret_cast<uint16_t *>(c)[(size_t)row * ldc + col] = (uint16_t)(w & 0xFFFFu);
    } else {
      reinterpret_cast<float *>(c)[(size_t)row * ldc + col] = acc;
    }
  }
}

__global__ void cast_f32_bf16_kernel(const float *__restrict__ src,
                                     uint16_t *__restrict__ dst, uint32_t rows,
                                     uint32_t cols, uint32_t ld_src,
                                     uint32_t ld_dst) {
  const size_t n = (size_t)rows * cols;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x) {
    const size_t r = i / cols, cc = i % cols;
    const float x = src[r * ld_src + cc];
    uint32_t u = __float_as_uint(x);
    uint16_t h;
    if ((u & 0x7f800000u) == 0x7f800000u && (u & 0x007fffffu))
      h = (uint16_t)((u >> 16) | 0x0040u);  // quiet NaN
    else
      h = (uint16_t)((u + 0x7fffu + ((u >> 16) & 1u)) >> 16);  // nearest even
    dst[r * ld_dst + cc] = h;
  }
}

bool g_attr_set[8][64] = {};
int g_pair_clusters[4][64] = {};  // resident CTA pairs per device (0: not queried)

inline bool al16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Split-tail scratch of ctx: 2 * num_sms fp32 slots of BM x BN (a CTA-pair
// slot takes two of them; a launch uses at most cap slots) and, per slot, an
// (arrived, written) pair of 64-bit class counters for each of the 2 CTAs x
// 8 epilogue warps.  Allocated on first use; never when the caller owns the
// workspace (then GEMMs use the half-tile tail).
bool gemm_scratch(BwppCudaCtx *ctx) {
  if (ctx->gemm_partials) return true;
  if (ctx->user_workspace || ctx->gemm_scratch_failed) return false;
  const size_t slots = 2 * (size_t)ctx->num_sms;
  const size_t part_bytes = slots * BM * BN * sizeof(float);
  const size_t counter_bytes = slots * 2 * EPI_WARPS * 2 * sizeof(unsigned long long);
  void *p = nullptr;
  if (cudaMalloc(&p, part_bytes + counter_bytes) != cudaSuccess) {
    (void)cudaGetLastError();
    ctx->gemm_scratch_failed = 1;
    return false;
  }
  if (cudaMemsetAsync(static_cast<uint8_t *>(p) + part_bytes, 0, counter_bytes, ctx->stream) !=
      cudaSuccess) {
    (void)cudaGetLastError();
    cudaFree(p);
    ctx->gemm_scratch_failed = 1;
    return false;
  }
  ctx->gemm_partials = static_cast<float *>(p);
  ctx->gemm_counters = reinterpret_cast<unsigned long long *>(static_cast<uint8_t *>(p) + part_bytes);
  ctx->gemm_epoch = 0;
  return true;
}

// CTA pairs are used unless BWPP_GEMM_CTA_PAIR=0 (then every GEMM runs the
// single-CTA kernel).
bool pairs_enabled() {
  static const int on = [] {
    const char *e = getenv("BWPP_GEMM_CTA_PAIR");
    return (e && e[0] == '0') ? 0 : 1;
  }();
  return on != 0;
}

// Split parts run before the whole tiles unless BWPP_GEMM_SPLIT_FIRST=0.
bool split_first_enabled() {
  static const int on = [] {
    const char *e = getenv("BWPP_GEMM_SPLIT_FIRST");
    return (e && e[0] == '0') ? 0 : 1;
  }();
  return on != 0;
}

// Launches the tensor-core kernel.  Returns BWPP_CUDA_ERR_UNSUPPORTED (with
// nothing launched) when a CTA pair cannot be made resident, so the caller
// can take the single-CTA kernel.
//
// Wave tail: with `cap` tiles in flight (CTA pairs, or SMs) the last wave
// holds tiles % cap tiles.  Those tiles are cut into K parts in the same
// launch (GemmWork: split tail), so the tail takes a fraction of a tile's
// time; a GEMM of fewer tiles than cap is all tail.  (At 8 GPUs the
// 8192 x 4096 x 11008 GEMM leaves 1024 rows per GPU: 172 pair tiles, 2.3
// waves; the 24-tile tail runs as 3 x 24 third-tiles in one round.)  When
// no split applies (a tail of more than half a round, under 8 K blocks, or
// no scratch), a tail that fits twice into one round runs as N halves.
template <bool A_MN, bool B_MN, bool PAIR>
int launch_tc(BwppCudaCtx *ctx, const CUtensorMap &ta, const CUtensorMap &tb,
              const CUtensorMap &tcm, const GemmEpi &epi, uint32_t M, uint32_t N,
              uint32_t K, uint32_t ab_f16) {
  using Cfg = GemmCfg<PAIR>;
  auto kern = gemm_tc_kernel<A_MN, B_MN, PAIR>;
  const int v = (A_MN ? 2 : 0) + (B_MN ? 1 : 0);
  const int dev = ctx->device;
  if (dev >= 64) return bwpp_set_error(ctx, BWPP_CUDA_ERR_UNSUPPORTED, "gemm: device index >= 64");
  if (!g_attr_set[v + (PAIR ? 4 : 0)][dev]) {
    int rc = bwpp_check_cuda(ctx,
                             cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                  Cfg::SMEM_ALLOC),
                             "gemm smem attribute");
    if (rc) return rc;
    g_attr_set[v + (PAIR ? 4 : 0)][dev] = true;
  }
  const uint32_t tiles = ((M + Cfg::TILE_M - 1) / Cfg::TILE_M) * ((N + BN - 1) / BN);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = PAIR ? 2 : 1;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(ctx->num_sms & ~1), 1, 1);
  cfg.blockDim = dim3(THREADS, 1, 1);
  cfg.dynamicSmemBytes = Cfg::SMEM_ALLOC;
  cfg.stream = ctx->stream;
  cfg.attrs = attr;
  cfg.numAttrs = PAIR ? 1 : 0;
  uint32_t cap = (uint32_t)ctx->num_sms;
  if constexpr (PAIR) {
    int &pairs = g_pair_clusters[v][dev];
    if (pairs == 0) {
      int n = 0;
      if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess || n <= 0) {
        (void)cudaGetLastError();
        pairs = -1;
      } else {
        pairs = n;
      }
    }
    if (pairs < 0) return BWPP_CUDA_ERR_UNSUPPORTED;
    cap = (uint32_t)pairs;
  }
  const uint32_t full = tiles / cap, tail = tiles % cap;
  const uint32_t num_kb = (K + BK - 1) / BK;
  GemmWork w{};
  w.workers = cap;
  w.items = w.split_begin = full * cap;
  // Split tail: cut the `tail` tiles after the full waves into as many K
  // parts as fit in one round (tail * parts <= cap), at most 8, each at
  // least 4 K blocks.
  uint32_t parts = 1;
  if (tail > 0) {
    parts = cap / tail;
    if (parts > 8) parts = 8;
    while (parts > 1 && num_kb / parts < 4) --parts;
    if (parts > 1 && !gemm_scratch(ctx)) parts = 1;
  }
  if (parts > 1) {
    w.sk_tile0 = w.items;
    w.sk_tiles = tail;
    w.sk_parts = parts;
    w.split_first = split_first_enabled() ? 1u : 0u;
    w.epoch = ++ctx->gemm_epoch;
    if (w.epoch == 0) w.epoch = ++ctx->gemm_epoch;  // 0 is the counters' initial tag
    w.partials = ctx->gemm_partials;
    w.counters = ctx->gemm_counters;
  } else {
    // whole tiles; a tail that fits twice into one round runs as N halves
    const bool halve = tail > 0 && tail * 2 <= cap;
    w.split_begin = halve ? full * cap : tiles;
    w.items = halve ? full * cap + 2 * tail : tiles;
  }
  const uint64_t total = (uint64_t)w.items + (uint64_t)w.sk_tiles * w.sk_parts;
  const uint32_t n = total < cap ? (uint32_t)total : cap;
  w.workers = n;
  cfg.gridDim = dim3((PAIR ? 2 : 1) * n, 1, 1);
  int *status = ctx->status_word;
  return bwpp_check_cuda(
      ctx, cudaLaunchKernelEx(&cfg, kern, ta, tb, tcm, epi, M, N, K, ab_f16, w, status),
      PAIR ? "gemm tcgen05 pair" : "gemm tcgen05");
}

template <bool A_MN, bool B_MN>
int launch_tc_any(BwppCudaCtx *ctx, const CUtensorMap &ta, const CUtensorMap &tb,
                  const CUtensorMap &tcm, const GemmEpi &epi,
                  uint32_t M, uint32_t N, uint32_t K, bool pair, uint32_t ab_f16) {
  if (pair) {
    const int rc = launch_tc<A_MN, B_MN, true>(ctx, ta, tb, tcm, epi, M, N, K, ab_f16);
    if (rc != BWPP_CUDA_ERR_UNSUPPORTED) return rc;
  }
  return launch_tc<A_MN, B_MN, false>(ctx, ta, tb, tcm, epi, M, N, K, ab_f16);
}

}  // namespace

// General entry used by the public API and by composite paths (the training
// step).  a_mn / b_mn select the operand layouts described at the top;
// ab_f16 = 1 takes f16 A and B (else bf16); out_bf16 = 1 writes 16-bit C,
// f16 when out_f16 = 1 (else bf16); out_bf16 = 0 writes fp32 C.  The
// residual is fp32 (res16 = 0), bf16 (1) or f16 (2), added, or with 4 set in
// res16 multiplied (SwiGLU gate); it may alias C.
int bwpp_gemm_launch_dt(BwppCudaCtx *ctx, const uint16_t *a, int a_mn, uint32_t lda,
                        const uint16_t *b, int b_mn, uint32_t ldb, void *c,
                        uint32_t ldc, uint32_t M, uint32_t N, uint32_t K,
                        const float *bias, int silu, const void *residual,
                        uint32_t ldr, int out_bf16, int force_simt, int ab_f16,
                        int out_f16, int res16) {
  if (M == 0 || N == 0) return BWPP_CUDA_OK;
  // res16: residual element type in bits 0-1 (0 fp32, 1 bf16, 2 f16); bit 2
  // makes the residual a multiplier
  GemmEpi epi{bias, residual, ldr, silu ? 1 : 0, out_bf16 ? 1 : 0, out_f16 ? 1 : 0, res16 & 3};
  epi.res_mul = (res16 >> 2) & 1;
  const uint32_t out_es = out_bf16 ? 2 : 4;
  const bool tc_ok = !force_simt && K > 0 && al16(a) && al16(b) && al16(c) &&
                     (lda % 8) == 0 && (ldb % 8) == 0 && ((ldc * out_es) % 16) == 0 &&
                     (!bias || al16(bias));
  cudaStream_t s = ctx->stream;
  if (!tc_ok) {
    dim3 grid((N + ST - 1) / ST, (M + ST - 1) / ST);
    gemm_simt_kernel<<<grid, dim3(ST, ST), 0, s>>>(a, b, c, M, N, K, lda, ldb, ldc, a_mn, b_mn, epi,
                                                   ab_f16 ? 1 : 0);
    BWPP_LAUNCH_CHECK(ctx, "gemm simt");
    return BWPP_CUDA_OK;
  }
  // CTA pairs take GEMMs with more than one 128-row block (the second CTA
  // of a pair would otherwise compute rows past M only).
  const bool pair = pairs_enabled() && M > (uint32_t)BM;
  CUtensorMap ta, tb, tcm;
  const auto BF = ab_f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  const auto OUT16 = out_f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  const auto SW = CU_TENSOR_MAP_SWIZZLE_128B;
  int rc = a_mn ? bwpp_make_tmap_2d(ctx, &ta, a, BF, M, K, (uint64_t)lda * 2, 64, BK, SW)
                : bwpp_make_tmap_2d(ctx, &ta, a, BF, K, M, (uint64_t)lda * 2, BK, BM, SW);
  // B boxes: MN-major 64 columns x 64 K rows; K-major 64 K x 64 rows of N
  if (!rc)
    rc = b_mn ? bwpp_make_tmap_2d(ctx, &tb, b, BF, N, K, (uint64_t)ldb * 2, 64, BK, SW)
              : bwpp_make_tmap_2d(ctx, &tb, b, BF, K, N, (uint64_t)ldb * 2, BK, 64, SW);
  if (!rc)
    rc = out_bf16 ? bwpp_make_tmap_2d(ctx, &tcm, c, OUT16, N, M, (uint64_t)ldc * 2, 64, 32, SW)
                  : bwpp_make_tmap_2d(ctx, &tcm, c, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, N, M,
                                      (uint64_t)ldc * 4, EPI_COLS, 32, SW);
  if (rc) return rc;
  const uint32_t f = ab_f16 ? 1u : 0u;
  if (a_mn) {
    return b_mn ? launch_tc_any<true, true>(ctx, ta, tb, tcm, epi, M, N, K, pair, f)
                : launch_tc_any<true, false>(ctx, ta, tb, tcm, epi, M, N, K, pair, f);
  }
  return b_mn ? launch_tc_any<false, true>(ctx, ta, tb, tcm, epi, M, N, K, pair, f)
              : launch_tc_any<false, false>(ctx, ta, tb, tcm, epi, M, N, K, pair, f);
}

// d(gate | up) of a SwiGLU from the product d(a) = A B (M x F), fused into the
// tensor-core GEMM's epilogue: dgu[m, f] = d(gate), dgu[m, F + f] = d(up),
// read against gu = [gate | up] (all bf16, pitch ldgu = 2F or more).  The
// fp32 d(a) is never stored.  BWPP_CUDA_ERR_UNSUPPORTED (nothing launched)
// for shapes the tensor-core path cannot take.
int bwpp_gemm_launch_glu_bwd(BwppCudaCtx *ctx, const uint16_t *a, int a_mn, uint32_t lda,
                             const uint16_t *b, int b_mn, uint32_t ldb, const uint16_t *gu,
                             uint16_t *dgu, uint32_t ldgu, uint32_t M, uint32_t F, uint32_t K) {
  if (M == 0 || F == 0) return BWPP_CUDA_OK;
  if (K == 0 || !al16(a) || !al16(b) || !al16(dgu) || !al16(gu) || (lda % 8) || (ldb % 8) ||
      (ldgu % 8) || (F % 8) || ldgu < 2 * F)
    return BWPP_CUDA_ERR_UNSUPPORTED;
  GemmEpi epi{};
  epi.out_bf16 = 1;
  epi.glu = gu;
  epi.glu_up_out = dgu + F;
  epi.ldglu = ldgu;
  epi.glu_F = F;
  const bool pair = pairs_enabled() && M > (uint32_t)BM;
  CUtensorMap ta, tb, tcm;
  const auto BF = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  const auto SW = CU_TENSOR_MAP_SWIZZLE_128B;
  int rc = a_mn ? bwpp_make_tmap_2d(ctx, &ta, a, BF, M, K, (uint64_t)lda * 2, 64, BK, SW)
                : bwpp_make_tmap_2d(ctx, &ta, a, BF, K, M, (uint64_t)lda * 2, BK, BM, SW);
  if (!rc)
    rc = b_mn ? bwpp_make_tmap_2d(ctx, &tb, b, BF, F, K, (uint64_t)ldb * 2, 64, BK, SW)
              : bwpp_make_tmap_2d(ctx, &tb, b, BF, K, F, (uint64_t)ldb * 2, BK, 64, SW);
  if (!rc) rc = bwpp_make_tmap_2d(ctx, &tcm, dgu, BF, F, M, (uint64_t)ldgu * 2, 64, 32, SW);
  if (rc) return rc;
  if (a_mn) {
    return b_mn ? launch_tc_any<true, true>(ctx, ta, tb, tcm, epi, M, F, K, pair, 0)
                : launch_tc_any<true, false>(ctx, ta, tb, tcm, epi, M, F, K, pair, 0);
  }
  return b_mn ? launch_tc_any<false, true>(ctx, ta, tb, tcm, epi, M, F, K, pair, 0)
              : launch_tc_any<false, false>(ctx, ta, tb, tcm, epi, M, F, K, pair, 0);
}

int bwpp_gemm_launch_ex(BwppCudaCtx *ctx, const uint16_t *a, int a_mn, uint32_t lda,
                        const uint16_t *b, int b_mn, uint32_t ldb, void *c,
                        uint32_t ldc, uint32_t M, uint32_t N, uint32_t K,
                        const float *bias, int silu, const float *residual,
                        uint32_t ldr, int out_bf16, int force_simt) {
  return bwpp_gemm_launch_dt(ctx, a, a_mn, lda, b, b_mn, ldb, c, ldc, M, N, K, bias, silu,
                             residual, ldr, out_bf16, force_simt, 0, 0, 0);
}

// The reference-shaped matmul: A K-major, B MN-major, fp32 out.
int bwpp_gemm_launch(BwppCudaCtx *ctx, const uint16_t *a, const uint16_t *b,
                     float *c, uint32_t M, uint32_t N, uint32_t K, uint32_t lda,
                     uint32_t ldb, uint32_t ldc, const float *bias,
                     int apply_silu, int apply_bias, int force_simt) {
  return bwpp_gemm_launch_ex(ctx, a, 0, lda, b, 1, ldb, c, ldc, M, N, K,
                             (apply_bias && bias) ? bias : nullptr, apply_silu, nullptr, 0,
                             0, force_simt);
}

int bwpp_cast_launch(BwppCudaCtx *ctx, const float *src, uint16_t *dst,
                     uint32_t rows, uint32_t cols, uint32_t ld_src,
                     uint32_t ld_dst) {
  const size_t n = (size_t)rows * cols;
  if (n == 0) return BWPP_CUDA_OK;
  size_t blocks = (n + 255) / 256;
  const size_t cap = (size_t)ctx->num_sms * 16;
  if (blocks > cap) blocks = cap;
  cast_f32_bf16_kernel<<<(unsigned)blocks, 256, 0, ctx->stream>>>(src, dst, rows, cols, ld_src,
                                                                   ld_dst);
  BWPP_LAUNCH_CHECK(ctx, "cast f32->bf16");
  return BWPP_CUDA_OK;
}

extern "C" {

int bwpp_cuda_matmul_bf16(BwppCudaCtx *ctx, const uint16_t *a,
                          const uint16_t *b, float *c, uint32_t M, uint32_t N,
                          uint32_t K, uint32_t lda, uint32_t ldb, uint32_t ldc,
                          const float *bias, int apply_silu, int apply_bias) {
  int rc = bwpp_ctx_enter(ctx);
  if (rc) return rc;
  // A and B are not read when K == 0 (C = epilogue(0)); nothing is touched
  // when M or N is 0.
  if (M && N && (!c || (K && (!a || !b))))
    return bwpp_set_error(ctx, BWPP_CUDA_ERR_ARG, "matmul: NULL buffer");
  if (lda < K || ldb < N || ldc < N)
    return bwpp_set_error(ctx, BWPP_CUDA_ERR_ARG, "matmul: leading dim smaller than row");
  return bwpp_gemm_launch(ctx, a, b, c, M, N, K, lda, ldb, ldc, bias, apply_silu,
                          apply_bias, 0);
}

int bwpp_cuda_gemm_bf16_ex(BwppCudaCtx *ctx, const uint16_t *a, const uint16_t *b,
                           void *c, const BwppCudaGemmParams *p) {
  int rc = bwpp_ctx_enter(ctx);
  if (rc) return rc;
  if (!p) return bwpp_set_error(ctx, BWPP_CUDA_ERR_ARG, "gemm_ex: NULL params");
  if (p->M && p->N && (!c || (p->K && (!a || !b))))
    return bwpp_set_error(ctx, BWPP_CUDA_ERR_ARG, "gemm_ex: NULL buffer");
  if (p->lda < (p->a_mn_major ? p->M : p->K) || p->ldb < (p->b_mn_major ? p->N : p->K) ||
      p->ldc < p->N || (p->residual && p->ldr < p->N))
    return bwpp_set_error(ctx, BWPP_CUDA_ERR_ARG, "gemm_ex: leading dim smaller than row");
  return bwpp_gemm_launch_ex(ctx, a, p->a_mn_major, p->lda, b, p->b_mn_major, p->ldb, c,
                             p->ldc, p->M, p->N, p->K, p->bias, p->apply_silu, p->residual,
                             p->ldr, p->out_bf16, 0);
}

int bwpp_cuda_cast_f32_bf16(BwppCudaCtx *ctx, const float *src, uint16_t *dst,
                            uint32_t rows, uint32_t cols, uint32_t ld_src) {
  int rc = bwpp_ctx_enter(ctx);
  if (rc) return rc;
  if (!src || !dst || ld_src < cols) return bwpp_set_error(ctx, BWPP_CUDA_ERR_ARG, "cast: bad args");
  return bwpp_cast_launch(ctx, src, dst, rows, cols, ld_src, cols);
}

}  // extern "C"

// The split-work scratch of ctx (the GEMM's split-tail partials and epoch
// counters), for other kernels that cut a launch's last work items in two:
// false when the caller owns the workspace or the allocation failed.  The
// launch gets a fresh epoch tag; its counts from earlier launches read as 0.
bool bwpp_split_scratch(BwppCudaCtx *ctx, float **partials, size_t *partial_floats,
                        unsigned long long **counters, size_t *ncounters, uint32_t *epoch) {
  if (!gemm_scratch(ctx)) return false;
  const size_t slots = 2 * (size_t)ctx->num_sms;
  *partials = ctx->gemm_partials;
  *partial_floats = slots * BM * BN;
  *counters = ctx->gemm_counters;
  *ncounters = slots * 2 * EPI_WARPS * 2;
  *epoch = ++ctx->gemm_epoch;
  if (*epoch == 0) *epoch = ++ctx->gemm_epoch;  // 0 is the counters' initial tag
  return true;
}
