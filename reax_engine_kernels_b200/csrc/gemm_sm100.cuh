// Warp-specialised tcgen05 GEMM for sm_100a, shared by libreax_gv, libreax_plain and libreax_slices.
//
//   C[s][m, n] = sum_{k < Kseg} A[m, s*Kseg + k] * B[n, s*Kseg + k]      (A = X [M, K], B = W [N, K], both K-major)
//
// One persistent CTA per SM (320 threads; 192 for the transposed small-M kinds), or one persistent cluster of two
// CTAs per SM pair (PAIR, below):
//   warp 0      TMA producer: 128 x 64 A tile + BN x 64 B tile per stage (128-byte swizzle), ST-deep ring;
//   warp 1      TMEM allocator + MMA issuer: one elected thread issues tcgen05.mma (M=128, N=BN, K=16) into one of
//               two TMEM accumulators (2*BN fp32 columns), commits stage release / accumulator-ready barriers;
//   warps 2..9  epilogue: tcgen05.ld of the accumulator (warp w owns TMEM lanes 32*(w%4)..+31 = tile rows; the two
//               warps of a lane quarter take alternate 128-byte output column blocks, so each SM sub-partition runs
//               two epilogue warps and hides the other's latency), the fused elementwise op, 128-byte rows staged
//               in a swizzled per-warp buffer, coalesced 16-byte global stores with row / column bounds checks.
//               The transposed kinds keep four epilogue warps (warps 2..5).
// Tiles are visited in a grouped raster (up to 16 M-tiles per group, M fastest) so the CTAs working at the same
// time share B tiles in L2.  K tails and M/N tails are zero-filled by TMA.  Each output element's K-reduction
// order depends only on K (never on the tile shape), so every tile configuration produces identical bits.
//
// Split last waves (SPLIT = true).  When the tiles leave a last wave that is only partly full, the whole waves but
// two keep the round-robin raster above, and the remaining tiles (two full waves plus the partial one; all tiles
// when there are fewer than two waves) are shared out by k-blocks: CTA c takes the k-blocks [c U / G, (c+1) U / G)
// of those tiles laid end to end (U = their k-blocks, G = CTAs).  Every CTA then finishes at the same time instead
// of idling through most of a wave.  A CTA's share holds at least one tile's k-blocks, so a tile is cut at most
// once, between CTA c (its first k-blocks, the HEAD piece) and CTA c + 1 (the rest, the TAIL piece).  A CTA runs
// its head first: the epilogue warps copy the fp32 accumulator to a scratch slot of their own and publish it with a
// flag (release, gpu scope) tagged with the launch's epoch.  A CTA runs its tail last: its epilogue warps wait for
// the flag (acquire, bounded), load the partial back into the TMEM accumulator with tcgen05.st, and the MMA issuer
// continues the same tile at the cut k-block with accumulation on.  With two or more waves split, a share of at
// least two tiles' k-blocks puts a whole tile between a CTA's head and tail, and the restore overlaps its MMAs.  The
// accumulator is restored exactly, and the MMAs run in the same k order, so the output has the same bits as the
// unsplit raster.
//
// CTA pairs (PAIR = true).  A cluster of two CTAs on two SMs runs one 256 x BN tile with cta_group::2 MMAs (M = 256):
// each CTA loads its own 128 rows of A and BN/2 of the tile's B rows (no load is multicast).  The leader (cluster rank
// 0) issues the MMAs, which read both CTAs' shared memory at the same offsets and write each CTA's 128 rows into that
// CTA's TMEM.  Both CTAs' copies count on the leader's full barriers; the MMA commits arrive on both CTAs' stage and
// accumulator barriers; each CTA's epilogue drains its own TMEM and hands the accumulator back on the leader's
// barrier.  Work is dealt to clusters, so the split above works unchanged with clusters in place of CTAs: a tail's
// head piece was computed by the CTA of the same rank in the preceding cluster.  Same MMAs, same k order, same bits.
//
// Epilogues (the fused ops of the reference libraries):
//   EPI_GV   : accumulator columns 8j..8j+3 = gate features 4j..4j+3, 8j+4..8j+7 = up features (weights interleaved
//              in groups of 4 rows); out[m, 4j+i] = bf16(bf16(silu(bf16 g)) * bf16 u), silu(g) = g / (1 + expf(-g))
//              with IEEE division -- libreax_gv/gateup_vis2.cu:54-68.  The gate is a bf16 value, so bf16(silu(g))
//              is read from a 65536-entry table that a kernel fills once per device with exactly that expression
//              (silu_exact); the gates that occur sit in a few KB of it, which stay in L1.
//   EPI_BF16 : out = bf16(acc)                      -- libreax_plain/gemm_plain2.cu:1-3
//   EPI_F32  : out = acc (fp32 partials)            -- libreax_slices/gemm_slices_v2.cu:1-3
//   EPI_BF16_T, EPI_F32_T: the same outputs for a swapped problem (A = W, B = X, used when X has few rows): the
//              accumulator tile is the output tile transposed, so lane l (accumulator row = output column n) writes
//              out[m][n] for each accumulator column m -- a warp's store is 32 consecutive n of one output row.
#pragma once
#include "common.cuh"

namespace reax {

enum EpiKind { EPI_GV = 0, EPI_BF16 = 1, EPI_F32 = 2, EPI_BF16_T = 3, EPI_F32_T = 4 };

struct GemmParams {
  int M;                  // rows of A (and of the output)
  int Nacc;               // rows of B = accumulator columns per batch
  int Kseg;               // reduction length per batch
  int S;                  // batches (K segments)
  int nM, nN;             // tile counts
  int num_tiles;          // S * nM * nN
  void* out;              // output base
  long long ld_out;       // output leading dimension (elements)
  long long batch_out;    // output batch stride (elements)
  int out_cols;           // valid output columns (N2 for EPI_GV, N otherwise; output ROWS for the transposed kinds)
  int vec16;              // 1: 16-byte stores are aligned for every row
  const uint16_t* silu_tab;  // EPI_GV: bf16(silu(g)) indexed by the bf16 bits of g
  // split last waves (SPLIT kernels only)
  int rr_tiles;           // tiles [0, rr_tiles) in the round-robin raster (a multiple of the grid size)
  float* part;            // scratch: one BM x BN fp32 partial accumulator slot per CTA
  unsigned int* flag;     // scratch: kSplitFlagsPerCta flags per CTA (one per epilogue warp), = epoch once that
                          // warp's share of the CTA's partial is written
  unsigned int epoch;     // this launch's tag (never 0)
};

template <int BN>
struct GemmCfg {
  static constexpr int BM = 128, BK = 64;
  static constexpr uint32_t A_BYTES = BM * BK * 2;
  static constexpr uint32_t B_BYTES = BN * BK * 2;
  static constexpr uint32_t STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr uint32_t TMEM_COLS = (2 * BN <= 32) ? 32 : (2 * BN <= 64) ? 64 : (2 * BN <= 128) ? 128 : (2 * BN <= 256) ? 256 : 512;
};

// epilogue warps: two per TMEM lane quarter for the row-major kinds, one for the transposed kinds (which stage nothing)
__host__ __device__ constexpr int gemm_epi_warps(int kind) { return (kind == EPI_BF16_T || kind == EPI_F32_T) ? 4 : 8; }
__host__ __device__ constexpr int gemm_threads(int kind) { return 64 + 32 * gemm_epi_warps(kind); }
// split last waves: hand-over flags per CTA (one per epilogue warp) and the widest tile a partial slot holds
constexpr int kSplitFlagsPerCta = 8;
constexpr int kSplitSlotCols = 256;

// bytes of one pipeline stage in one CTA: the 128 x 64 A tile and the B tile (half of it in each CTA of a pair)
template <int BN, bool PAIR>
__host__ __device__ constexpr uint32_t gemm_stage_bytes() {
  return GemmCfg<BN>::A_BYTES + (PAIR ? GemmCfg<BN>::B_BYTES / 2 : GemmCfg<BN>::B_BYTES);
}

template <int BN, int ST, int KIND, bool PAIR = false>
constexpr int gemm_smem_bytes() {
  // alignment slack + operand ring + one 32-row x 128-byte staging buffer per epilogue warp + barriers
  return 1024 + ST * (int)gemm_stage_bytes<BN, PAIR>() + gemm_epi_warps(KIND) * 32 * 128 + 256;
}

__device__ __forceinline__ void tile_coords(int t, int nM, int nN, int& s, int& m, int& n) {
  const int per_batch = nM * nN;
  s = t / per_batch;
  int r = t - s * per_batch;
  constexpr int GM = 16;
  const int per_group = GM * nN;
  const int g = r / per_group;
  r -= g * per_group;
  const int m0 = g * GM;
  const int gm = min(GM, nM - m0);
  n = r / gm;
  m = m0 + (r - n * gm);
}

enum WorkKind { WK_FULL = 0, WK_HEAD = 1, WK_TAIL = 2 };

// Split last waves: the tiles kept in the round-robin raster (a multiple of the G work units) -- all whole waves but
// two; the rest, at least one and at most three waves, is dealt out by k-blocks.
__host__ __device__ constexpr int split_rr_tiles(int tiles, int G) { return tiles / G >= 2 ? (tiles / G - 2) * G : 0; }

// The work items of one CTA, in the order it runs them: round-robin tiles, then (SPLIT) its head piece, the whole
// tiles inside its k-block share and its tail piece.  Tile indices of the split part are absolute.
struct WorkList {
  int c, G, nk, count, n_rr, rr_tiles;
  int head, tail, nwhole, w0, tf, kf, tl, ke;
  template <bool SPLIT, bool PAIR = false>
  __device__ __forceinline__ static WorkList make(const GemmParams& p, int nk) {
    WorkList w;
    // PAIR: the work units are the clusters (both CTAs of a pair run the same items)
    const int c = PAIR ? (int)cluster_id_x() : (int)blockIdx.x;
    const int G = PAIR ? (int)cluster_count_x() : (int)gridDim.x;
    w.init<SPLIT>(p.num_tiles, p.rr_tiles, nk, c, G);
    return w;
  }
  // work unit c of G (a CTA, or a cluster of two); host-callable so the schedule can be checked on the CPU
  template <bool SPLIT>
  __host__ __device__ __forceinline__ void init(int num_tiles, int rr, int nk_, int c_, int G_) {
    c = c_;
    G = G_;
    nk = nk_;
    head = tail = nwhole = w0 = tf = kf = tl = ke = 0;
    if (!SPLIT) {
      rr_tiles = num_tiles;
      n_rr = (num_tiles - c + G - 1) / G;
      count = n_rr;
      return;
    }
    rr_tiles = rr;
    n_rr = rr_tiles / G;
    const long long U = (long long)(num_tiles - rr_tiles) * nk;
    const long long u0 = U * c / G, u1 = U * (c + 1) / G;  // u1 - u0 >= nk: at least one tile's k-blocks
    tf = (int)(u0 / nk);
    kf = (int)(u0 % nk);
    tl = (int)((u1 - 1) / nk);
    ke = (int)((u1 - 1) % nk) + 1;
    head = ke < nk;
    tail = kf > 0;
    w0 = tf + tail;
    const int w1 = tl - head;
    nwhole = w1 >= w0 ? w1 - w0 + 1 : 0;
    count = n_rr + head + nwhole + tail;
  }
  __host__ __device__ __forceinline__ void item(int i, int& t, int& kb0, int& kb1, int& kind) const {
    kb0 = 0;
    kb1 = nk;
    kind = WK_FULL;
    if (i < n_rr) {
      t = c + i * G;
      return;
    }
    i -= n_rr;
    if (head) {
      if (i == 0) {
        t = rr_tiles + tl;
        kb1 = ke;
        kind = WK_HEAD;
        return;
      }
      --i;
    }
    if (i < nwhole) {
      t = rr_tiles + w0 + i;
      return;
    }
    t = rr_tiles + tf;
    kb0 = kf;
    kind = WK_TAIL;
  }
};

template <int BN, int ST, int KIND, bool SPLIT = false, bool PAIR = false>
__global__ void __launch_bounds__(gemm_threads(KIND), 1)
gemm_kernel(const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_b, const GemmParams p) {
  using C = GemmCfg<BN>;
  constexpr int BM = C::BM, BK = C::BK;
  constexpr bool TRANS = KIND == EPI_BF16_T || KIND == EPI_F32_T;
  constexpr int ACC_PER_ITER = KIND == EPI_GV ? 128 : (KIND == EPI_BF16 ? 64 : 32);  // -> 128 output bytes per row
  constexpr int ITERS = (BN + ACC_PER_ITER - 1) / ACC_PER_ITER;
  constexpr int OUT_PER_ITER = KIND == EPI_GV ? 64 : ACC_PER_ITER;                       // output elements per row
  constexpr int OUT_PER_TILE = KIND == EPI_GV ? BN / 2 : BN;
  constexpr int ES = (KIND == EPI_F32 || KIND == EPI_F32_T) ? 4 : 2;                      // output element bytes
  constexpr int EPC = 16 / ES;                                                           // elements per 16-B chunk
  static_assert(BN % 32 == 0 && BN <= 256, "BN");
  static_assert(KIND != EPI_GV || BN % 128 == 0, "gate-up epilogue handles 128 accumulator columns per pass");
  static_assert(!(SPLIT && TRANS), "split last waves serve the row-major kinds");
  static_assert(!(PAIR && TRANS), "CTA pairs serve the row-major kinds");
  static_assert(!PAIR || (BN % 32 == 0 && BN >= 64), "a pair's B tile is two halves of a multiple of 16 rows");
  constexpr int EW = gemm_epi_warps(KIND);  // epilogue warps
  constexpr int EH = EW / 4;                // epilogue warps per TMEM lane quarter
  constexpr uint32_t STAGE = gemm_stage_bytes<BN, PAIR>();  // this CTA's bytes per stage
  constexpr int PM = PAIR ? 2 * BM : BM;                    // rows of a tile (a pair's tile spans both CTAs)

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t sbase = (raw + 1023u) & ~1023u;
  const uint32_t staging = sbase + ST * STAGE;
  const uint32_t bars = staging + (uint32_t)(EW * 32 * 128);
  // barrier block: full[ST] | empty[ST] | tfull[2] | tempty[2] | drain | tmem holder | abort flag | restored |
  // (PAIR teardown) exchange barrier | drained barrier | the other producer's fill count
  auto full_bar = [&](int s) { return bars + 8u * s; };
  auto empty_bar = [&](int s) { return bars + 8u * (ST + s); };
  auto tfull_bar = [&](int a) { return bars + 8u * (2 * ST + a); };
  auto tempty_bar = [&](int a) { return bars + 8u * (2 * ST + 2 + a); };
  const uint32_t drain_bar = bars + 8u * (2 * ST + 4);
  const uint32_t holder = bars + 8u * (2 * ST + 5);
  const uint32_t restored_bar = bars + 8u * (2 * ST + 7);  // SPLIT: the tail's partial is back in TMEM
  const uint32_t xchg_bar = bars + 8u * (2 * ST + 8);      // PAIR: the other producer's fill count has arrived
  const uint32_t drained_bar = bars + 8u * (2 * ST + 9);   // PAIR (peer): the leader saw every copy land
  const uint32_t xcnt = bars + 8u * (2 * ST + 10);         // PAIR: the other producer's fill count
  static_assert(8 * (2 * ST + 11) <= 256, "barrier block");
  uint8_t* bars_ptr = smem_raw + (bars - raw);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars_ptr + 8u * (2 * ST + 5) + 8);
  const uint32_t* holder_ptr = reinterpret_cast<const uint32_t*>(bars_ptr + 8u * (2 * ST + 5));

  const int warp = warp_id(), lane = lane_id();
  // PAIR: rank 0 (the leader) issues the pair's MMAs and owns the barriers they wait on: full[] counts both CTAs'
  // copies, tempty[] both CTAs' epilogue threads.  The MMAs' commits arrive on empty[] and tfull[] of both CTAs.
  const uint32_t crank = PAIR ? cluster_rank() : 0u;
  const bool leader = crank == 0;
  if (threadIdx.x == 0) {
    for (int s = 0; s < ST; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(tfull_bar(a), 1);
      mbar_init(tempty_bar(a), (PAIR ? 2 : 1) * 32 * EW);
    }
    mbar_init(drain_bar, 1);
    if (SPLIT) mbar_init(restored_bar, (PAIR ? 2 : 1) * 32 * EW);
    if (PAIR) {
      mbar_init(xchg_bar, 1);
      mbar_init(drained_bar, 1);
    }
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tma_a);
    tma_prefetch_desc(&tma_b);
  }
  if (warp == 1) {
    if constexpr (PAIR) {
      tmem_alloc_pair(holder, C::TMEM_COLS);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(holder, C::TMEM_COLS);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  __syncwarp();
  if constexpr (PAIR) cluster_sync_all();  // both CTAs' barriers are initialised before either signals the other
  else __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *holder_ptr;
  const int nk = (p.Kseg + BK - 1) / BK;
  const WorkList wl = WorkList::make<SPLIT, PAIR>(p, nk);
  // hand the accumulator back to the MMA issuer (PAIR: the leader's barrier, from both CTAs)
  auto release_acc = [&](int a) {
    tc_fence_before();
    if constexpr (PAIR) mbar_arrive_cluster(mapa_shared(tempty_bar(a), 0));
    else mbar_arrive(tempty_bar(a));
  };

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t armed = 0;  // bit s: stage s has an arming whose completion has not been observed
      uint32_t armed_par = 0;
      int fills = 0;  // stages this producer has filled
      bool ok = true;
      for (int i = 0; i < wl.count && ok; ++i) {
        int t, kb0, kb1, kind;
        wl.item(i, t, kb0, kb1, kind);
        int s, m, n;
        tile_coords(t, p.nM, p.nN, s, m, n);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(empty_bar(stage), phase ^ 1u, abort_flag, ST_TIMEOUT_PRODUCER)) { ok = false; break; }
          const uint32_t sa = sbase + stage * STAGE, sb = sa + C::A_BYTES;
          if constexpr (PAIR) {
            // this CTA's 128 rows of A and half of B; both CTAs' copies count on the leader's full barrier, which
            // the leader arms for both (a copy landing before the arming leaves the count negative until then)
            const uint32_t fb = mapa_shared(full_bar(stage), 0);
            if (leader) mbar_arrive_expect_tx(full_bar(stage), 2 * STAGE);
            tma_load_3d_pair(sa, &tma_a, fb, kb * BK, s, m * PM + (int)crank * BM);
            tma_load_3d_pair(sb, &tma_b, fb, kb * BK, s, n * BN + (int)crank * (BN / 2));
          } else {
            mbar_arrive_expect_tx(full_bar(stage), STAGE);
            tma_load_3d(sa, &tma_a, full_bar(stage), kb * BK, s, m * BM);
            tma_load_3d(sb, &tma_b, full_bar(stage), kb * BK, s, n * BN);
          }
          if constexpr (!PAIR) {
            armed |= 1u << stage;
            armed_par = (armed_par & ~(1u << stage)) | (phase << stage);
          }
          ++fills;
          if (++stage == ST) { stage = 0; phase ^= 1u; }
        }
      }
      if constexpr (PAIR) {
        // the leader's MMA commits release the stages of both CTAs: wait for the release of every stage's last fill,
        // so that no commit arrives on this CTA's barriers after it has left
        for (int i = 0; i < ST && ok; ++i) {
          if (!mbar_wait(empty_bar(stage), phase ^ 1u, abort_flag, ST_TIMEOUT_PRODUCER)) break;
          if (++stage == ST) { stage = 0; phase ^= 1u; }
        }
        // Copies in flight.  The peer's copies count on the leader's full barriers, so no CTA can see alone whether
        // its own copies have landed, and after a give-up the two producers may have stopped at different fills
        // (neither runs more than ST fills ahead of the other: a fill waits for the MMAs of the one ST before it,
        // which waited for both CTAs' copies).  The producers exchange their fill counts; the leader then completes
        // the phases of the last ST fills -- arming a fill that only the peer issued (the peer's bytes), standing in
        // for the peer's bytes of a fill that only the leader issued -- waits for each, and tells the peer.  In a
        // normal run both counts are equal and every one of those phases has completed already.
        const uint32_t other = crank ^ 1u;
        st_shared_cluster_u32(mapa_shared(xcnt, other), (uint32_t)fills);
        mbar_arrive_cluster(mapa_shared(xchg_bar, other));
        int other_fills = fills;
        if (drain_wait_cl(xchg_bar, 0)) other_fills = (int)ld_shared_u32(xcnt);
        if (leader) {
          const int fmax = fills > other_fills ? fills : other_fills;
          for (int f = fmax > ST ? fmax - ST : 0; f < fmax; ++f) {
            const int s2 = f % ST;
            if (f >= fills) mbar_arrive_expect_tx(full_bar(s2), STAGE);
            else if (f >= other_fills) mbar_complete_tx_cl(mapa_shared(full_bar(s2), 0), STAGE);
            drain_wait_cl(full_bar(s2), (uint32_t)(f / ST) & 1u);
          }
          mbar_arrive_cluster(mapa_shared(drained_bar, 1));
        } else {
          drain_wait_cl(drained_bar, 0);
        }
      } else {
        // teardown: never leave the CTA while a copy into its shared memory may still be in flight
        for (int s2 = 0; s2 < ST; ++s2)
          if (armed & (1u << s2)) {
            const long long t0 = clock64();
            while (!mbar_try_wait(full_bar(s2), (armed_par >> s2) & 1u)) {
              if (clock64() - t0 > REAX_DRAIN_LIMIT) { record_status(ST_TIMEOUT_DRAIN); break; }
            }
          }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0 && leader) {  // PAIR: the leader issues the pair's MMAs
      constexpr uint32_t IDESC = idesc_bf16(PM, BN);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int local = 0; local < wl.count && ok; ++local) {
        int t, kb0, kb1, kind;
        wl.item(local, t, kb0, kb1, kind);
        const int acc = local & 1;
        const uint32_t acc_par = (uint32_t)(local >> 1) & 1u;
        if (!(PAIR ? mbar_wait_cl(tempty_bar(acc), acc_par ^ 1u, abort_flag, ST_TIMEOUT_MMA_ACC)
                   : mbar_wait(tempty_bar(acc), acc_par ^ 1u, abort_flag, ST_TIMEOUT_MMA_ACC)))
          break;
        if (SPLIT && kind == WK_TAIL &&
            !(PAIR ? mbar_wait_cl(restored_bar, 0, abort_flag, ST_TIMEOUT_MMA_ACC)
                   : mbar_wait(restored_bar, 0, abort_flag, ST_TIMEOUT_MMA_ACC)))
          break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(acc * BN);
        const bool cont = SPLIT && kind == WK_TAIL;  // the accumulator already holds k-blocks [0, kb0)
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(full_bar(stage), phase, abort_flag, ST_TIMEOUT_MMA_FULL)) { ok = false; break; }
          tc_fence_after();
          const uint32_t sa = sbase + stage * STAGE, sb = sa + C::A_BYTES;
          const uint64_t adesc = sw128_desc(sa), bdesc = sw128_desc(sb);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            const uint32_t accum = (cont || kb != kb0 || k != 0) ? 1u : 0u;
            if constexpr (PAIR) mma_bf16_ss_pair(d_tmem, adesc + (uint64_t)(2 * k), bdesc + (uint64_t)(2 * k), IDESC, accum);
            else mma_bf16_ss(d_tmem, adesc + (uint64_t)(2 * k), bdesc + (uint64_t)(2 * k), IDESC, accum);
          }
          // stage free (PAIR: in both CTAs) once these MMAs have read it
          if constexpr (PAIR) mma_commit_pair_both(empty_bar(stage));
          else mma_commit(empty_bar(stage));
          if (++stage == ST) { stage = 0; phase ^= 1u; }
        }
        if (!ok) break;
        // accumulator ready for the epilogue (PAIR: both CTAs' epilogues)
        if constexpr (PAIR) mma_commit_pair_both(tfull_bar(acc));
        else mma_commit(tfull_bar(acc));
      }
      // teardown: wait for every issued MMA before TMEM can be released
      if constexpr (PAIR) mma_commit_pair(drain_bar);
      else mma_commit(drain_bar);
      const long long t0 = clock64();
      while (!mbar_try_wait(drain_bar, 0)) {
        if (clock64() - t0 > REAX_DRAIN_LIMIT) { record_status(ST_TIMEOUT_DRAIN); break; }
      }
    }
  } else {
    // ------------------------------------------------------------------ epilogue (warps 2 .. 2 + EW - 1)
    const int ew = warp - 2;                    // epilogue warp index
    const int q = warp & 3;                     // TMEM lane quarter this warp may access
    const int h = ew >> 2;                      // which of the quarter's EH warps: its share of the columns
    const uint32_t stg = staging + (uint32_t)ew * (32 * 128);
    const int row = 32 * q + lane;              // tile row = TMEM lane of this thread
    // Column ownership: warp (q, h) reads, and (SPLIT) saves and restores, only the accumulator columns of its
    // output passes it = h, h + EH, .. (pass it = columns [it ACC_PER_ITER, (it+1) ACC_PER_ITER)), so no warp ever
    // writes TMEM columns that another warp may still have to read.
    // SPLIT: partial slots hold column groups of 4 for all 128 rows (float4 (j, row) at j * 128 + row), so a warp's
    // 16-byte accesses cover 512 contiguous bytes.  Each warp hands its rows and columns over with its own flag; the
    // same warp of the next CTA takes exactly those back.  PAIR: work is dealt to clusters, so a tail's head piece
    // was computed by the CTA of the same rank in the preceding cluster, whose TMEM holds the same rows.
    const int split_src = (int)blockIdx.x - (PAIR ? 2 : 1);
    constexpr int CPI = ACC_PER_ITER / 32;      // 32-column chunks per output pass
    static_assert(!SPLIT || CPI * ITERS * 32 == BN, "whole chunks per pass");
    static_assert(!SPLIT || (EW <= kSplitFlagsPerCta && BN <= kSplitSlotCols), "hand-over scratch layout");
    const int tail_i = (SPLIT && wl.tail) ? wl.count - 1 : -1;
    auto restore = [&]() -> bool {
      // the preceding CTA cut this CTA's tail tile: wait for its partial, then load it into accumulator tail_i & 1
      const int src = split_src;
      const unsigned int* f = p.flag + EW * src + ew;
      bool ok = true;
      if (ld_acquire_gpu_u32(f) != p.epoch) {
        const long long t0 = clock64();
        while (ld_acquire_gpu_u32(f) != p.epoch) {
          if (*abort_flag) { ok = false; break; }
          if (clock64() - t0 > REAX_WAIT_LIMIT) {
            *abort_flag = 1;
            record_status(ST_TIMEOUT_SPLIT);
            ok = false;
            break;
          }
          __nanosleep(128);
        }
      }
      if (!__all_sync(0xffffffffu, ok)) return false;
      const float4* slot = reinterpret_cast<const float4*>(p.part) + (size_t)src * (BM * BN / 4);
      const uint32_t tb = tmem_base + ((uint32_t)(32 * q) << 16) + (uint32_t)((tail_i & 1) * BN);
#pragma unroll 1
      for (int cc = 0; cc < BN / 32; ++cc) {
        if ((cc / CPI) % EH != h) continue;  // not one of this warp's columns (warp-uniform)
        uint32_t r[32];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float4 v = __ldcg(slot + (size_t)(cc * 8 + j) * BM + row);
          r[4 * j + 0] = __float_as_uint(v.x);
          r[4 * j + 1] = __float_as_uint(v.y);
          r[4 * j + 2] = __float_as_uint(v.z);
          r[4 * j + 3] = __float_as_uint(v.w);
        }
        tmem_st32_nowait(tb + (uint32_t)(cc * 32), r);
      }
      tmem_wait_st();
      tc_fence_before();
      if constexpr (PAIR) mbar_arrive_cluster(mapa_shared(restored_bar, 0));  // the leader issues the tail's MMAs
      else mbar_arrive(restored_bar);
      return true;
    };
    // Restore point: once accumulator tail_i & 1 is free (after item tail_i - 2), and never before this CTA's own
    // head is published -- the head waits for nothing, so no chain of CTAs waiting on one another can form.
    int restore_after = tail_i - 2;
    if (SPLIT && wl.head && wl.n_rr > restore_after) restore_after = wl.n_rr;
    bool alive = true;
    if (SPLIT && tail_i >= 0 && restore_after < 0) alive = restore();  // its accumulator has not been used yet
    bool restored = false;
    for (int local = 0; local < wl.count && alive; ++local) {
      int t, kb0, kb1, kind;
      wl.item(local, t, kb0, kb1, kind);
      int s, m, n;
      tile_coords(t, p.nM, p.nN, s, m, n);
      const int acc = local & 1;
      const uint32_t acc_par = (uint32_t)(local >> 1) & 1u;
      if (SPLIT && kind == WK_HEAD && tail_i == local + 1) {
        // The tail follows the head directly and its accumulator is already free: restore it first if the preceding
        // CTA's partial arrives before this head's MMAs finish, so the tail's MMAs can follow the head's at once.
        // The head is saved as soon as its MMAs finish otherwise; it never waits for a flag, so no chain can form.
        const unsigned int* f = p.flag + EW * split_src + ew;
        const long long t0 = clock64();
        for (;;) {
          int st = 0;
          if (lane == 0)
            st = (PAIR ? mbar_try_wait_cl(tfull_bar(acc), acc_par) : mbar_try_wait(tfull_bar(acc), acc_par))
                     ? 1
                     : (ld_acquire_gpu_u32(f) == p.epoch ? 2 : 0);
          st = __shfl_sync(0xffffffffu, st, 0);
          if (st == 1) break;
          if (st == 2) {
            alive = restore();
            restored = true;
            break;
          }
          if (*abort_flag || clock64() - t0 > REAX_WAIT_LIMIT) break;  // the waits below give up and record it
          __nanosleep(64);
        }
        if (!alive) break;
      }
      if (!(PAIR ? mbar_wait_warp_cl(tfull_bar(acc), acc_par, abort_flag, ST_TIMEOUT_EPI)
                 : mbar_wait_warp(tfull_bar(acc), acc_par, abort_flag, ST_TIMEOUT_EPI)))
        break;
      tc_fence_after();
      __syncwarp();  // tcgen05.ld is warp-collective: reconverge after the per-lane wait loop
      const uint32_t tbase = tmem_base + ((uint32_t)(32 * q) << 16) + (uint32_t)(acc * BN);
      const int grow0 = m * PM + (int)crank * BM + 32 * q;  // first global row of this warp's slab
      uint8_t* outb = reinterpret_cast<uint8_t*>(p.out) + (size_t)s * (size_t)p.batch_out * ES;
      if (SPLIT && kind == WK_HEAD) {
        // the following CTA finishes this tile: hand it the fp32 accumulator
        float4* slot = reinterpret_cast<float4*>(p.part) + (size_t)blockIdx.x * (BM * BN / 4);
        const int my_last_cc = h < ITERS ? (h + ((ITERS - 1 - h) / EH) * EH + 1) * CPI - 1 : -1;
        if (my_last_cc < 0) {
          release_acc(acc);
        }
#pragma unroll 1
        for (int cc = 0; cc < BN / 32; ++cc) {
          if ((cc / CPI) % EH != h) continue;  // not one of this warp's columns (warp-uniform)
          uint32_t r[32];
          tmem_ld32(tbase + (uint32_t)(cc * 32), r);
          if (cc == my_last_cc) {
            release_acc(acc);
          }
#pragma unroll
          for (int j = 0; j < 8; ++j)
            __stcg(slot + (size_t)(cc * 8 + j) * BM + row,
                   make_float4(__uint_as_float(r[4 * j]), __uint_as_float(r[4 * j + 1]), __uint_as_float(r[4 * j + 2]),
                               __uint_as_float(r[4 * j + 3])));
        }
        __threadfence();
        __syncwarp();
        if (lane == 0) st_release_gpu_u32(p.flag + EW * blockIdx.x + ew, p.epoch);
      } else if constexpr (TRANS) {
        // accumulator row (this lane) = output column; accumulator column = output row
        const int n_out = grow0 + lane;
#pragma unroll 1
        for (int it = 0; it < BN / 32; ++it) {
          uint32_t r[32];
          tmem_ld32(tbase + (uint32_t)(it * 32), r);
          if (it == BN / 32 - 1) {
            release_acc(acc);
          }
          const int m0 = n * BN + it * 32;
          if (n_out < p.M) {
#pragma unroll
            for (int c = 0; c < 32; ++c) {
              const int m_out = m0 + c;
              if (m_out < p.out_cols) {
                uint8_t* dst = outb + ((size_t)m_out * (size_t)p.ld_out + (size_t)n_out) * ES;
                if (ES == 4) *reinterpret_cast<uint32_t*>(dst) = r[c];
                else *reinterpret_cast<uint16_t*>(dst) = (uint16_t)(pack_bf16(__uint_as_float(r[c]), 0.f) & 0xffffu);
              }
            }
          }
        }
      } else {
      // this warp's passes: it = h, h + EH, ..  (the last one hands the accumulator back; a warp without a pass
      // hands it back at once)
      const int my_last = h < ITERS ? h + ((ITERS - 1 - h) / EH) * EH : -1;
      if (my_last < 0) {
        release_acc(acc);
      }
#pragma unroll 1
      for (int it = h; it < ITERS; it += EH) {
        uint4 chunk[8];
        if (KIND == EPI_GV) {
          // all four loads in flight before the one wait; then 16 independent gates per chunk
          uint32_t r[4][32];
#pragma unroll
          for (int c4 = 0; c4 < 4; ++c4) tmem_ld32_nowait(tbase + (uint32_t)(it * 128 + c4 * 32), r[c4]);
#pragma unroll
          for (int c4 = 0; c4 < 4; ++c4) tmem_wait_ld32(r[c4]);
#pragma unroll
          for (int c4 = 0; c4 < 4; ++c4) {
            float sg[16];
#pragma unroll
            for (int e = 0; e < 16; ++e) {
              const uint32_t gb = __bfloat16_as_ushort(__float2bfloat16_rn(__uint_as_float(r[c4][(e >> 2) * 8 + (e & 3)])));
              sg[e] = __uint_as_float((uint32_t)__ldg(p.silu_tab + gb) << 16);
            }
            uint32_t o[8];
#pragma unroll
            for (int e = 0; e < 16; e += 2) {
              const float u0 = bf16_round(__uint_as_float(r[c4][(e >> 2) * 8 + 4 + (e & 3)]));
              const float u1 = bf16_round(__uint_as_float(r[c4][((e + 1) >> 2) * 8 + 4 + ((e + 1) & 3)]));
              o[e >> 1] = pack_bf16(__fmul_rn(sg[e], u0), __fmul_rn(sg[e + 1], u1));
            }
            chunk[c4 * 2 + 0] = make_uint4(o[0], o[1], o[2], o[3]);
            chunk[c4 * 2 + 1] = make_uint4(o[4], o[5], o[6], o[7]);
          }
        } else if (KIND == EPI_BF16) {
#pragma unroll
          for (int c2 = 0; c2 < 2; ++c2) {
            uint32_t r[32];
            tmem_ld32(tbase + (uint32_t)(it * 64 + c2 * 32), r);
#pragma unroll
            for (int c = 0; c < 4; ++c)
              chunk[c2 * 4 + c] = make_uint4(pack_bf16(__uint_as_float(r[8 * c + 0]), __uint_as_float(r[8 * c + 1])),
                                             pack_bf16(__uint_as_float(r[8 * c + 2]), __uint_as_float(r[8 * c + 3])),
                                             pack_bf16(__uint_as_float(r[8 * c + 4]), __uint_as_float(r[8 * c + 5])),
                                             pack_bf16(__uint_as_float(r[8 * c + 6]), __uint_as_float(r[8 * c + 7])));
          }
        } else {
          uint32_t r[32];
          tmem_ld32(tbase + (uint32_t)(it * 32), r);
#pragma unroll
          for (int c = 0; c < 8; ++c) chunk[c] = make_uint4(r[4 * c], r[4 * c + 1], r[4 * c + 2], r[4 * c + 3]);
        }
        if (it == my_last) {
          // all of this warp's TMEM reads of the accumulator are complete: hand it back to the MMA issuer
          release_acc(acc);
        }
        // stage: row `lane`, 16-byte chunk c at (c ^ (lane & 7)) -> conflict-free both ways
#pragma unroll
        for (int c = 0; c < 8; ++c) st_shared_v4(stg + (uint32_t)lane * 128u + (uint32_t)((c ^ (lane & 7)) << 4), chunk[c]);
        __syncwarp();
        const int col0 = n * OUT_PER_TILE + it * OUT_PER_ITER;  // first output column of this pass
#pragma unroll
        for (int pass = 0; pass < 8; ++pass) {
          const int rl = pass * 4 + (lane >> 3), c = lane & 7;
          const uint4 v = ld_shared_v4(stg + (uint32_t)rl * 128u + (uint32_t)((c ^ (rl & 7)) << 4));
          const int grow = grow0 + rl, gcol = col0 + c * EPC;
          if (grow < p.M && gcol < p.out_cols) {
            uint8_t* dst = outb + ((size_t)grow * (size_t)p.ld_out + (size_t)gcol) * ES;
            if (p.vec16 && gcol + EPC <= p.out_cols) {
              *reinterpret_cast<uint4*>(dst) = v;
            } else {
              const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
              for (int e = 0; e < EPC; ++e) {
                if (gcol + e < p.out_cols) {
                  if (ES == 2)
                    reinterpret_cast<uint16_t*>(dst)[e] = (uint16_t)((w[e >> 1] >> (16 * (e & 1))) & 0xffffu);
                  else
                    reinterpret_cast<uint32_t*>(dst)[e] = w[e];
                }
              }
            }
          }
        }
        __syncwarp();
      }
      }
      if (SPLIT && tail_i >= 0 && local == restore_after && !restored) alive = restore();
    }
  }

  __syncwarp();
  tc_fence_before();
  // PAIR: neither CTA leaves (or frees the pair's TMEM) while the other may still signal it or read its operands
  if constexpr (PAIR) cluster_sync_all();
  else __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    if constexpr (PAIR) tmem_dealloc_pair(tmem_base, C::TMEM_COLS);
    else tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
}

}  // namespace reax

// ------------------------------------------------------------------------------------------------
// host launcher
// ------------------------------------------------------------------------------------------------
namespace reax_host {

struct GemmProblem {
  const void* a;       // [M, K] bf16 row-major (lda = K)
  const void* b;       // [Nacc, K] bf16 row-major (ldb = K)
  void* out;
  int M, Nacc, K;      // full K (row length of A and B)
  int Kseg, S;         // per-batch reduction length and batch count (S = 1, Kseg = K for plain GEMMs)
  long long ld_out, batch_out;
  int out_cols;
  const uint16_t* silu_tab = nullptr;  // EPI_GV only: the device table of bf16(silu(g)) by the bf16 bits of g
};

// Split last waves: whether a problem of `tiles` tiles on `sms` SMs takes the split kernel.  REAX_GEMM_SPLIT=0
// turns it off and =1 takes it whenever the last wave is partial.  By default it is taken when the tiles fill at
// most three whole waves and the last wave is at most 85 % full.  Measured on B200 (gate-up, M = 2048, K = 4096):
// the split saves 7 % at 3.03 and 1.51 waves, while at 6 and 12 waves it is even or 1 % slower -- SMs differ in
// speed by up to 8 %, the unsplit raster happens to give its extra tiles to the faster ones, and an even split of
// k-blocks is paced by the slowest.  Both kernels give identical bits, so the choice is a speed setting only.
inline bool split_wanted(int tiles, int sms) {
  if (tiles <= sms || tiles % sms == 0) return false;
  const char* e = std::getenv("REAX_GEMM_SPLIT");
  if (e != nullptr && e[0] == '0') return false;
  if (e != nullptr && e[0] == '1') return true;
  return tiles / sms <= 3 && (long long)(tiles % sms) * 100 <= 85LL * sms;
}

// Scratch of the split kernel: a flag block (kSplitFlagsPerCta flags per CTA) and one 128 x kSplitSlotCols fp32
// partial accumulator slot per CTA (18.9 MB for 148 SMs).  Each device has a pool of kSplitPool such buffers,
// allocated on first use and kept for the life of the process, so the scratch never grows with the number of streams
// a caller uses.  Launches take the buffers in turn; each buffer carries an event recorded after its last launch, and
// a launch on any stream first waits for it, so two launches never use one buffer at the same time (launches on up to
// kSplitPool streams still run side by side).  Each launch takes a new epoch, so a flag left by an earlier launch (or
// one that gave up) never matches.
struct SplitScratch {
  float* part;
  unsigned int* flag;
  unsigned int epoch;
};
constexpr int kSplitPool = 4;

// Runs launch(scratch) with a pool buffer reserved for it on stream `st` and returns true, or returns false without
// calling it (the caller runs the unsplit kernel) when a buffer cannot be allocated or ordered.  `rc` receives
// launch's return code.
template <typename Launch>
inline bool with_split_scratch(int dev, cudaStream_t st, int slots, Launch&& launch, int& rc) {
  struct Buf {
    void* base = nullptr;
    cudaEvent_t last = nullptr;  // recorded after the buffer's latest launch
    bool used = false;
    unsigned int epoch = 0;
  };
  struct Pool {
    Buf buf[kSplitPool];
    int slots = 0;
    unsigned int next = 0;
  };
  static std::mutex mu;
  static std::map<int, Pool> pools;
  const size_t flag_bytes = ((size_t)reax::kSplitFlagsPerCta * slots * sizeof(unsigned int) + 255) & ~(size_t)255;
  std::lock_guard<std::mutex> lk(mu);  // held until the launch and its event are enqueued
  Pool& pool = pools[dev];
  if (pool.slots == 0) pool.slots = slots;
  if (pool.slots < slots) return false;
  Buf& b = pool.buf[pool.next % kSplitPool];
  if (b.base == nullptr) {
    void* base = nullptr;
    if (cudaMalloc(&base, flag_bytes + (size_t)slots * 128 * reax::kSplitSlotCols * sizeof(float)) != cudaSuccess) {
      (void)cudaGetLastError();
      return false;
    }
    if (cudaEventCreateWithFlags(&b.last, cudaEventDisableTiming) != cudaSuccess ||
        cudaMemsetAsync(base, 0, flag_bytes, st) != cudaSuccess) {
      (void)cudaGetLastError();
      if (b.last != nullptr) cudaEventDestroy(b.last);
      b.last = nullptr;
      cudaFree(base);
      return false;
    }
    b.base = base;
  }
  if (b.used && cudaStreamWaitEvent(st, b.last, 0) != cudaSuccess) {
    (void)cudaGetLastError();
    return false;
  }
  ++pool.next;
  if (++b.epoch == 0) b.epoch = 1;
  SplitScratch sc;
  sc.flag = static_cast<unsigned int*>(b.base);
  sc.part = reinterpret_cast<float*>(static_cast<uint8_t*>(b.base) + flag_bytes);
  sc.epoch = b.epoch;
  rc = launch(sc);
  if (cudaEventRecord(b.last, st) == cudaSuccess) {
    b.used = true;
  } else {
    // without the event the next user of this buffer could overlap this launch: order it behind the whole device
    (void)cudaGetLastError();
    (void)cudaDeviceSynchronize();
    b.used = false;
  }
  return true;
}

// CTA pairs (cta_group::2 MMAs over two SMs, 256-row tiles: each SM loads half of a tile's B, a third less operand
// traffic per SM for the same MMA work).  Taken by default for row-major GEMMs of more than 256 rows; REAX_GEMM_PAIR=0
// never takes them, =1 always.  Measured on B200: gate-up (M = 2048, K = 4096) 305 -> 291 us unsplit, 280 us with the
// split below; the qkv projection 581 -> 512 us; with a single row of pair tiles (the sliced GEMM at M = 256, 20 us
// launches) the one-SM kernel is 10 % faster.  Both kernels give identical bits, so the choice is a speed setting only.
inline bool pair_wanted(int M) {
  const char* e = std::getenv("REAX_GEMM_PAIR");
  if (e != nullptr && e[0] == '0') return false;
  if (e != nullptr && e[0] == '1') return true;
  return M > 256;
}

// Split last waves of pair tiles: whenever the last wave is partial (REAX_GEMM_SPLIT=0 turns it off).  Measured on
// B200 (gate-up, M = 2048, K = 4096) at 12.1, 6.05, 3.03 and 1.51 waves of pair tiles: 291 -> 280, 172 -> 160, 95 ->
// 84 and 55 -> 50 us.
inline bool split_wanted_pairs(int tiles, int clusters) {
  if (tiles <= clusters || tiles % clusters == 0) return false;
  const char* e = std::getenv("REAX_GEMM_SPLIT");
  return !(e != nullptr && e[0] == '0');
}

// pipeline depth of the pair kernel: as many stages as shared memory holds (a pair's stage carries half of B)
template <int BN, int KIND>
constexpr int pair_stages() {
  constexpr int room = 232448 - 1024 - reax::gemm_epi_warps(KIND) * 32 * 128 - 256;
  constexpr int st = room / (int)reax::gemm_stage_bytes<BN, true>();
  return st > 8 ? 8 : st;
}

// Clusters of two of `kernel` that fit on device `dev` at once (0: none, or the query failed), kept per device.
template <typename K>
inline int pair_clusters(K kernel, int smem, int threads, int dev, int sms) {
  static std::mutex mu;
  static std::map<int, int> cache;
  std::lock_guard<std::mutex> lk(mu);
  auto it = cache.find(dev);
  if (it != cache.end()) return it->second;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(sms & ~1));
  cfg.blockDim = dim3((unsigned)threads);
  cfg.dynamicSmemBytes = (size_t)smem;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = 2;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, kernel, &cfg) != cudaSuccess) {
    (void)cudaGetLastError();
    n = 0;
  }
  cache[dev] = n;
  return n;
}

// Launch codes follow the reference: 1 = not implementable, 2 = initialisation (attribute) failure,
// 3/4 = launch failure (caller maps), 0 = ok.
// `fixed`: scratch supplied by the caller for the split kernel (flags, partial slots for every SM, the launch's
// epoch); when given, nothing is allocated here.
template <int BN, int ST, int KIND>
inline int launch_gemm(const GemmProblem& pr, cudaStream_t stream, int launch_err_code,
                       const SplitScratch* fixed = nullptr) {
  using namespace reax;
  static SmemAttr attr;
  constexpr int SMEM = gemm_smem_bytes<BN, ST, KIND>();
  static_assert(SMEM <= 232448, "shared memory");
  if (pr.M <= 0 || pr.Nacc <= 0 || pr.S <= 0) return 0;
  CUtensorMap ma, mb;
  const uint64_t row_bytes = (uint64_t)pr.K * 2;
  const uint64_t seg_bytes = (uint64_t)pr.Kseg * 2;
  {
    const uint64_t dims[3] = {(uint64_t)pr.Kseg, (uint64_t)pr.S, (uint64_t)pr.M};
    const uint64_t strides[2] = {seg_bytes, row_bytes};
    const uint32_t box[3] = {64, 1, 128};
    if (!make_map_bf16(&ma, pr.a, 3, dims, strides, box)) return 1;
  }
  {
    const uint64_t dims[3] = {(uint64_t)pr.Kseg, (uint64_t)pr.S, (uint64_t)pr.Nacc};
    const uint64_t strides[2] = {seg_bytes, row_bytes};
    const uint32_t box[3] = {64, 1, (uint32_t)BN};
    if (!make_map_bf16(&mb, pr.b, 3, dims, strides, box)) return 1;
  }
  GemmParams p;
  p.M = pr.M;
  p.Nacc = pr.Nacc;
  p.Kseg = pr.Kseg;
  p.S = pr.S;
  p.nM = (pr.M + 127) / 128;
  p.nN = (pr.Nacc + BN - 1) / BN;
  p.num_tiles = p.S * p.nM * p.nN;
  p.out = pr.out;
  p.ld_out = pr.ld_out;
  p.batch_out = pr.batch_out;
  p.out_cols = pr.out_cols;
  constexpr int ES = (KIND == EPI_F32 || KIND == EPI_F32_T) ? 4 : 2;
  p.silu_tab = pr.silu_tab;
  if (KIND == EPI_GV && p.silu_tab == nullptr) return 2;
  p.vec16 = ((reinterpret_cast<uintptr_t>(pr.out) & 15) == 0) && ((pr.ld_out * ES) % 16 == 0) &&
            ((pr.batch_out * ES) % 16 == 0);
  p.rr_tiles = p.num_tiles;
  p.part = nullptr;
  p.flag = nullptr;
  p.epoch = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  const int sms = device_sms(dev);
  if constexpr (KIND != EPI_BF16_T && KIND != EPI_F32_T && BN >= 64) {
    if (pair_wanted(pr.M)) {
      constexpr int PST = pair_stages<BN, KIND>();
      constexpr int PSMEM = gemm_smem_bytes<BN, PST, KIND, true>();
      static_assert(PSMEM <= 232448, "shared memory");
      static SmemAttr attr_pair, attr_pair_split;
      auto kern = gemm_kernel<BN, PST, KIND, false, true>;
      auto kern_split = gemm_kernel<BN, PST, KIND, true, true>;
      if (ensure_smem(attr_pair, kern, PSMEM) != cudaSuccess) return 2;
      const int ncl = pair_clusters(kern, PSMEM, gemm_threads(KIND), dev, sms);
      if (ncl > 0) {
        // each CTA of a pair loads half of the tile's B rows
        CUtensorMap mb2;
        const uint64_t dims[3] = {(uint64_t)pr.Kseg, (uint64_t)pr.S, (uint64_t)pr.Nacc};
        const uint64_t strides[2] = {seg_bytes, row_bytes};
        const uint32_t box[3] = {64, 1, (uint32_t)(BN / 2)};
        if (!make_map_bf16(&mb2, pr.b, 3, dims, strides, box)) return 1;
        GemmParams pp = p;
        pp.nM = (pr.M + 255) / 256;
        pp.num_tiles = pp.S * pp.nM * pp.nN;
        pp.rr_tiles = pp.num_tiles;
        cudaLaunchAttribute at[1];
        at[0].id = cudaLaunchAttributeClusterDimension;
        at[0].val.clusterDim.x = 2;
        at[0].val.clusterDim.y = 1;
        at[0].val.clusterDim.z = 1;
        cudaLaunchConfig_t cfg = {};
        cfg.blockDim = dim3((unsigned)gemm_threads(KIND));
        cfg.dynamicSmemBytes = (size_t)PSMEM;
        cfg.stream = stream;
        cfg.attrs = at;
        cfg.numAttrs = 1;
        if (split_wanted_pairs(pp.num_tiles, ncl) &&
            ensure_smem(attr_pair_split, kern_split, PSMEM) == cudaSuccess) {
          // split last waves over the clusters: every CTA of the grid is resident at once (the grid is the number
          // of clusters that fit), which the hand-over between neighbouring clusters needs
          auto launch = [&](const SplitScratch& sc) -> int {
            pp.rr_tiles = split_rr_tiles(pp.num_tiles, ncl);
            pp.part = sc.part;
            pp.flag = sc.flag;
            pp.epoch = sc.epoch;
            cfg.gridDim = dim3((unsigned)(2 * ncl));
            if (cudaLaunchKernelEx(&cfg, kern_split, ma, mb2, pp) != cudaSuccess) {
              (void)cudaGetLastError();
              return launch_err_code;
            }
            return 0;
          };
          if (fixed != nullptr) return launch(*fixed);
          int rc = 0;
          if (with_split_scratch(dev, stream, sms, launch, rc)) return rc;
        }
        const int clusters = pp.num_tiles < ncl ? pp.num_tiles : ncl;
        cfg.gridDim = dim3((unsigned)(2 * clusters));
        if (cudaLaunchKernelEx(&cfg, kern, ma, mb2, pp) != cudaSuccess) {
          (void)cudaGetLastError();
          return launch_err_code;
        }
        return 0;
      }
    }
    if (split_wanted(p.num_tiles, sms)) {
      static SmemAttr attr_split;
      if (ensure_smem(attr_split, gemm_kernel<BN, ST, KIND, true>, SMEM) != cudaSuccess) return 2;
      auto launch = [&](const SplitScratch& sc) -> int {
        // all whole waves but two in the raster; the rest (at least 1 and at most 3 waves) is split by k-blocks
        p.rr_tiles = split_rr_tiles(p.num_tiles, sms);
        p.part = sc.part;
        p.flag = sc.flag;
        p.epoch = sc.epoch;
        gemm_kernel<BN, ST, KIND, true><<<sms, gemm_threads(KIND), SMEM, stream>>>(ma, mb, p);
        return cudaGetLastError() == cudaSuccess ? 0 : launch_err_code;
      };
      if (fixed != nullptr) return launch(*fixed);
      int rc = 0;
      if (with_split_scratch(dev, stream, sms, launch, rc)) return rc;
    }
  }
  if (ensure_smem(attr, gemm_kernel<BN, ST, KIND>, SMEM) != cudaSuccess) return 2;
  const int grid = p.num_tiles < sms ? p.num_tiles : sms;
  gemm_kernel<BN, ST, KIND><<<grid, gemm_threads(KIND), SMEM, stream>>>(ma, mb, p);
  return cudaGetLastError() == cudaSuccess ? 0 : launch_err_code;
}

// X with few rows (M <= 64): run the swapped problem C^T = W X^T so that W's rows fill the 128-row MMA dimension and
// every CTA streams a slab of W with a narrow X tile (32 or 64 columns); KIND_T writes the transposed tile back as
// the [M][N] output.  All configuration indices take this path for such M, so they still give identical bits.
template <int KIND_T>
inline int launch_gemm_swapped(const GemmProblem& pr, cudaStream_t stream, int launch_err_code) {
  GemmProblem sw = pr;
  sw.a = pr.b;
  sw.b = pr.a;
  sw.M = pr.Nacc;
  sw.Nacc = pr.M;
  sw.out_cols = pr.M;  // output rows
  if (pr.M <= 32) return launch_gemm<32, 10, KIND_T>(sw, stream, launch_err_code);
  return launch_gemm<64, 8, KIND_T>(sw, stream, launch_err_code);
}

}  // namespace reax_host
