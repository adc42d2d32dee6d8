// Chunked KKT + unit-lower-triangular inverse for the gated delta rule, sm_100a.
//
// Semantics (libreax_howu/reax_kkt.cu:85-104 inputs, :133-159 decay/mask/beta, :160-245 inverse, :246-260 writes):
//   per chunk c of sequence n (tokens bos + 64c .. + nval) and value head hv (key head hv / 2):
//     L[r][s] = beta[r] * (k_r . k_s) * 2^(g[r] - g[s])  for s < r < nval (else 0);   A = (I + L)^-1
//   A is written as bf16 for rows r < nval and 16x16 blocks on or below the diagonal only (columns < 16*(r/16+1));
//   the strictly-upper 16x16 blocks are never written.
//
// One CTA per (chunk, key head) = both value heads of that key head (the raw k k^T is shared), 256 threads, five
// phases:
//   P0  k chunk -> shared memory by 16-byte cp.async (rows >= nval zero-filled), g and beta of both heads;
//   P1  k k^T (64 x 64, K = 128) on the tensor core: eight tcgen05 MMAs (M = N = 64, the k tile as both operands)
//       issued by one thread into 64 TMEM columns; warps 0-3 read diagonal block w back (tcgen05.ld in the m16n8
//       fragment layout) and turn it into both heads' L_ii: (raw * 2^(g_r - g_c)) * beta_r with 2^x by MUFU ex2 as
//       the reference computes it, stored fp32 and transposed for the solve;
//   P2  warps 0-3: A_ii = (I + L_ii)^-1 by forward substitution, one thread per column (right-looking: the
//       dependent chain is 16 FMAs long), between two barriers of their own.  Warps 4-7 meanwhile (through P1 and
//       P2): the six off-diagonal blocks of k k^T -> -L_ij, one 16-row panel per warp where possible so that the A
//       fragments are loaded once;
//   P3  the off-diagonal inverse blocks from A (I + L) = I, i.e. for i > j
//           A_ij = -(sum_{k=j+1..i} A_ik L_kj) A_jj,
//       as three dependent rounds per head (4 warps per head, per-head named barriers): round 1 A_10, A_21, A_32 and
//       the partial sums A_22 L_20, A_33 L_31, A_33 L_30; round 2 A_20, A_31 and A_32 L_20; round 3 A_30;
//   P4  coalesced 16-byte bf16 stores of the written set.
//
// Every 16x16 operand of the P3 products (L_ij for i > j and all A blocks) is held once in shared memory as a pair
// of bf16 tiles x = hi + lo (hi = bf16(x) round-to-nearest, lo = bf16(x - hi)), so one 16x16x16 product is four
// ldmatrix and six m16n8k16 mma (lo*hi + hi*lo + hi*hi, fp32 accumulate): about 2^-16 relative per product where
// the reference used single TF32 products (2^-11).  The partial sum sum_k A_ik L_kj is the LEFT factor of the
// final product, so its accumulator fragments are reused as the A operand in registers (the m16n8 C layout of two
// n-tiles is the m16k16 A layout).  The hi tile of an inverse block is exactly its bf16 output.
//
// Tile layout (512 bytes, bf16 16x16 row-major, 16-byte halves swizzled by row bit 2): element (r, c) at byte
// r*32 + (((c >> 3) ^ ((r >> 2) & 1)) << 4) + (c & 7)*2.  With lane address row = lane & 15, half = lane >> 4 the
// same per-lane offset serves ldmatrix.x4 (A operand), ldmatrix.x4.trans (B operand of a row-major [k][n] tile)
// and stmatrix.x4 (C fragments of two n-tiles), all bank-conflict free.
#pragma once
#include "common.cuh"

namespace reax {

struct KktSmem {
  union {
    uint8_t k[2][64 * 128];          // k chunk in the tcgen05 operand layout (K-major, 128-byte swizzle): dims
                                     // 64h..64h+63 of row r at h*8192 + r*128 + ((c ^ (r & 7)) << 4), c the 16-byte
                                     // chunk; dead once the k k^T MMAs have completed
    uint16_t aoff[2][6][2][256];     // per head: off-diagonal inverse blocks (index i(i-1)/2 + j), hi and lo tiles
  } u;
  float ld[2][4][324];               // per head: L_ii transposed (L[r][m] at m*20 + r); A_ii's tile pair overlays it.
                                     // 324 floats apart (4 banks): the same word of all 8 blocks sits in 8 bank quads
  uint16_t loff[2][6][2][256];       // per head: -L_ij (i > j), hi and lo tiles
  float g[2][64];
  float beta[2][64];
  unsigned long long bar;            // k k^T accumulator complete
  uint32_t tmem;                     // TMEM base of the 64-column accumulator
  int abort;
};
constexpr int kKktSmemBytes = (int)sizeof(KktSmem) + 1024;  // + slack: the k tile starts on a 1024-byte boundary

__device__ __forceinline__ int kkt_oidx(int i, int j) { return i * (i - 1) / 2 + j; }

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr)
               : "memory");
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr)
               : "memory");
}
__device__ __forceinline__ void stsm_x4(uint32_t addr, const uint32_t (&r)[4]) {
  asm volatile("stmatrix.sync.aligned.m8n8.x4.shared.b16 [%0], {%1,%2,%3,%4};\n" ::"r"(addr), "r"(r[0]), "r"(r[1]),
               "r"(r[2]), "r"(r[3])
               : "memory");
}
__device__ __forceinline__ void stsm_x2(uint32_t addr, uint32_t r0, uint32_t r1) {
  asm volatile("stmatrix.sync.aligned.m8n8.x2.shared.b16 [%0], {%1,%2};\n" ::"r"(addr), "r"(r0), "r"(r1) : "memory");
}
__device__ __forceinline__ void mma_bf16_16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
               : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
               : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// (x0, x1) -> packed hi = bf16x2(x0, x1) and lo = bf16x2(x0 - hi0, x1 - hi1); x - hi is exact in fp32
__device__ __forceinline__ void split_pair(float x0, float x1, uint32_t& h, uint32_t& l) {
  h = pack_bf16(x0, x1);
  l = pack_bf16(__fsub_rn(x0, bf_lo(h)), __fsub_rn(x1, bf_hi(h)));
}
// accumulator fragments of two n-tiles (rows gq, gq+8; columns 8nt + 2tq + {0,1}) -> A-operand / stmatrix registers
__device__ __forceinline__ void split_c(const float (&c)[2][4], uint32_t (&h)[4], uint32_t (&l)[4]) {
  split_pair(c[0][0], c[0][1], h[0], l[0]);
  split_pair(c[0][2], c[0][3], h[1], l[1]);
  split_pair(c[1][0], c[1][1], h[2], l[2]);
  split_pair(c[1][2], c[1][3], h[3], l[3]);
}
// acc += X Y, X given as A-operand registers (hi, lo), Y a tile pair at this lane's address y (lo tile at y + 512)
__device__ __forceinline__ void kkt_mm_ft(float (&acc)[2][4], const uint32_t (&xh)[4], const uint32_t (&xl)[4], uint32_t y) {
  uint32_t bh[4], bl[4];
  ldsm_x4_t(bh, y);
  ldsm_x4_t(bl, y + 512);
  mma_bf16_16816(acc[0], xl, bh[0], bh[1]);
  mma_bf16_16816(acc[1], xl, bh[2], bh[3]);
  mma_bf16_16816(acc[0], xh, bl[0], bl[1]);
  mma_bf16_16816(acc[1], xh, bl[2], bl[3]);
  mma_bf16_16816(acc[0], xh, bh[0], bh[1]);
  mma_bf16_16816(acc[1], xh, bh[2], bh[3]);
}
// acc += X Y, both tile pairs
__device__ __forceinline__ void kkt_mm_tt(float (&acc)[2][4], uint32_t x, uint32_t y) {
  uint32_t xh[4], xl[4];
  ldsm_x4(xh, x);
  ldsm_x4(xl, x + 512);
  kkt_mm_ft(acc, xh, xl, y);
}
// dst tile pair = Y' A_jj with Y' = sum_k A_ik (-L_kj) in acc (so dst = A_ij)
__device__ __forceinline__ void kkt_finish(const float (&y)[2][4], uint32_t ajj, uint32_t dst) {
  uint32_t h[4], l[4];
  split_c(y, h, l);
  float r[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
  kkt_mm_ft(r, h, l, ajj);
  split_c(r, h, l);
  stsm_x4(dst, h);
  stsm_x4(dst + 512, l);
}

// Forward substitution for columns j = 4W + jj of one diagonal block: x = (I + L)^-1 e_j with Lt[m*20 + r] = L[r][m].
// Right-looking: once x[m] is final it is applied to every later row, so each x[r] still accumulates its terms in
// the order m = 0, 1, .. while the dependent chain is 16 FMAs long.  x[m] = 0 for m < j, so the steps below 4W are
// skipped for the whole warp.
template <int W>
__device__ __forceinline__ void kkt_solve_cols(const float* Lt, int j, float (&x)[16]) {
#pragma unroll
  for (int r = 0; r < 16; ++r) x[r] = r == j ? 1.f : 0.f;
#pragma unroll
  for (int m = 4 * W; m < 15; ++m) {
    float lm[16];
#pragma unroll
    for (int q = (m + 1) / 4; q < 4; ++q) {
      const float4 t4 = *reinterpret_cast<const float4*>(&Lt[m * 20 + 4 * q]);
      lm[4 * q] = t4.x;
      lm[4 * q + 1] = t4.y;
      lm[4 * q + 2] = t4.z;
      lm[4 * q + 3] = t4.w;
    }
#pragma unroll
    for (int r = m + 1; r < 16; ++r) x[r] = __fmaf_rn(-lm[r], x[m], x[r]);
  }
}

__global__ void __launch_bounds__(256, 5)
kkt_kernel(const uint16_t* __restrict__ k, const float* __restrict__ g, const uint16_t* __restrict__ beta,
           uint16_t* __restrict__ A, const long long* __restrict__ cu, const long long* __restrict__ cidx, int H, int HV) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  KktSmem& S = *reinterpret_cast<KktSmem*>(smem_raw + (((raw + 1023u) & ~1023u) - raw));
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, gq = lane >> 2, tq = lane & 3;
  const long long i_n = cidx[2 * blockIdx.x], i_t = cidx[2 * blockIdx.x + 1];
  const int kh = blockIdx.y;
  const long long bos = cu[i_n], T = cu[i_n + 1] - bos;
  const long long t0 = i_t * 64;
  const int nval = (int)min(64LL, T - t0);
  if (nval <= 0) return;

  // ---- P0: TMEM (64 columns), the MMA barrier, k chunk (cp.async, rows >= nval zero-filled), g, beta
  if (warp == 0) {
    tmem_alloc(smem_u32(&S.tmem), 64);
    tmem_relinquish();
  }
  const uint32_t bar = smem_u32(&S.bar);
  if (tid == 0) {
    mbar_init(bar, 1);
    fence_mbar_init();
    S.abort = 0;
  }
  const uint32_t kbase = smem_u32(S.u.k);
  {
    // thread: 16-byte chunk c16 = tid & 15 of rows tid / 16 + 16e (the swizzle r & 7 is the same for all four rows)
    const int c16 = tid & 15, r0 = tid >> 4;
    const uint16_t* src = k + ((bos + t0 + r0) * H + kh) * 128 + 8 * c16;
    const uint32_t dst = kbase + (uint32_t)((c16 >> 3) * 8192 + r0 * 128 + (((c16 & 7) ^ (r0 & 7)) << 4));
    const long long rstep = 16LL * H * 128;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const bool ok = r0 + 16 * e < nval;
      cp_async16(dst + 2048u * e, ok ? src + rstep * e : k, ok);
    }
  }
  cp_async_commit();
  if (tid < 128) {
    const int v = tid >> 6, r = tid & 63, hv = kh * 2 + v;
    S.g[v][r] = r < nval ? g[(bos + t0 + r) * HV + hv] : 0.f;
    S.beta[v][r] = r < nval ? __uint_as_float((uint32_t)beta[(bos + t0 + r) * HV + hv] << 16) : 0.f;
  }
  cp_async_wait<0>();
  fence_proxy_async_smem();  // the k tile is read by the tensor core (async proxy)
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = S.tmem;

  // ---- P1: k k^T on the tensor core: 8 MMAs (M = N = 64, K = 16 each; A and B are both the k tile), issued by one
  // thread; accumulator row 16q + i in TMEM lane 32q + i, column = key
  if (tid == 0) {
    constexpr uint32_t IDESC = idesc_bf16(64, 64);
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      const uint64_t d = sw128_desc(kbase + (uint32_t)((kk >> 2) * 8192 + (kk & 3) * 32));
      mma_bf16_ss(tmem, d, d, IDESC, kk > 0);
    }
    mma_commit(bar);
  }
  if (!__syncthreads_and(mbar_wait(bar, 0, &S.abort, ST_TIMEOUT_KKT))) {
    // gave up: let the MMAs finish (bounded) before the TMEM is released, write nothing
    if (warp == 0) {
      if (lane == 0) {
        const long long tw = clock64();
        while (!mbar_try_wait(bar, 0) && clock64() - tw < REAX_DRAIN_LIMIT) {
        }
      }
      __syncwarp();
      tc_fence_after();
      tmem_dealloc(tmem, 64);
    }
    return;
  }
  tc_fence_after();
  // the 16x16 block (bi, bj) of k k^T as two m16n8 accumulator fragments (warp w may read lane quarter w % 4 only)
  auto kkt_block = [&](float (&c)[2][4], int bi, int bj) {
    uint32_t r[8];
    tmem_ld_16x256b_x2(tmem + ((uint32_t)(32 * bi) << 16) + (uint32_t)(16 * bj), r);
#pragma unroll
    for (int e = 0; e < 8; ++e) c[e >> 2][e & 3] = __uint_as_float(r[e]);
  };
  // (raw * 2^(g_r - g_c)) * beta_r for the fragment elements (rows 16bi + gq (+8), columns 16bj + 8nt + 2tq (+1)),
  // zero outside the mask (a diagonal block always needs it, an off-diagonal one only in a partial chunk);
  // sgn = -1 gives -L.  The row values of a head and row panel are read once (RowV).
  const bool partial = nval < 64;
  struct RowV {
    float gA, gB, bA, bB;
  };
  auto rowv = [&](int v2, int bi, float sgn) {
    const int rA = 16 * bi + gq;
    return RowV{S.g[v2][rA], S.g[v2][rA + 8], sgn * S.beta[v2][rA], sgn * S.beta[v2][rA + 8]};
  };
  auto decay = [&](const float (&c)[4], float (&x)[4], const RowV& rv, int v2, int bi, int bj, int nt, bool diag) {
    const int c0 = 16 * bj + 8 * nt + 2 * tq;
    const float2 gc = *reinterpret_cast<const float2*>(&S.g[v2][c0]);
    float e[4] = {ex2_approx(__fsub_rn(rv.gA, gc.x)), ex2_approx(__fsub_rn(rv.gA, gc.y)),
                  ex2_approx(__fsub_rn(rv.gB, gc.x)), ex2_approx(__fsub_rn(rv.gB, gc.y))};
    if (diag || partial) {
      const int rA = 16 * bi + gq;
#pragma unroll
      for (int qq = 0; qq < 4; ++qq) {
        const int r = qq < 2 ? rA : rA + 8, cc = c0 + (qq & 1);
        if (!(r < nval && cc < nval && r > cc)) e[qq] = 0.f;
      }
    }
    const uint64_t xA = f2mul(f2mul(f2(c[0], c[1]), f2(e[0], e[1])), f2(rv.bA, rv.bA));
    const uint64_t xB = f2mul(f2mul(f2(c[2], c[3]), f2(e[2], e[3])), f2(rv.bB, rv.bB));
    f2get(xA, x[0], x[1]);
    f2get(xB, x[2], x[3]);
  };

  // per-lane offset into a tile for ldmatrix / stmatrix (row lane & 15, 16-byte half lane >> 4, swizzled)
  const uint32_t lo16 = (uint32_t)((lane & 15) * 32 + ((((lane >> 4) ^ (lane >> 2)) & 1) << 4));

  if (warp < 4) {
    // ---- P1 epilogue: diagonal block bb = warp -> L_ii of both heads (fp32, transposed)
    {
      const int bb = warp;
      float c[2][4];
      kkt_block(c, bb, bb);
#pragma unroll
      for (int v2 = 0; v2 < 2; ++v2) {
        const RowV rv = rowv(v2, bb, 1.f);
        float* Lt = S.ld[v2][bb];
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) {
          float x[4];
          decay(c[nt], x, rv, v2, bb, bb, nt, true);
          const int lr = gq, lc = 8 * nt + 2 * tq;
          Lt[lc * 20 + lr] = x[0];
          Lt[(lc + 1) * 20 + lr] = x[1];
          Lt[lc * 20 + lr + 8] = x[2];
          Lt[(lc + 1) * 20 + lr + 8] = x[3];
        }
      }
    }
    named_bar_sync<1, 128>();  // all eight L_ii stored

    // ---- P2: A_ii by forward substitution; lane = 4 (4v + bb) + jj owns column j = 4 warp + jj of block (v, bb),
    // so that a warp's columns share their zero prefix
    const int blk = lane >> 2, v = blk >> 2, bb = blk & 3, j = 4 * warp + (lane & 3);
    const float* Lt = S.ld[v][bb];
    float x[16];
    switch (warp) {
      case 0: kkt_solve_cols<0>(Lt, j, x); break;
      case 1: kkt_solve_cols<1>(Lt, j, x); break;
      case 2: kkt_solve_cols<2>(Lt, j, x); break;
      default: kkt_solve_cols<3>(Lt, j, x); break;
    }
    // column pairs (j, j^1) -> packed words: even j writes rows 0-7, odd j rows 8-15
    const bool odd = j & 1;
    float y[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) y[q] = __shfl_xor_sync(0xffffffffu, odd ? x[q] : x[q + 8], 1);
    // every column of every diagonal block is final before any tile pair overwrites an L_ii (each warp reads all 8)
    named_bar_sync<1, 128>();
    const uint32_t tile = smem_u32(Lt);
    const int c0 = j & ~1;
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const int r = odd ? q + 8 : q;
      uint32_t h, l;
      if (odd) split_pair(y[q], x[q + 8], h, l);
      else split_pair(x[q], y[q], h, l);
      const uint32_t a = tile + (uint32_t)(r * 32 + ((((c0 >> 3) ^ (r >> 2)) & 1) << 4) + (c0 & 7) * 2);
      asm volatile("st.shared.b32 [%0], %1;" ::"r"(a), "r"(h) : "memory");
      asm volatile("st.shared.b32 [%0], %1;" ::"r"(a + 512), "r"(l) : "memory");
    }
  } else {
    // ---- P1 epilogue / P2 (warps 4-7, alongside the solve): off-diagonal blocks (q, j < q) of row q = warp - 4
    // -> -L_qj tile pairs of both heads
    const int qr = warp - 4;
    for (int j = 0; j < qr; ++j) {
      float c[2][4];
      kkt_block(c, qr, j);
#pragma unroll
      for (int v2 = 0; v2 < 2; ++v2) {
        const RowV rv = rowv(v2, qr, -1.f);
        float x[2][4];
        decay(c[0], x[0], rv, v2, qr, j, 0, false);
        decay(c[1], x[1], rv, v2, qr, j, 1, false);
        uint32_t h[4], l[4];
        split_c(x, h, l);
        const uint32_t tf = smem_u32(S.loff[v2][kkt_oidx(qr, j)]) + lo16;
        stsm_x4(tf, h);
        stsm_x4(tf + 512, l);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {  // every TMEM read is done
    tc_fence_after();
    tmem_dealloc(tmem, 64);
  }

  // ---- P3: off-diagonal inverse blocks; warp (v, q): 4 warps per head, per-head named barriers 1 + v
  {
    const int v = warp >> 2, q = warp & 3;
    auto AD = [&](int i) { return smem_u32(S.ld[v][i]) + lo16; };
    auto AO = [&](int i, int j) { return smem_u32(S.u.aoff[v][kkt_oidx(i, j)]) + lo16; };
    auto LO = [&](int i, int j) { return smem_u32(S.loff[v][kkt_oidx(i, j)]) + lo16; };
    float p[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
    // round 1: A_{q+1,q} for q < 3; partial sums A_22 (-L_20), A_33 (-L_31), A_33 (-L_30)
    if (q < 3) {
      float y[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
      kkt_mm_tt(y, AD(q + 1), LO(q + 1, q));
      kkt_finish(y, AD(q), AO(q + 1, q));
    }
    if (q == 0) kkt_mm_tt(p, AD(2), LO(2, 0));
    if (q == 1) kkt_mm_tt(p, AD(3), LO(3, 1));
    if (q == 3) kkt_mm_tt(p, AD(3), LO(3, 0));
    if (v == 0) named_bar_sync<1, 128>();
    else named_bar_sync<2, 128>();
    // round 2: A_20, A_31; A_32 (-L_20) into the (3, 0) partial sum
    if (q == 0) {
      kkt_mm_tt(p, AO(2, 1), LO(1, 0));
      kkt_finish(p, AD(0), AO(2, 0));
    }
    if (q == 1) {
      kkt_mm_tt(p, AO(3, 2), LO(2, 1));
      kkt_finish(p, AD(1), AO(3, 1));
    }
    if (q == 3) kkt_mm_tt(p, AO(3, 2), LO(2, 0));
    if (v == 0) named_bar_sync<1, 128>();
    else named_bar_sync<2, 128>();
    // round 3: A_30
    if (q == 3) {
      kkt_mm_tt(p, AO(3, 1), LO(1, 0));
      kkt_finish(p, AD(0), AO(3, 0));
    }
  }
  __syncthreads();

  // ---- P4: stores from the hi tiles: 2 heads x 64 rows x 8 chunks of 8 columns, blocks on or below the diagonal
  {
    // thread: chunk ch = tid & 7 of rows r0 = tid / 8 and r0 + 32, both heads
    const int ch = tid & 7, r0 = tid >> 3, cb = ch >> 1;
    const uint32_t in_tile = (uint32_t)((r0 & 15) * 32 + ((((ch & 1) ^ (r0 >> 2)) & 1) << 4));
    uint16_t* dst = A + ((bos + t0 + r0) * HV + kh * 2) * 64 + 8 * ch;
#pragma unroll
    for (int it = 0; it < 2; ++it) {
      const int r = r0 + 32 * it, rb = r >> 4;
      if (r < nval && cb <= rb) {
#pragma unroll
        for (int vv = 0; vv < 2; ++vv) {
          const void* tile = cb == rb ? (const void*)S.ld[vv][rb] : (const void*)S.u.aoff[vv][kkt_oidx(rb, cb)][0];
          const uint4 w4 = ld_shared_v4(smem_u32(tile) + in_tile);
          *reinterpret_cast<uint4*>(dst + 32LL * it * HV * 64 + 64 * vv) = w4;
        }
      }
    }
  }
}

}  // namespace reax

// libreax_howu/reax_kkt.cu:263-272 argument list and codes
#define REAX_DEFINE_KKT_EXPORTS()                                                                                   \
  REAX_API int reax_kkt(const void* k, const void* g, const void* beta, void* A, const void* cu, const void* cidx,   \
                        int NT, int H, int HV, void* stream) {                                                       \
    static reax_host::SmemAttr attr;                                                                                  \
    if (HV != 2 * H) return -1;                                                                                       \
    if (NT <= 0 || H <= 0) return 0;                                                                                  \
    if ((((uintptr_t)k | (uintptr_t)A) & 15) || H > 65535) return -1;                                                 \
    if (reax_host::ensure_smem(attr, reax::kkt_kernel, reax::kKktSmemBytes, true) != cudaSuccess)                   \
      return (int)cudaErrorInvalidValue;                                                                              \
    reax::kkt_kernel<<<dim3(NT, H), 256, reax::kKktSmemBytes, (cudaStream_t)stream>>>(                              \
        (const uint16_t*)k, (const float*)g, (const uint16_t*)beta, (uint16_t*)A, (const long long*)cu,               \
        (const long long*)cidx, H, HV);                                                                               \
    return (int)cudaGetLastError();                                                                                   \
  }                                                                                                                   \
  REAX_API int reax_kkt_smem() { return reax::kKktSmemBytes; }
