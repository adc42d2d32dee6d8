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
//   P1  warps 0-3: diagonal block w of k k^T (bf16 mma.sync, fp32 accumulate), turned into both heads' L_ii in the
//       epilogue: (raw * 2^(g_r - g_c)) * beta_r with 2^x by MUFU ex2 as the reference computes it, stored fp32 and
//       transposed for the solve;
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
    uint4 k[64 * 16];                // k chunk: row r, 16-byte chunk c at r*16 + (c ^ (r & 7)); dead after P2
    uint16_t aoff[2][6][2][256];     // per head: off-diagonal inverse blocks (index i(i-1)/2 + j), hi and lo tiles
  } u;
  float ld[2][4][324];               // per head: L_ii transposed (L[r][m] at m*20 + r); A_ii's tile pair overlays it.
                                     // 324 floats apart (4 banks): the same word of all 8 blocks sits in 8 bank quads
  uint16_t loff[2][6][2][256];       // per head: -L_ij (i > j), hi and lo tiles
  float g[2][64];
  float beta[2][64];
};

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
  KktSmem& S = *reinterpret_cast<KktSmem*>(smem_raw);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, gq = lane >> 2, tq = lane & 3;
  const long long i_n = cidx[2 * blockIdx.x], i_t = cidx[2 * blockIdx.x + 1];
  const int kh = blockIdx.y;
  const long long bos = cu[i_n], T = cu[i_n + 1] - bos;
  const long long t0 = i_t * 64;
  const int nval = (int)min(64LL, T - t0);
  if (nval <= 0) return;

  // ---- P0: k chunk (cp.async, rows >= nval zero-filled), g, beta
  const uint32_t kbase = smem_u32(S.u.k);
  {
    // thread: 16-byte chunk c = tid & 15 of rows tid / 16 + 16e (the swizzle r & 7 is the same for all four rows)
    const int c = tid & 15, r0 = tid >> 4;
    const uint16_t* src = k + ((bos + t0 + r0) * H + kh) * 128 + 8 * c;
    const uint32_t dst = kbase + (uint32_t)((r0 * 16 + (c ^ (r0 & 7))) * 16);
    const long long rstep = 16LL * H * 128;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const bool ok = r0 + 16 * e < nval;
      cp_async16(dst + 4096u * e, ok ? src + rstep * e : k, ok);
    }
  }
  cp_async_commit();
  if (tid < 128) {
    const int v = tid >> 6, r = tid & 63, hv = kh * 2 + v;
    S.g[v][r] = r < nval ? g[(bos + t0 + r) * HV + hv] : 0.f;
    S.beta[v][r] = r < nval ? __uint_as_float((uint32_t)beta[(bos + t0 + r) * HV + hv] << 16) : 0.f;
  }
  cp_async_wait<0>();
  __syncthreads();

  // k k^T fragments: A operand rows 16bi + (lane & 15) at k-chunk 2kk + (lane >> 4); B operand (k^T, keys as n) rows
  // 16bj + 8nt + (lane & 7) at k-chunk 2kk + (lane >> 3), which covers k-steps kk and kk + 1 in one ldmatrix.x4
  auto ka = [&](int bi, int kk) {
    const int row = 16 * bi + (lane & 15), c = 2 * kk + (lane >> 4);
    return kbase + (uint32_t)((row * 16 + (c ^ (row & 7))) * 16);
  };
  auto kb = [&](int bj, int nt, int kk) {
    const int row = 16 * bj + 8 * nt + (lane & 7), c = 2 * kk + (lane >> 3);
    return kbase + (uint32_t)((row * 16 + (c ^ (row & 7))) * 16);
  };
  // B operand of both n-tiles of block bj at one k-step: keys 16bj + (lane & 7) + 8 (lane >> 4), chunk 2kk + bit 3
  auto kb2 = [&](int bj, int kk) {
    const int row = 16 * bj + (lane & 7) + 8 * (lane >> 4), c = 2 * kk + ((lane >> 3) & 1);
    return kbase + (uint32_t)((row * 16 + (c ^ (row & 7))) * 16);
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
    // ---- P1: diagonal block bb = warp of k k^T -> L_ii of both heads (fp32, transposed)
    {
      const int bb = warp;
      float c[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        uint32_t a[4], b[4];
        ldsm_x4(a, ka(bb, kk));
        ldsm_x4(b, kb2(bb, kk));
        mma_bf16_16816(c[0], a, b[0], b[1]);
        mma_bf16_16816(c[1], a, b[2], b[3]);
      }
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
    // ---- P1/P2 (warps 4-7, alongside): off-diagonal blocks of k k^T -> -L_ij tile pairs of both heads.  Warp u does
    // one whole block (fi, fj) and one 16x8 half (hi_, 1, hnt), sharing the A fragments when both lie in one row panel:
    //   u = 0: (3,0) + (3,1)/0   u = 1: (3,2) + (3,1)/1   u = 2: (2,0) + (2,1)/0   u = 3: (1,0) + (2,1)/1
    const int u = warp - 4;
    const int fi = u < 2 ? 3 : (u == 2 ? 2 : 1), fj = u == 1 ? 2 : 0;
    const int hi_ = u < 2 ? 3 : 2, hj = 1, hnt = u & 1;
    const bool shared_a = fi == hi_;
    float cf[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}}, ch[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int kk = 0; kk < 8; kk += 2) {
      uint32_t a0[4], a1[4], b0[4], b1[4];
      ldsm_x4(a0, ka(fi, kk));
      ldsm_x4(a1, ka(fi, kk + 1));
      ldsm_x4(b0, kb2(fj, kk));
      ldsm_x4(b1, kb2(fj, kk + 1));
      mma_bf16_16816(cf[0], a0, b0[0], b0[1]);
      mma_bf16_16816(cf[1], a0, b0[2], b0[3]);
      mma_bf16_16816(cf[0], a1, b1[0], b1[1]);
      mma_bf16_16816(cf[1], a1, b1[2], b1[3]);
      if (shared_a) {
        uint32_t bh[4];
        ldsm_x4(bh, kb(hj, hnt, kk));
        mma_bf16_16816(ch, a0, bh[0], bh[1]);
        mma_bf16_16816(ch, a1, bh[2], bh[3]);
      }
    }
    if (!shared_a) {
#pragma unroll
      for (int kk = 0; kk < 8; kk += 2) {
        uint32_t a0[4], a1[4], bh[4];
        ldsm_x4(a0, ka(hi_, kk));
        ldsm_x4(a1, ka(hi_, kk + 1));
        ldsm_x4(bh, kb(hj, hnt, kk));
        mma_bf16_16816(ch, a0, bh[0], bh[1]);
        mma_bf16_16816(ch, a1, bh[2], bh[3]);
      }
    }
#pragma unroll
    for (int v2 = 0; v2 < 2; ++v2) {
      const RowV rf = rowv(v2, fi, -1.f);
      const RowV rh = shared_a ? rf : rowv(v2, hi_, -1.f);
      float x[2][4], z[4];
      decay(cf[0], x[0], rf, v2, fi, fj, 0, false);
      decay(cf[1], x[1], rf, v2, fi, fj, 1, false);
      decay(ch, z, rh, v2, hi_, hj, hnt, false);
      uint32_t h[4], l[4];
      split_c(x, h, l);
      const uint32_t tf = smem_u32(S.loff[v2][kkt_oidx(fi, fj)]) + lo16;
      stsm_x4(tf, h);
      stsm_x4(tf + 512, l);
      // half block: matrices (rows 0-7, half hnt) and (rows 8-15, half hnt); lanes 0-15 give the row addresses
      const uint32_t th = smem_u32(S.loff[v2][kkt_oidx(hi_, hj)]) +
                          (uint32_t)((lane & 15) * 32 + (((hnt ^ (lane >> 2)) & 1) << 4));
      uint32_t h0, l0, h1, l1;
      split_pair(z[0], z[1], h0, l0);
      split_pair(z[2], z[3], h1, l1);
      stsm_x2(th, h0, h1);
      stsm_x2(th + 512, l0, l1);
    }
  }
  __syncthreads();

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
    if (reax_host::ensure_smem(attr, reax::kkt_kernel, (int)sizeof(reax::KktSmem), true) != cudaSuccess)                   \
      return (int)cudaErrorInvalidValue;                                                                              \
    reax::kkt_kernel<<<dim3(NT, H), 256, sizeof(reax::KktSmem), (cudaStream_t)stream>>>(                              \
        (const uint16_t*)k, (const float*)g, (const uint16_t*)beta, (uint16_t*)A, (const long long*)cu,               \
        (const long long*)cidx, H, HV);                                                                               \
    return (int)cudaGetLastError();                                                                                   \
  }                                                                                                                   \
  REAX_API int reax_kkt_smem() { return (int)sizeof(reax::KktSmem); }
