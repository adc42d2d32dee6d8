// Chunked KKT + unit-lower-triangular inverse for the gated delta rule, sm_100a.
//
// Semantics (libreax_howu/reax_kkt.cu:85-104 inputs, :133-159 decay/mask/beta, :160-245 inverse, :246-260 writes):
//   per chunk c of sequence n (tokens bos + 64c .. + nval) and value head hv (key head hv / 2):
//     L[r][s] = beta[r] * (k_r . k_s) * 2^(g[r] - g[s])  for s < r < nval (else 0);   A = (I + L)^-1
//   A is written as bf16 for rows r < nval and 16x16 blocks on or below the diagonal only (columns < 16*(r/16+1));
//   the strictly-upper 16x16 blocks are never written.
//
// One CTA per (chunk, key head) = both value heads of that key head (the raw k k^T is shared), 256 threads:
//   1. k chunk -> shared memory (16-byte loads);
//   2. k k^T on the 10 lower 16x16 blocks with bf16 mma.sync (fp32 acc), each block turned into both heads' L blocks
//      straight from the accumulator fragments: (raw * 2^(g_r - g_s)) * beta_r in fp32 (masked), 2^x by MUFU ex2 as
//      the reference computes it;
//   3. diagonal blocks A_ii = (I + L_ii)^-1 by forward substitution, one thread per column (right-looking);
//   4. off-diagonal blocks by the blocked recurrence A_ij = -A_ii * sum_{k=j}^{i-1} L_ik A_kj, level by level
//      (i - j = 1, 2, 3), each 16x16 product on the tensor core as three TF32 mma.sync (hi*hi + hi*lo + lo*hi
//      split operands: fp32-level accuracy, where the reference used single TF32 products);
//   5. coalesced 16-byte bf16 stores of the written set.
#pragma once
#include "common.cuh"

namespace reax {

struct KktSmem {
  union {
    uint16_t k[64 * 136];        // k chunk, rows padded to 136 elements (conflict-free ldmatrix); dead after step 2
    struct {
      float Ai[2][10][16 * 17];  // per head: inverse blocks (written from step 3 on)
      float scr[8][16 * 17];     // per warp scratch of step 4
    } p;
  } u;
  float L[2][10][16 * 17];       // per head: decayed, masked, beta-scaled blocks (index i*(i+1)/2 + j), rows padded
  float g[2][64];
  float beta[2][64];
};

__device__ __forceinline__ int kkt_bidx(int i, int j) { return i * (i + 1) / 2 + j; }

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr)
               : "memory");
}
__device__ __forceinline__ void mma_bf16_16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
               : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
               : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void mma_tf32_1688(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile("mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
               : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
               : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t to_tf32(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return r;
}
// x = hi + lo: hi = x with the 13 low mantissa bits cleared (exactly a TF32 value), lo = x - hi exactly; the tensor
// core reads lo's top 19 bits, so hi*y + lo*y carries x to about 2^-21 relative
__device__ __forceinline__ void split_tf32(float x, uint32_t& hi, uint32_t& lo) {
  hi = __float_as_uint(x) & 0xffffe000u;
  lo = __float_as_uint(__fsub_rn(x, __uint_as_float(hi)));
}

// C (16x16, per-thread fragments c[2][4] for two 8-column tiles) += X * Y, X and Y 16x16 fp32 row-major (stride 17)
__device__ __forceinline__ void mm16_acc(float (&c)[2][4], const float* X, const float* Y, int lane) {
  const int gq = lane >> 2, tq = lane & 3;
#pragma unroll
  for (int ks = 0; ks < 2; ++ks) {
    const int k0 = 8 * ks + tq, k1 = k0 + 4;
    uint32_t ah[4], al[4];
    split_tf32(X[gq * 17 + k0], ah[0], al[0]);
    split_tf32(X[(gq + 8) * 17 + k0], ah[1], al[1]);
    split_tf32(X[gq * 17 + k1], ah[2], al[2]);
    split_tf32(X[(gq + 8) * 17 + k1], ah[3], al[3]);
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      uint32_t bh0, bl0, bh1, bl1;
      split_tf32(Y[k0 * 17 + 8 * nt + gq], bh0, bl0);
      split_tf32(Y[k1 * 17 + 8 * nt + gq], bh1, bl1);
      mma_tf32_1688(c[nt], al, bh0, bh1);
      mma_tf32_1688(c[nt], ah, bl0, bl1);
      mma_tf32_1688(c[nt], ah, bh0, bh1);
    }
  }
}
__device__ __forceinline__ void st16(float* M, const float (&c)[2][4], int lane, float sign) {
  const int gq = lane >> 2, tq = lane & 3;
#pragma unroll
  for (int nt = 0; nt < 2; ++nt) {
    M[gq * 17 + 8 * nt + 2 * tq] = sign * c[nt][0];
    M[gq * 17 + 8 * nt + 2 * tq + 1] = sign * c[nt][1];
    M[(gq + 8) * 17 + 8 * nt + 2 * tq] = sign * c[nt][2];
    M[(gq + 8) * 17 + 8 * nt + 2 * tq + 1] = sign * c[nt][3];
  }
}

__global__ void __launch_bounds__(256)
kkt_kernel(const uint16_t* __restrict__ k, const float* __restrict__ g, const uint16_t* __restrict__ beta,
           uint16_t* __restrict__ A, const long long* __restrict__ cu, const long long* __restrict__ cidx, int H, int HV) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  KktSmem& S = *reinterpret_cast<KktSmem*>(smem_raw);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const long long i_n = cidx[2 * blockIdx.x], i_t = cidx[2 * blockIdx.x + 1];
  const int kh = blockIdx.y;
  const long long bos = cu[i_n], T = cu[i_n + 1] - bos;
  const long long t0 = i_t * 64;
  const int nval = (int)min(64LL, T - t0);
  if (nval <= 0) return;

  // ---- 1. load k chunk (rows >= nval zero), g, beta
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const int i = tid + 256 * e, r = i >> 4, c = i & 15;
    uint4 val = make_uint4(0, 0, 0, 0);
    if (r < nval) val = __ldg(reinterpret_cast<const uint4*>(k + ((bos + t0 + r) * H + kh) * 128 + 8 * c));
    *reinterpret_cast<uint4*>(&S.u.k[r * 136 + 8 * c]) = val;
  }
  if (tid < 128) {
    const int v = tid >> 6, r = tid & 63, hv = kh * 2 + v;
    S.g[v][r] = r < nval ? g[(bos + t0 + r) * HV + hv] : 0.f;
    S.beta[v][r] = r < nval ? __uint_as_float((uint32_t)beta[(bos + t0 + r) * HV + hv] << 16) : 0.f;
  }
  __syncthreads();

  // ---- 2. k k^T blocks -> L blocks of both heads: warp w computes block w (and warps 0, 1 also blocks 8, 9)
  auto l_block = [&](int idx) {
    const int bi = (idx >= 1) + (idx >= 3) + (idx >= 6), bj = idx - bi * (bi + 1) / 2;
    float c[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
    const uint32_t kb = smem_u32(S.u.k);
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      uint32_t a[4], b[4];
      // A: rows 16bi + (lane & 15), cols 16kk + 8 (lane >> 4)
      ldsm_x4(a, kb + (uint32_t)(((16 * bi + (lane & 15)) * 136 + 16 * kk + 8 * (lane >> 4)) * 2));
      // B (k^T): rows of k = keys 16bj + (lane & 7) + 8 (lane >> 4), cols 16kk + 8 ((lane >> 3) & 1)
      ldsm_x4(b, kb + (uint32_t)(((16 * bj + (lane & 7) + 8 * (lane >> 4)) * 136 + 16 * kk + 8 * ((lane >> 3) & 1)) * 2));
      mma_bf16_16816(c[0], a, b[0], b[1]);
      mma_bf16_16816(c[1], a, b[2], b[3]);
    }
    // fragment element (nt, qq) is row gq + 8 (qq >> 1), column 8 nt + 2 tq + (qq & 1) of the block
    const int gq = lane >> 2, tq = lane & 3;
    const int rA = 16 * bi + gq, rB = rA + 8;
    const bool all_visible = nval == 64 && bi > bj;  // every element below the diagonal and inside the chunk
#pragma unroll
    for (int v2 = 0; v2 < 2; ++v2) {
      float* Lb = S.L[v2][idx];
      const float gA = S.g[v2][rA], gB = S.g[v2][rB];
      const uint64_t bA2 = f2(S.beta[v2][rA], S.beta[v2][rA]), bB2 = f2(S.beta[v2][rB], S.beta[v2][rB]);
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        const int c0 = 16 * bj + 8 * nt + 2 * tq;
        const float2 gc = *reinterpret_cast<const float2*>(&S.g[v2][c0]);
        float e[4] = {ex2_approx(__fsub_rn(gA, gc.x)), ex2_approx(__fsub_rn(gA, gc.y)), ex2_approx(__fsub_rn(gB, gc.x)),
                      ex2_approx(__fsub_rn(gB, gc.y))};
        if (!all_visible) {
#pragma unroll
          for (int qq = 0; qq < 4; ++qq) {
            const int r = qq < 2 ? rA : rB, cc = c0 + (qq & 1);
            if (!(r < nval && cc < nval && r > cc)) e[qq] = 0.f;
          }
        }
        // (raw * 2^(g_r - g_c)) * beta_r, two elements per instruction
        const uint64_t xA = f2mul(f2mul(f2(c[nt][0], c[nt][1]), f2(e[0], e[1])), bA2);
        const uint64_t xB = f2mul(f2mul(f2(c[nt][2], c[nt][3]), f2(e[2], e[3])), bB2);
        const int lc = 8 * nt + 2 * tq;
        f2get(xA, Lb[gq * 17 + lc], Lb[gq * 17 + lc + 1]);
        f2get(xB, Lb[(gq + 8) * 17 + lc], Lb[(gq + 8) * 17 + lc + 1]);
      }
    }
  };
  l_block(warp);
  if (warp < 2) l_block(warp + 8);
  __syncthreads();

  // ---- 3. diagonal blocks by forward substitution: 2 heads x 4 blocks x 16 columns = 128 threads.  Right-looking:
  // once x[m] is final it is applied to every later row, so each x[r] still accumulates its terms in the order
  // m = 0, 1, .. (the left-looking result bit for bit) while the dependent chain is 16 FMAs long instead of 120.
  if (tid < 128) {
    const int v = tid >> 6, bb = (tid >> 4) & 3, j = tid & 15;
    const float* Lb = S.L[v][kkt_bidx(bb, bb)];
    float x[16];
#pragma unroll
    for (int r = 0; r < 16; ++r) x[r] = r == j ? 1.f : 0.f;
#pragma unroll
    for (int m = 0; m < 16; ++m) {
      if (m < j) x[m] = 0.f;  // the inverse is lower triangular: rows above the column are zero
#pragma unroll
      for (int r = m + 1; r < 16; ++r) x[r] = __fmaf_rn(-Lb[r * 17 + m], x[m], x[r]);
    }
    float* Ab = S.u.p.Ai[v][kkt_bidx(bb, bb)];
#pragma unroll
    for (int r = 0; r < 16; ++r) Ab[r * 17 + j] = x[r];
  }
  __syncthreads();

  // ---- 4. off-diagonal levels; warp (v = warp / 4, i = warp % 4) computes block (i, i - d) when i >= d
  const int v = warp >> 2, bi = warp & 3;
  for (int d = 1; d <= 3; ++d) {
    if (bi >= d) {
      const int bj = bi - d;
      float acc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
      for (int kk = bj; kk < bi; ++kk) mm16_acc(acc, S.L[v][kkt_bidx(bi, kk)], S.u.p.Ai[v][kkt_bidx(kk, bj)], lane);
      st16(S.u.p.scr[warp], acc, lane, 1.f);
      __syncwarp();
      float res[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
      mm16_acc(res, S.u.p.Ai[v][kkt_bidx(bi, bi)], S.u.p.scr[warp], lane);
      st16(S.u.p.Ai[v][kkt_bidx(bi, bj)], res, lane, -1.f);
    }
    __syncthreads();
  }

  // ---- 5. stores: 2 heads x 64 rows x 8 chunks of 8 columns
  for (int e = tid; e < 2 * 64 * 8; e += 256) {
    const int vv = e >> 9, r = (e >> 3) & 63, ch = e & 7;
    const int rb = r >> 4, cb = ch >> 1;
    if (r >= nval || cb > rb) continue;
    const float* Ab = S.u.p.Ai[vv][kkt_bidx(rb, cb)];
    const int lr = r & 15, lc = (ch & 1) * 8;
    uint32_t w4[4];
#pragma unroll
    for (int q2 = 0; q2 < 4; ++q2) w4[q2] = pack_bf16(Ab[lr * 17 + lc + 2 * q2], Ab[lr * 17 + lc + 2 * q2 + 1]);
    *reinterpret_cast<uint4*>(A + ((bos + t0 + r) * HV + kh * 2 + vv) * 64 + 8 * ch) = make_uint4(w4[0], w4[1], w4[2], w4[3]);
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
    if (reax_host::ensure_smem(attr, reax::kkt_kernel, (int)sizeof(reax::KktSmem)) != cudaSuccess)                   \
      return (int)cudaErrorInvalidValue;                                                                              \
    reax::kkt_kernel<<<dim3(NT, H), 256, sizeof(reax::KktSmem), (cudaStream_t)stream>>>(                              \
        (const uint16_t*)k, (const float*)g, (const uint16_t*)beta, (uint16_t*)A, (const long long*)cu,               \
        (const long long*)cidx, H, HV);                                                                               \
    return (int)cudaGetLastError();                                                                                   \
  }                                                                                                                   \
  REAX_API int reax_kkt_smem() { return (int)sizeof(reax::KktSmem); }
