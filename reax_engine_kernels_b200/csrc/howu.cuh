// Chunked gated delta rule (WY form, 64-token chunks) with optional fused gated RMSNorm, sm_100a.
//
// Semantics (libreax_howu/reax_howu.cu:124-347, libreax_howu/reax_howu_norm_v3.cu:347-374), per (sequence, value
// head hv, key head kh = hv / (HV/H)), chunk of nval <= 64 tokens, state h[128 k][128 v] (fp32):
//   vb = bf16(beta v);  kb = bf16(bf16(beta k) 2^g);  u = A vb;  w = bf16(A kb)     (A: lower 16x16 blocks, or all)
//   Aq[t][s] = bf16((q_t . k_s) 2^(g_t - g_s)) for s <= t (valid), else 0
//   Hb = bf16(h);  x = bf16(u) - w Hb;  vn = bf16(x);  vdec = bf16(x 2^(g_last - g_t))
//   o = bf16(scale (Aq vn) + scale 2^(g_t) (q Hb));   h <- h 2^(g_last) + k^T vdec
//   norm: out[f2s[t]][hv] = bf16( bf16(nw * bf16(o * rsqrt(sum(o^2) factor + eps))) * silu(z) ), f2s < 0 skipped.
//
// One CTA (8 warps) per (sequence, value head, column slice), serial over the chunks of that sequence; the value
// columns of the state are split in two slices (CW = 64) while the doubled grid still fits on the GPU at once.  The
// chunk inputs arrive by cp.async, each tile copied for the next chunk as soon as the current one stops reading it.  The chunk matmuls are
// 64-row tiles on bf16 mma.sync from padded shared-memory tiles (conflict-free ldmatrix); the state h lives in
// registers (warp w owns k rows 16w..16w+15) for the whole sequence and is re-published as bf16 each chunk.
#pragma once
#include "common.cuh"

namespace reax {

constexpr int HW_LD = 136;  // row stride (elements) of 128-wide tiles
constexpr int HA_LD = 72;   // row stride of 64-wide tiles

struct HowuSmem {
  uint16_t A[64 * HA_LD];
  uint16_t AQ[64 * HA_LD];
  uint16_t V[64 * HW_LD];   // v -> vb
  uint16_t K[64 * HW_LD];
  uint16_t KB[64 * HW_LD];
  uint16_t Q[64 * HW_LD];
  uint16_t W[64 * HW_LD];
  uint16_t VN[64 * HW_LD];
  uint16_t VD[64 * HW_LD];
  uint16_t O[64 * HW_LD];
  uint16_t H[128 * HW_LD];
  float g[64], eg[64], beta[64], da[64];
  int f2s[64];
};

__device__ __forceinline__ void ldsm4(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(addr) : "memory");
}
__device__ __forceinline__ void ldsm4t(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(addr) : "memory");
}
__device__ __forceinline__ void hmma(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
               : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
               : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t sh_addr(const uint16_t* base, int row, int col, int ld) {
  return smem_u32(base) + (uint32_t)((row * ld + col) * 2);
}
// acc[NT] (16 rows x 8NT cols) += A[r0.., k0..k0+15] * B[k0..k0+15][n0..n0+8NT), A row-major, B row-major [K][N]
template <int NT>
__device__ __forceinline__ void mma_kstep_rb(float (&acc)[NT][4], const uint16_t* A, int lda, int r0, int k0,
                                             const uint16_t* B, int ldb, int n0, int lane) {
  uint32_t a[4];
  ldsm4(a, sh_addr(A, r0 + (lane & 15), k0 + 8 * (lane >> 4), lda));
#pragma unroll
  for (int p = 0; p < NT / 2; ++p) {
    uint32_t b[4];
    ldsm4t(b, sh_addr(B, k0 + (lane & 15), n0 + 16 * p + 8 * (lane >> 4), ldb));
    hmma(acc[2 * p], a, b[0], b[1]);
    hmma(acc[2 * p + 1], a, b[2], b[3]);
  }
}
template <int NT>
__device__ __forceinline__ void zero_acc(float (&acc)[NT][4]) {
#pragma unroll
  for (int i = 0; i < NT; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
}
__device__ __forceinline__ float silu_exact(float z) { return __fdiv_rn(z, __fadd_rn(1.f, expf(-z))); }

template <bool SKIPA, bool NORM, int CW>
__global__ void __launch_bounds__(256, 1)
howu_kernel(const uint16_t* __restrict__ q, const uint16_t* __restrict__ k, const uint16_t* __restrict__ v,
            const uint16_t* __restrict__ beta, const uint16_t* __restrict__ Ag, const float* __restrict__ g,
            uint16_t* __restrict__ o, const long long* __restrict__ cu, float scale, int NSEQ, int H, int HV,
            const int* __restrict__ f2s, const uint16_t* __restrict__ zg, long long ZS, const uint16_t* __restrict__ nw,
            float eps, float factor) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  HowuSmem& S = *reinterpret_cast<HowuSmem*>(smem_raw);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int gq = lane >> 2, tq = lane & 3;
  // longest sequences first is not needed: one CTA per (seq, head); dispatch the last sequence first like the
  // reference so equal-length batches fill the GPU in the same order
  // CW value columns per CTA: the state recurrence is independent per value column, so a (sequence, head) is split
  // into 128 / CW column slices (w = A kb and Aq, which every column needs, are computed by each slice)
  static_assert(CW == 128 || (CW == 64 && !NORM), "the fused norm needs whole rows");
  constexpr int NSL = 128 / CW, NTO = CW / 16;
  const int sl = (int)(blockIdx.x % NSL), bx = (int)(blockIdx.x / NSL), c_lo = sl * CW;
  const int n = NSEQ - 1 - bx / HV, hv = bx % HV, kh = hv / (HV / H);
  const long long bos = cu[n], T = cu[n + 1] - bos;
  // 64 x CW outputs: rows 16rb.., local columns cs.. (CW / 2 wide); w: cols 64ch..; Aq: cols 32ch..
  const int rb = warp & 3, ch = warp >> 2, cs = (CW / 2) * ch;

  float h[CW / 8][4];  // state rows 16*warp + {gq, gq+8}, local cols 8j + 2tq + {0,1}
  zero_acc(h);
  for (int i = tid; i < 128 * HW_LD / 8; i += 256) reinterpret_cast<uint4*>(S.H)[i] = make_uint4(0, 0, 0, 0);

  // Chunk inputs arrive by cp.async (no registers held while in flight), each tile copied for the next chunk as soon
  // as this chunk no longer reads it: v and A after u/w, raw k (into the tile that held kb, so the raw-k and kb tiles
  // trade roles every chunk) after u/w, q after q Hb; the 64 decay / beta scalars ride along in registers.
  auto copy_va_k = [&](long long tc, uint16_t* kdst) {
    const int nv = (int)min(64LL, T - tc), c = tid & 15;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int r = (tid >> 4) + 16 * e;
      const bool ok = r < nv;
      const long long tok = bos + tc + r;
      if (c < CW / 8)
        cp_async16(smem_u32(&S.V[r * HW_LD + 8 * c]), ok ? v + (tok * HV + hv) * 128 + c_lo + 8 * c : v, ok);
      if (c < 8) cp_async16(smem_u32(&S.A[r * HA_LD + 8 * c]), ok ? Ag + (tok * HV + hv) * 64 + 8 * c : Ag, ok);
      cp_async16(smem_u32(&kdst[r * HW_LD + 8 * c]), ok ? k + (tok * H + kh) * 128 + 8 * c : k, ok);
    }
    cp_async_commit();
  };
  auto copy_q = [&](long long tc) {
    const int nv = (int)min(64LL, T - tc), c = tid & 15;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int r = (tid >> 4) + 16 * e;
      const bool ok = r < nv;
      const long long tok = bos + tc + r;
      cp_async16(smem_u32(&S.Q[r * HW_LD + 8 * c]), ok ? q + (tok * H + kh) * 128 + 8 * c : q, ok);
    }
    cp_async_commit();
  };
  float sg = 0.f, sb = 0.f;  // scalars of the chunk in flight (threads < 64: its row tid)
  int sf = -1;
  auto load_scalars = [&](long long tc) {
    if (tid < 64) {
      const bool ok = tid < min(64LL, T - tc);
      const long long tok = bos + tc + tid;
      sg = ok ? g[tok * HV + hv] : 0.f;
      sb = ok ? __uint_as_float((uint32_t)beta[tok * HV + hv] << 16) : 0.f;
      if (NORM) sf = ok ? f2s[tok] : -1;
    }
  };
  if (T > 0) {
    copy_va_k(0, S.K);
    copy_q(0);
    load_scalars(0);
  }

  for (long long t0 = 0; t0 < T; t0 += 64) {
    const int nval = (int)min(64LL, T - t0);
    const bool first = t0 == 0;
    const bool odd = ((t0 >> 6) & 1) != 0;
    uint16_t* const KR = odd ? S.KB : S.K;  // raw k of this chunk
    uint16_t* const KS = odd ? S.K : S.KB;  // kb of this chunk
    cp_async_wait<0>();
    if (tid < 64) {
      S.g[tid] = sg;
      S.eg[tid] = exp2f(sg);
      S.beta[tid] = sb;
      if (NORM) S.f2s[tid] = sf;
    }
    __syncthreads();  // the chunk's tiles and scalars are visible to every thread
    const float glast = S.g[nval - 1];
    if (tid < 64) S.da[tid] = tid < nval ? exp2f(glast - S.g[tid]) : 0.f;  // read two barriers later
    // ---- vb = bf16(beta v) in place, kb = bf16(bf16(beta k) 2^g)
    {
      const int c = tid & 15;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int r = (tid >> 4) + 16 * e;
        const float b = S.beta[r], eg = S.eg[r];
        uint4 x = *reinterpret_cast<const uint4*>(&S.V[r * HW_LD + 8 * c]);
        uint4 y = *reinterpret_cast<const uint4*>(&KR[r * HW_LD + 8 * c]);
        uint32_t* xp = reinterpret_cast<uint32_t*>(&x);
        uint32_t* yp = reinterpret_cast<uint32_t*>(&y);
#pragma unroll
        for (int e2 = 0; e2 < 4; ++e2) {
          xp[e2] = pack_bf16(bf_lo(xp[e2]) * b, bf_hi(xp[e2]) * b);
          const uint32_t t = pack_bf16(bf_lo(yp[e2]) * b, bf_hi(yp[e2]) * b);
          yp[e2] = pack_bf16(bf_lo(t) * eg, bf_hi(t) * eg);
        }
        if (c < CW / 8) *reinterpret_cast<uint4*>(&S.V[r * HW_LD + 8 * c]) = x;
        *reinterpret_cast<uint4*>(&KS[r * HW_LD + 8 * c]) = y;
      }
    }
    __syncthreads();

    // ---- u = A vb, w = A kb (rows 16rb.., cols 64ch..); Aq = q k^T (rows 16rb.., cols 32ch..)
    float u[NTO][4], wacc[8][4];
    zero_acc(u);
    zero_acc(wacc);
#pragma unroll
    for (int kb = 0; kb < 4; ++kb) {
      if (SKIPA && kb > rb) continue;
      mma_kstep_rb<NTO>(u, S.A, HA_LD, 16 * rb, 16 * kb, S.V, HW_LD, cs, lane);
      mma_kstep_rb<8>(wacc, S.A, HA_LD, 16 * rb, 16 * kb, KS, HW_LD, 64 * ch, lane);
    }
    {
      float c[4][4];
      zero_acc(c);
      if (32 * ch <= 16 * rb + 15) {  // tiles entirely above the diagonal are masked anyway
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          uint32_t a[4];
          ldsm4(a, sh_addr(S.Q, 16 * rb + (lane & 15), 16 * kk + 8 * (lane >> 4), HW_LD));
#pragma unroll
          for (int p = 0; p < 2; ++p) {
            uint32_t b[4];
            ldsm4(b, sh_addr(KR, 32 * ch + 16 * p + (lane & 7) + 8 * (lane >> 4), 16 * kk + 8 * ((lane >> 3) & 1), HW_LD));
            hmma(c[2 * p], a, b[0], b[1]);
            hmma(c[2 * p + 1], a, b[2], b[3]);
          }
        }
      }
#pragma unroll
      for (int nt = 0; nt < 4; ++nt) {
        const int s0 = 32 * ch + 8 * nt + 2 * tq;
#pragma unroll
        for (int hr = 0; hr < 2; ++hr) {
          const int t = 16 * rb + gq + 8 * hr;
          float y[2];
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int s = s0 + e;
            y[e] = (s <= t && t < nval && s < nval) ? c[nt][2 * hr + e] * exp2f(S.g[t] - S.g[s]) : 0.f;
          }
          *reinterpret_cast<uint32_t*>(&S.AQ[t * HA_LD + s0]) = pack_bf16(y[0], y[1]);
        }
      }
    }
    uint32_t ub[NTO][2];
#pragma unroll
    for (int nt = 0; nt < NTO; ++nt) {
      ub[nt][0] = pack_bf16(u[nt][0], u[nt][1]);
      ub[nt][1] = pack_bf16(u[nt][2], u[nt][3]);
    }
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      const int col = 64 * ch + 8 * nt + 2 * tq;
      *reinterpret_cast<uint32_t*>(&S.W[(16 * rb + gq) * HW_LD + col]) = pack_bf16(wacc[nt][0], wacc[nt][1]);
      *reinterpret_cast<uint32_t*>(&S.W[(16 * rb + gq + 8) * HW_LD + col]) = pack_bf16(wacc[nt][2], wacc[nt][3]);
    }
    __syncthreads();
    if (t0 + 64 < T) copy_va_k(t0 + 64, KS);  // vb, A and kb of this chunk are read no more

    // ---- vw = w Hb, oi = q Hb; x = bf16(u) - vw -> vn, vdec
    float oi[NTO][4];
    {
      float vw[NTO][4];
      zero_acc(vw);
      zero_acc(oi);
      if (!first) {
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          mma_kstep_rb<NTO>(vw, S.W, HW_LD, 16 * rb, 16 * kk, S.H, HW_LD, cs, lane);
          mma_kstep_rb<NTO>(oi, S.Q, HW_LD, 16 * rb, 16 * kk, S.H, HW_LD, cs, lane);
        }
      }
      const int ta = 16 * rb + gq, tb = ta + 8;
      const float da = S.da[ta], db = S.da[tb];
#pragma unroll
      for (int nt = 0; nt < NTO; ++nt) {
        const int col = cs + 8 * nt + 2 * tq;
        const float x0 = bf_lo(ub[nt][0]) - vw[nt][0], x1 = bf_hi(ub[nt][0]) - vw[nt][1];
        const float x2 = bf_lo(ub[nt][1]) - vw[nt][2], x3 = bf_hi(ub[nt][1]) - vw[nt][3];
        *reinterpret_cast<uint32_t*>(&S.VN[ta * HW_LD + col]) = pack_bf16(x0, x1);
        *reinterpret_cast<uint32_t*>(&S.VN[tb * HW_LD + col]) = pack_bf16(x2, x3);
        *reinterpret_cast<uint32_t*>(&S.VD[ta * HW_LD + col]) = pack_bf16(x0 * da, x1 * da);
        *reinterpret_cast<uint32_t*>(&S.VD[tb * HW_LD + col]) = pack_bf16(x2 * db, x3 * db);
      }
    }
    __syncthreads();
    if (t0 + 64 < T) {  // q of this chunk is read no more
      copy_q(t0 + 64);
      load_scalars(t0 + 64);
    }

    // ---- o = bf16(scale (Aq vn) + scale 2^g (q Hb)) -> staging; h = h 2^glast + k^T vdec
    {
      float ci[NTO][4];
      zero_acc(ci);
#pragma unroll
      for (int kb = 0; kb < 4; ++kb) {
        if (kb > rb) continue;
        mma_kstep_rb<NTO>(ci, S.AQ, HA_LD, 16 * rb, 16 * kb, S.VN, HW_LD, cs, lane);
      }
      const int ta = 16 * rb + gq, tb = ta + 8;
      const float ea = S.eg[ta], eb = S.eg[tb];
#pragma unroll
      for (int nt = 0; nt < NTO; ++nt) {
        const int col = cs + 8 * nt + 2 * tq;
        float r[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) r[e] = __fmaf_rn(ci[nt][e], scale, (oi[nt][e] * (e < 2 ? ea : eb)) * scale);
        *reinterpret_cast<uint32_t*>(&S.O[ta * HW_LD + col]) = pack_bf16(r[0], r[1]);
        *reinterpret_cast<uint32_t*>(&S.O[tb * HW_LD + col]) = pack_bf16(r[2], r[3]);
      }
    }
    {
      const float gl = exp2f(glast);
#pragma unroll
      for (int j = 0; j < CW / 8; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) h[j][e] *= gl;
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        uint32_t a[4];
        // A = k^T (rows = key dims 16*warp.., cols = tokens 16kk..), loaded transposed from k [t][d]
        ldsm4t(a, sh_addr(KR, 16 * kk + (lane & 7) + 8 * (lane >> 4), 16 * warp + 8 * ((lane >> 3) & 1), HW_LD));
#pragma unroll
        for (int p = 0; p < CW / 16; ++p) {
          uint32_t b[4];
          ldsm4t(b, sh_addr(S.VD, 16 * kk + (lane & 15), 16 * p + 8 * (lane >> 4), HW_LD));
          hmma(h[2 * p], a, b[0], b[1]);
          hmma(h[2 * p + 1], a, b[2], b[3]);
        }
      }
    }
    __syncthreads();

    // ---- outputs of this chunk, and Hb = bf16(h) for the next one
    if (!NORM) {
      for (int i = tid; i < 64 * (CW / 8); i += 256) {
        const int r = i / (CW / 8), c = i % (CW / 8);
        if (r < nval)
          *reinterpret_cast<uint4*>(o + ((bos + t0 + r) * HV + hv) * 128 + c_lo + 8 * c) =
              *reinterpret_cast<const uint4*>(&S.O[r * HW_LD + 8 * c]);
      }
    } else {
      const uint2 wv = __ldg(reinterpret_cast<const uint2*>(nw + 4 * lane));
      const float wn[4] = {bf_lo(wv.x), bf_hi(wv.x), bf_lo(wv.y), bf_hi(wv.y)};
      for (int r = warp; r < nval; r += 8) {
        const int sr = S.f2s[r];
        if (sr < 0) continue;  // warp-uniform
        const uint2 xv = *reinterpret_cast<const uint2*>(&S.O[r * HW_LD + 4 * lane]);
        const float x[4] = {bf_lo(xv.x), bf_hi(xv.x), bf_lo(xv.y), bf_hi(xv.y)};
        float ss = x[0] * x[0] + x[1] * x[1] + x[2] * x[2] + x[3] * x[3];
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
        const float rr = rsqrtf(__fadd_rn(__fmul_rn(ss, factor), eps));
        const uint2 zv = __ldg(reinterpret_cast<const uint2*>(zg + (long long)sr * ZS + (long long)hv * 128 + 4 * lane));
        const float z[4] = {bf_lo(zv.x), bf_hi(zv.x), bf_lo(zv.y), bf_hi(zv.y)};
        float res[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float y = bf16_round(x[e] * rr);
          const float y2 = bf16_round(wn[e] * y);
          res[e] = y2 * silu_exact(z[e]);
        }
        *reinterpret_cast<uint2*>(o + ((long long)sr * HV + hv) * 128 + 4 * lane) =
            make_uint2(pack_bf16(res[0], res[1]), pack_bf16(res[2], res[3]));
      }
    }
#pragma unroll
    for (int j = 0; j < CW / 8; ++j) {
      const int col = 8 * j + 2 * tq;
      *reinterpret_cast<uint32_t*>(&S.H[(16 * warp + gq) * HW_LD + col]) = pack_bf16(h[j][0], h[j][1]);
      *reinterpret_cast<uint32_t*>(&S.H[(16 * warp + gq + 8) * HW_LD + col]) = pack_bf16(h[j][2], h[j][3]);
    }
    __syncthreads();
  }
}

}  // namespace reax

namespace reax_host {
template <bool SKIPA, bool NORM, int CW>
inline int howu_launch_cw(const void* q, const void* k, const void* v, const void* beta, const void* A, const void* g,
                          void* o, const void* cu, float scale, int N, int H, int HV, void* stream, const void* f2s,
                          const void* z, long long ZS, const void* nw, float eps, float factor) {
  static SmemAttr attr;
  if (ensure_smem(attr, reax::howu_kernel<SKIPA, NORM, CW>, (int)sizeof(reax::HowuSmem)) != cudaSuccess)
    return (int)cudaErrorInvalidValue;
  reax::howu_kernel<SKIPA, NORM, CW><<<N * HV * (128 / CW), 256, sizeof(reax::HowuSmem), (cudaStream_t)stream>>>(
      (const uint16_t*)q, (const uint16_t*)k, (const uint16_t*)v, (const uint16_t*)beta, (const uint16_t*)A, (const float*)g,
      (uint16_t*)o, (const long long*)cu, scale, N, H, HV, (const int*)f2s, (const uint16_t*)z, ZS, (const uint16_t*)nw, eps,
      factor);
  return (int)cudaGetLastError();
}

template <bool SKIPA, bool NORM>
inline int howu_launch(const void* q, const void* k, const void* v, const void* beta, const void* A, const void* g, void* o,
                       const void* cu, float scale, int N, int H, int HV, void* stream, const void* f2s = nullptr,
                       const void* z = nullptr, long long ZS = 0, const void* nw = nullptr, float eps = 0.f,
                       float factor = 0.f) {
  if (N <= 0 || HV <= 0) return 0;
  if (H <= 0 || HV % H) return -1;
  if ((((uintptr_t)q | (uintptr_t)k | (uintptr_t)v | (uintptr_t)A | (uintptr_t)o) & 15)) return -1;
  // one CTA per SM: split the value columns in two while the doubled grid still fits on the GPU at once
  int dev = 0;
  cudaGetDevice(&dev);
  if (!NORM && 2LL * N * HV <= device_sms(dev))
    return howu_launch_cw<SKIPA, false, 64>(q, k, v, beta, A, g, o, cu, scale, N, H, HV, stream, f2s, z, ZS, nw, eps,
                                            factor);
  return howu_launch_cw<SKIPA, NORM, 128>(q, k, v, beta, A, g, o, cu, scale, N, H, HV, stream, f2s, z, ZS, nw, eps,
                                          factor);
}
}  // namespace reax_host

// libreax_howu/reax_howu.cu:363-376 and libreax_howu/reax_howu_norm_v3.cu:431-435 argument lists
#define REAX_DEFINE_HOWU_EXPORTS()                                                                                     \
  REAX_API int howu3_dense(const void* q, const void* k, const void* v, const void* beta, const void* A, const void* g,  \
                           void* o, const void* cu, float scale, int N, int H, int HV, void* stream) {                   \
    return reax_host::howu_tc_launch<false, false>(q, k, v, beta, A, g, o, cu, scale, N, H, HV, stream);                 \
  }                                                                                                                      \
  REAX_API int howu3_skip(const void* q, const void* k, const void* v, const void* beta, const void* A, const void* g,   \
                          void* o, const void* cu, float scale, int N, int H, int HV, void* stream) {                    \
    return reax_host::howu_tc_launch<true, false>(q, k, v, beta, A, g, o, cu, scale, N, H, HV, stream);                  \
  }                                                                                                                      \
  REAX_API int howu3_smem() { return reax::kHowuTcSmemBytes; }                                                           \
  REAX_API int reax_howu(const void* q, const void* k, const void* v, const void* beta, const void* A, const void* g,    \
                         void* o, const void* cu, float scale, int N, int H, int HV, void* stream) {                     \
    return reax_host::howu_tc_launch<true, false>(q, k, v, beta, A, g, o, cu, scale, N, H, HV, stream);                  \
  }                                                                                                                      \
  REAX_API int reax_howu_norm(const void* q, const void* k, const void* v, const void* beta, const void* A,             \
                              const void* g, void* out, const void* cu, float scale, int N, int H, int HV, void* stream, \
                              const void* f2s, const void* z, long long ZS, const void* nw, float eps, float factor) {   \
    return reax_host::howu_norm_tc_launch(q, k, v, beta, A, g, out, cu, scale, N, H, HV, stream, f2s, z, ZS, nw, eps,    \
                                          factor);                                                                       \
  }
