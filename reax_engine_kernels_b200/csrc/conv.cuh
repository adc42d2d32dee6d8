// Depthwise causal conv (4 taps) + SiLU (+ per-128-channel L2 norm for the q/k units), sm_100a.
//
// Semantics (libreax_howu/reax_conv_v2.cu:60-150, :164-189): token t with meta (pos, y, z, w); tap j reads source
// position src = pos - 3 + j (tap skipped when src < 0) from qkv[(z + src) * SX + c] when src >= y, else from
// cache[(w + src) * C + c].  acc = fp32 fma chain over the taps in order 0..3; y = bf16(acc);
// s = bf16(y / (1 + exp(-y))).  Units of 128 channels: u < KD/128 -> q head u, u < 2KD/128 -> k head u - KD/128
// (both scaled by 1 / sqrt(eps + sum(s^2)) over the unit, written `rep` times side by side), else v (written when
// !skip_v).
//
// HBM-bound (each qkv element is read once from DRAM; the 4 taps of neighbouring tokens hit L1/L2).  A half-warp
// owns one (token, unit): lane l holds channels 8l..8l+7 (one 16-byte load per tap), the L2 norm is a 4-step
// half-warp butterfly, and every store is a coalesced 16-byte write.  A CTA of 256 threads covers 16 tokens x
// CONV_NR rows per half-warp for one unit; all tap loads of a thread are issued before any arithmetic.
#pragma once
#include "common.cuh"

namespace reax {

constexpr int CONV_NR = 4;

__device__ __forceinline__ float silu_f(float y) { return __fdiv_rn(y, __fadd_rn(1.0f, expf(-y))); }

template <int REP, bool SKIP_V>
__global__ void __launch_bounds__(256)
conv_kernel(const uint16_t* __restrict__ qkv, long long SX, const uint16_t* __restrict__ cache, int C,
            const int4* __restrict__ meta, const uint16_t* __restrict__ w, uint16_t* __restrict__ q,
            uint16_t* __restrict__ k, uint16_t* __restrict__ v, int Tf, float eps, int KD, int VD, int u0) {
  const int lane = threadIdx.x & 31, hw = threadIdx.x >> 4, l16 = lane & 15;
  const int u = u0 + blockIdx.x;  // units fastest: co-resident CTAs read adjacent pieces of the same qkv rows
  const int c0 = u * 128 + 8 * l16;
  const int nq = KD / 128, nqk = 2 * nq;
  if (u >= nqk && SKIP_V) return;
  const int tbeg = blockIdx.y * (16 * CONV_NR);
  int4 m[CONV_NR];
#pragma unroll
  for (int r = 0; r < CONV_NR; ++r) {
    const int t = tbeg + hw + 16 * r;
    m[r] = t < Tf ? __ldg(meta + t) : make_int4(-1000, 0, 0, 0);
  }
  float wt[8][4];
  {
    const uint4 a = __ldg(reinterpret_cast<const uint4*>(w + (long long)c0 * 4));
    const uint4 b = __ldg(reinterpret_cast<const uint4*>(w + (long long)c0 * 4 + 8));
    const uint4 c = __ldg(reinterpret_cast<const uint4*>(w + (long long)c0 * 4 + 16));
    const uint4 d = __ldg(reinterpret_cast<const uint4*>(w + (long long)c0 * 4 + 24));
    const uint32_t ww[16] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w, c.x, c.y, c.z, c.w, d.x, d.y, d.z, d.w};
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      wt[i][0] = bf_lo(ww[2 * i]);
      wt[i][1] = bf_hi(ww[2 * i]);
      wt[i][2] = bf_lo(ww[2 * i + 1]);
      wt[i][3] = bf_hi(ww[2 * i + 1]);
    }
  }
  uint4 xv[CONV_NR][4];
#pragma unroll
  for (int r = 0; r < CONV_NR; ++r)
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int src = m[r].x - 3 + j;
      xv[r][j] = make_uint4(0, 0, 0, 0);
      if (src >= 0) {
        const uint16_t* rp = src >= m[r].y ? qkv + (long long)(m[r].z + src) * SX : cache + (long long)(m[r].w + src) * C;
        xv[r][j] = __ldg(reinterpret_cast<const uint4*>(rp + c0));
      }
    }
#pragma unroll
  for (int r = 0; r < CONV_NR; ++r) {
    const int t = tbeg + hw + 16 * r;
    float acc[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if (m[r].x - 3 + j < 0) continue;
      const uint32_t xw[4] = {xv[r][j].x, xv[r][j].y, xv[r][j].z, xv[r][j].w};
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] = __fmaf_rn(wt[i][j], (i & 1) ? bf_hi(xw[i >> 1]) : bf_lo(xw[i >> 1]), acc[i]);
    }
    float s[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) s[i] = bf16_round(silu_f(bf16_round(acc[i])));
    if (u < nqk) {
      float sum = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) sum = __fmaf_rn(s[i], s[i], sum);
      sum += __shfl_xor_sync(0xffffffffu, sum, 8);
      sum += __shfl_xor_sync(0xffffffffu, sum, 4);
      sum += __shfl_xor_sync(0xffffffffu, sum, 2);
      sum += __shfl_xor_sync(0xffffffffu, sum, 1);
      const float rstd = 1.0f / sqrtf(__fadd_rn(eps, sum));
      if (t >= Tf) continue;
      const uint4 ov = make_uint4(pack_bf16(s[0] * rstd, s[1] * rstd), pack_bf16(s[2] * rstd, s[3] * rstd),
                                  pack_bf16(s[4] * rstd, s[5] * rstd), pack_bf16(s[6] * rstd, s[7] * rstd));
      const int nh = REP * KD / 128, hq = u % nq;
      uint16_t* dst = (u < nq ? q : k) + (long long)t * (nh * 128) + REP * hq * 128 + 8 * l16;
      __stcs(reinterpret_cast<uint4*>(dst), ov);
      if (REP == 2) __stcs(reinterpret_cast<uint4*>(dst + 128), ov);
    } else {
      if (t >= Tf) continue;
      const uint4 ov = make_uint4(pack_bf16(s[0], s[1]), pack_bf16(s[2], s[3]), pack_bf16(s[4], s[5]), pack_bf16(s[6], s[7]));
      __stcs(reinterpret_cast<uint4*>(v + (long long)t * VD + (c0 - 2 * KD)), ov);
    }
  }
}

}  // namespace reax

namespace reax_host {
inline int conv_launch(const void* qkv, long long SX, const void* cache, int C, const void* meta, const void* w, void* q,
                       void* k, void* v, int Tf, float eps, int KD, int VD, int rep, int skip_v, int u0, int nunits,
                       cudaStream_t st) {
  using namespace reax;
  if (KD % 128 || VD % 128 || KD < 0 || VD < 0 || (rep != 1 && rep != 2)) return -1;
  if (SX % 8 || C % 8 || (((uintptr_t)qkv | (uintptr_t)w | (uintptr_t)q | (uintptr_t)k | (uintptr_t)v) & 15)) return -1;
  if (nunits <= 0) return 0;
  const int tblocks = (Tf + 16 * CONV_NR - 1) / (16 * CONV_NR);
  if (tblocks > 65535) return -1;
  dim3 grid(nunits, tblocks);
  const uint16_t* a = (const uint16_t*)qkv;
  const uint16_t* cc = (const uint16_t*)cache;
  const int4* mt = (const int4*)meta;
  const uint16_t* ww = (const uint16_t*)w;
  uint16_t *qq = (uint16_t*)q, *kk = (uint16_t*)k, *vv = (uint16_t*)v;
  if (rep == 1 && !skip_v) conv_kernel<1, false><<<grid, 256, 0, st>>>(a, SX, cc, C, mt, ww, qq, kk, vv, Tf, eps, KD, VD, u0);
  else if (rep == 1) conv_kernel<1, true><<<grid, 256, 0, st>>>(a, SX, cc, C, mt, ww, qq, kk, vv, Tf, eps, KD, VD, u0);
  else if (!skip_v) conv_kernel<2, false><<<grid, 256, 0, st>>>(a, SX, cc, C, mt, ww, qq, kk, vv, Tf, eps, KD, VD, u0);
  else conv_kernel<2, true><<<grid, 256, 0, st>>>(a, SX, cc, C, mt, ww, qq, kk, vv, Tf, eps, KD, VD, u0);
  return (int)cudaGetLastError();
}
}  // namespace reax_host

// libreax_howu/reax_conv_v2.cu:164-189 argument lists and codes (RT selects the reference's rows-per-CTA variant;
// it is validated the same way, the tiling here is independent of it)
#define REAX_DEFINE_CONV_EXPORTS()                                                                                    \
  REAX_API int reax_conv_l2(const void* qkv, long long SX, const void* cache, int C, const void* meta, const void* w,  \
                            void* q, void* k, void* v, int Tf, float eps, int KD, int VD, int rep, int skip_v, int RT, \
                            void* stream) {                                                                            \
    if (Tf <= 0) return 0;                                                                                             \
    if (RT != 8 && RT != 16 && RT != 32) return -1;                                                                    \
    const int units = 2 * KD / 128 + (skip_v ? 0 : VD / 128);                                                          \
    return reax_host::conv_launch(qkv, SX, cache, C, meta, w, q, k, v, Tf, eps, KD, VD, rep, skip_v, 0, units,         \
                                  (cudaStream_t)stream);                                                               \
  }                                                                                                                    \
  REAX_API int reax_conv_v(const void* qkv, long long SX, const void* cache, int C, const void* meta, const void* w,   \
                           void* v, int Tf, int KD, int VD, void* stream) {                                           \
    if (Tf <= 0) return 0;                                                                                             \
    return reax_host::conv_launch(qkv, SX, cache, C, meta, w, nullptr, nullptr, v, Tf, 1e-6f, KD, VD, 1, 0,            \
                                  2 * KD / 128, VD / 128, (cudaStream_t)stream);                                       \
  }
