// Reduce S bf16 partials + residual + RMSNorm with (1 + w), sm_100a.
//
// Semantics (libreax_howu/reax_rarn_final.cu:36-89):
//   d = bf16(sum_s part[s])            (serial: bf16 after the first term and after every add)
//   h = bf16(res + d) -> h_out;  out = bf16( (h * rsqrt(sum(h^2) * factor + eps)) * (1 + w) )
//
// HBM-bound: per row (S + 1) * D * 2 bytes read and 2 * D * 2 written.  One CTA of 256 threads per row; each thread
// owns up to RARN_MAXC 16-byte chunks of 8 columns (128-bit coalesced loads of every partial and of the residual),
// keeps h in registers, and the row's sum of squares is reduced with warp shuffles + one shared-memory step.
// Any D that is a multiple of 128 up to 256 * 8 * RARN_MAXC works (the reference accepted D = 2560 only).
#pragma once
#include "common.cuh"

namespace reax {

constexpr int RARN_THREADS = 256;
constexpr int RARN_MAXC = 4;  // D <= 8192

template <int S, bool SERIAL>
__global__ void __launch_bounds__(RARN_THREADS)
rarn_kernel(const uint16_t* __restrict__ part, long long pstride, const uint16_t* __restrict__ res,
            const uint16_t* __restrict__ w, uint16_t* __restrict__ h_out, uint16_t* __restrict__ out, int D, float eps,
            float factor) {
  __shared__ float red[RARN_THREADS / 32];
  const long long row = blockIdx.x;
  const int tid = threadIdx.x;
  const int nchunk = D >> 3;
  uint4 hv[RARN_MAXC];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < RARN_MAXC; ++i) {
    const int c = tid + i * RARN_THREADS;
    if (c >= nchunk) break;
    const long long off = row * D + 8LL * c;
    uint4 pv[S];
#pragma unroll
    for (int s = 0; s < S; ++s) pv[s] = __ldcs(reinterpret_cast<const uint4*>(part + s * pstride + off));
    const uint4 rv = __ldcs(reinterpret_cast<const uint4*>(res + off));
    const uint32_t rw[4] = {rv.x, rv.y, rv.z, rv.w};
    uint32_t ho[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      float hh[2];
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        auto get = [&](const uint4& u) {
          const uint32_t x = e == 0 ? u.x : e == 1 ? u.y : e == 2 ? u.z : u.w;
          return half ? bf_hi(x) : bf_lo(x);
        };
        float d = get(pv[0]);
#pragma unroll
        for (int s = 1; s < S; ++s) {
          d = __fadd_rn(d, get(pv[s]));
          if (SERIAL) d = bf16_round(d);
        }
        d = bf16_round(d);
        const float r = half ? bf_hi(rw[e]) : bf_lo(rw[e]);
        hh[half] = bf16_round(__fadd_rn(r, d));
        ss = __fmaf_rn(hh[half], hh[half], ss);
      }
      ho[e] = pack_bf16(hh[0], hh[1]);
    }
    hv[i] = make_uint4(ho[0], ho[1], ho[2], ho[3]);
    __stcs(reinterpret_cast<uint4*>(h_out + off), hv[i]);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((tid & 31) == 0) red[tid >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int i = 0; i < RARN_THREADS / 32; ++i) tot += red[i];
  const float r = rsqrtf(__fadd_rn(__fmul_rn(tot, factor), eps));
#pragma unroll
  for (int i = 0; i < RARN_MAXC; ++i) {
    const int c = tid + i * RARN_THREADS;
    if (c >= nchunk) break;
    const uint4 wv = __ldg(reinterpret_cast<const uint4*>(w + 8 * c));
    const uint32_t ww[4] = {wv.x, wv.y, wv.z, wv.w};
    const uint32_t hw[4] = {hv[i].x, hv[i].y, hv[i].z, hv[i].w};
    uint32_t o4[4];
#pragma unroll
    for (int e = 0; e < 4; ++e)
      o4[e] = pack_bf16(__fmul_rn(__fmul_rn(bf_lo(hw[e]), r), __fadd_rn(1.f, bf_lo(ww[e]))),
                        __fmul_rn(__fmul_rn(bf_hi(hw[e]), r), __fadd_rn(1.f, bf_hi(ww[e]))));
    __stcs(reinterpret_cast<uint4*>(out + row * D + 8LL * c), make_uint4(o4[0], o4[1], o4[2], o4[3]));
  }
}

}  // namespace reax

namespace reax_host {
template <int S, bool SER>
inline int rarn_go(const void* part, long long ps, const void* res, const void* w, void* h, void* o, int n, int D, float eps,
                   float f, cudaStream_t st) {
  reax::rarn_kernel<S, SER><<<n, reax::RARN_THREADS, 0, st>>>((const uint16_t*)part, ps, (const uint16_t*)res,
                                                               (const uint16_t*)w, (uint16_t*)h, (uint16_t*)o, D, eps, f);
  return (int)cudaGetLastError();
}
}  // namespace reax_host

// libreax_howu/reax_rarn_final.cu:98-106 argument list and codes (D now any positive multiple of 128 up to 8192;
// pointers and pstride must keep 16-byte alignment of every row, as the reference's vector loads also required)
#define REAX_DEFINE_RARN_EXPORT()                                                                                    \
  REAX_API int reax_rarn(const void* part, int S, int serial, long long pstride, const void* res, const void* w,      \
                         void* h_out, void* out, int n, int D, float eps, float factor, void* stream) {               \
    if (n <= 0) return 0;                                                                                              \
    if (D <= 0 || D % 128 || D > 256 * 8 * reax::RARN_MAXC) return -1;                                                 \
    if (pstride % 8 || (((uintptr_t)part | (uintptr_t)res | (uintptr_t)w | (uintptr_t)h_out | (uintptr_t)out) & 15)) \
      return -1;                                                                                                       \
    cudaStream_t st = (cudaStream_t)stream;                                                                            \
    switch (S) {                                                                                                       \
      case 2: return serial ? reax_host::rarn_go<2, true>(part, pstride, res, w, h_out, out, n, D, eps, factor, st)   \
                            : reax_host::rarn_go<2, false>(part, pstride, res, w, h_out, out, n, D, eps, factor, st); \
      case 3: return serial ? reax_host::rarn_go<3, true>(part, pstride, res, w, h_out, out, n, D, eps, factor, st)   \
                            : reax_host::rarn_go<3, false>(part, pstride, res, w, h_out, out, n, D, eps, factor, st); \
      case 4: return serial ? reax_host::rarn_go<4, true>(part, pstride, res, w, h_out, out, n, D, eps, factor, st)   \
                            : reax_host::rarn_go<4, false>(part, pstride, res, w, h_out, out, n, D, eps, factor, st); \
      case 5: return serial ? reax_host::rarn_go<5, true>(part, pstride, res, w, h_out, out, n, D, eps, factor, st)   \
                            : reax_host::rarn_go<5, false>(part, pstride, res, w, h_out, out, n, D, eps, factor, st); \
      case 6: return serial ? reax_host::rarn_go<6, true>(part, pstride, res, w, h_out, out, n, D, eps, factor, st)   \
                            : reax_host::rarn_go<6, false>(part, pstride, res, w, h_out, out, n, D, eps, factor, st); \
      case 7: return serial ? reax_host::rarn_go<7, true>(part, pstride, res, w, h_out, out, n, D, eps, factor, st)   \
                            : reax_host::rarn_go<7, false>(part, pstride, res, w, h_out, out, n, D, eps, factor, st); \
      case 8: return serial ? reax_host::rarn_go<8, true>(part, pstride, res, w, h_out, out, n, D, eps, factor, st)   \
                            : reax_host::rarn_go<8, false>(part, pstride, res, w, h_out, out, n, D, eps, factor, st); \
      default: return -2;                                                                                              \
    }                                                                                                                  \
  }
