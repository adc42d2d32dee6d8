// Depthwise causal conv (4 taps) + SiLU (+ per-128-channel L2 norm for the q/k units), sm_100a.
//
// Semantics (libreax_howu/reax_conv_v2.cu:60-150, :164-189): token t with meta (pos, y, z, w); tap j reads source
// position src = pos - 3 + j (tap skipped when src < 0) from qkv[(z + src) * SX + c] when src >= y, else from
// cache[(w + src) * C + c].  acc = fp32 fma chain over the taps in order 0..3; y = bf16(acc);
// s = bf16(y / (1 + exp(-y))).  Units of 128 channels: u < KD/128 -> q head u, u < 2KD/128 -> k head u - KD/128
// (both scaled by 1 / sqrt(eps + sum(s^2)) over the unit, written `rep` times side by side), else v (written when
// !skip_v).
//
// HBM-bound when lean enough: every qkv element is read once from DRAM and every output written once, ~4 bytes per
// element, so at ~8 TB/s the budget is about 20 issued instructions per element.  A CTA (256 threads) owns a block of
// 64 tokens and a run of up to CONV_UPC 128-channel units:
//   * shared-memory stages, filled with cp.async (no registers held while a copy is in flight; the next unit's rows
//     are in flight while this unit is computed): slot 3 + r holds token tbeg+r's own row (its tap 3, qkv[z + pos]),
//     slots 0..2 the sources of token tbeg's taps at distance 3..1 (qkv or cache).  Token row r reads its tap at
//     distance d from slot 3 + r - d whenever that slot holds exactly that source (same sequence, contiguous
//     positions); other sources (a sequence that starts inside the block with positions in the cache) are read from
//     global memory on a general path;
//   * the weights of the CTA's units converted to fp32 once, in shared memory;
//   * a warp owns 8 consecutive tokens and a lane 4 channels of them: the 11 source rows the warp needs are read
//     (8 bytes per lane) and unpacked once and shared by the 8 tokens; taps, gate and norm run on packed fp32 pairs
//     (fma/mul/add.rn.f32x2).  Accumulators (8 tokens x 2 pairs) and weights (4 taps x 2 pairs) fit the 64-register
//     budget of 4 CTAs per SM without spilling in the loop (8 channels x 4 tokens per thread did not);
//   * gate: s = y * rcp(1 + 2^(-y log2 e)) with MUFU ex2/rcp (relative error ~2^-20 before the bf16 rounding of s);
//     a thread holding any y <= -87 (where 2^(-y log2 e) overflows) recomputes with expf and IEEE division;
//   * norm: 1 / sqrt(eps + sum) as rsqrtf; the 8 per-token sums of a lane are reduce-scattered over the warp (lane
//     bits 4, 3, 2 pick the token a lane keeps, then a butterfly over bits 1, 0), and each lane fetches the 8 factors.
#pragma once
#include "common.cuh"

namespace reax {

constexpr int CONV_TB = 64;   // tokens per CTA
constexpr int CONV_TPT = 8;   // consecutive tokens per warp (one lane per 4 channels)
constexpr int CONV_UPC = 6;   // 128-channel units per CTA: the per-CTA set-up (meta, weights, tap sources) is spread
                              // over 6 units, and 48-unit layers give 8 CTAs per token block (whole waves at 4 per SM)

// y / (1 + exp(-y)) with expf and IEEE division (the general path)
__device__ __forceinline__ float silu_f(float y) { return __fdiv_rn(y, __fadd_rn(1.0f, expf(-y))); }
__device__ __forceinline__ float rcp_approx(float x) {
  float r;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}
// gate of a pair of bf16-valued y: y * rcp(1 + 2^(-y log2 e)) (valid for y > -87)
__device__ __forceinline__ uint64_t silu2(uint64_t y2) {
  constexpr float kNegLog2e = -1.4426950408889634f;
  const uint64_t a2 = f2mul(y2, f2(kNegLog2e, kNegLog2e));
  float a0, a1;
  f2get(a2, a0, a1);
  const uint64_t d2 = f2add(f2(ex2_approx(a0), ex2_approx(a1)), f2(1.0f, 1.0f));
  float d0, d1;
  f2get(d2, d0, d1);
  return f2mul(y2, f2(rcp_approx(d0), rcp_approx(d1)));
}
// bf16x2 word -> (lo, hi) fp32 pair
__device__ __forceinline__ uint64_t unpack2(uint32_t w) { return f2(bf_lo(w), bf_hi(w)); }
// fp32 pair -> bf16x2 word (round to nearest even)
__device__ __forceinline__ uint32_t pack2(uint64_t v) {
  float a, b;
  f2get(v, a, b);
  return pack_bf16(a, b);
}

template <int REP, bool SKIP_V>
__global__ void __launch_bounds__(256, 4)
conv_kernel(const uint16_t* __restrict__ qkv, long long SX, const uint16_t* __restrict__ cache, int C,
            const int4* __restrict__ meta, const uint16_t* __restrict__ w, uint16_t* __restrict__ q,
            uint16_t* __restrict__ k, uint16_t* __restrict__ v, int Tf, float eps, int KD, int VD, int u0, int u1) {
  constexpr int TB = CONV_TB, NSLOT = TB + 3, TPT = CONV_TPT;
  __shared__ __align__(16) uint4 tile[2][NSLOT][16];          // [stage][slot][16-byte column]
  __shared__ __align__(16) float wsm[CONV_UPC][4][128];       // [unit of the CTA][tap][channel], fp32
  __shared__ int4 smeta[TB];
  __shared__ const uint16_t* sptr[NSLOT];  // source row of each slot (nullptr: zero-filled), unit 0's columns
  const int tid = threadIdx.x, lane = tid & 31;
  const int r0 = TPT * (tid >> 5);  // first of this warp's 8 token rows
  const int tbeg = blockIdx.y * TB;
  const int ua = u0 + blockIdx.x * CONV_UPC, ub = min(ua + CONV_UPC, u1);
  const int nq = KD / 128, nqk = 2 * nq;
  for (int i = tid; i < TB; i += 256) {
    const int t = tbeg + i;
    smeta[i] = t < Tf ? __ldg(meta + t) : make_int4(-1000, 0, 0, 0);
  }
  for (int i = tid; i < (ub - ua) * 128; i += 256) {
    const uint2 wv = __ldg(reinterpret_cast<const uint2*>(w + (long long)(ua * 128 + i) * 4));
    float* wd = &wsm[i >> 7][0][i & 127];
    wd[0] = bf_lo(wv.x);
    wd[128] = bf_hi(wv.x);
    wd[256] = bf_lo(wv.y);
    wd[384] = bf_hi(wv.y);
  }
  __syncthreads();
  const int4 m0 = smeta[0];
  auto slot_src = [&](int slot) -> const uint16_t* {
    if (slot >= 3) {
      const int4 m = smeta[slot - 3];
      return (tbeg + slot - 3 < Tf && m.x >= m.y && m.x >= 0) ? qkv + (long long)(m.z + m.x) * SX : nullptr;
    }
    const int src = m0.x - (3 - slot);
    if (tbeg >= Tf || src < 0) return nullptr;
    return src >= m0.y ? qkv + (long long)(m0.z + src) * SX : cache + (long long)(m0.w + src) * C;
  };
  if (tid < NSLOT) sptr[tid] = slot_src(tid);
  __syncthreads();
  auto load_stage = [&](int stage, int u) {
#pragma unroll
    for (int i = 0; i < (NSLOT * 16 + 255) / 256; ++i) {
      const int id = tid + 256 * i;
      if (id < NSLOT * 16) {
        const int slot = id >> 4, c16 = id & 15;
        const uint16_t* src = sptr[slot];
        cp_async16(smem_u32(&tile[stage][slot][c16]), src ? src + u * 128 + 8 * c16 : qkv, src != nullptr);
      }
    }
    cp_async_commit();
  };
  // tap sources of this warp's tokens: bit (3*i + d-1) of tmask = token r0+i reads its distance-d tap from slot
  // 3 + r0 + i - d; `fast` = every token valid and every tap of every token in its slot.  Lane i < 8 works out token
  // r0 + i's bits; a warp OR and vote combine them.
  uint32_t mybits = 0;
  bool myok = true;
  if (lane < TPT) {
    const int row = r0 + lane;
    const int4 m = smeta[row];
    const bool valid = tbeg + row < Tf && m.x >= m.y && m.x >= 0;
    myok = valid;
    if (valid) {
#pragma unroll
      for (int d = 1; d <= 3; ++d) {
        const int src = m.x - d;
        bool hit = false;
        if (src >= 0) {
          if (row - d >= 0) {
            const int4 mn = smeta[row - d];
            hit = src >= m.y && mn.x >= mn.y && mn.x >= 0 && mn.z + mn.x == m.z + src;
          } else {  // halo: same sequence as token tbeg, contiguous from it
            hit = m.z == m0.z && m.y == m0.y && m.w == m0.w && m.x == m0.x + row;
          }
        }
        if (hit) mybits |= 1u << (3 * lane + d - 1);
        else myok = false;
      }
    }
  }
  const uint32_t tmask = __reduce_or_sync(0xffffffffu, mybits);
  const bool fast = __all_sync(0xffffffffu, myok);
  const bool b4 = lane & 16, b3 = lane & 8, b2 = lane & 4;
  const int nrows = Tf - (tbeg + r0);  // rows of this warp below Tf (may exceed TPT)
  if (ua < ub) load_stage(0, ua);
  for (int u = ua; u < ub; ++u) {
    const int stage = (u - ua) & 1;
    cp_async_wait<0>();
    // one barrier per unit: this stage has landed for every thread, and every thread has finished reading the other
    // stage (unit u-1), which the copy of unit u+1 now refills while unit u is computed
    __syncthreads();
    if (u + 1 < ub) load_stage(stage ^ 1, u + 1);
    const int cu = 4 * lane, c0 = u * 128 + cu;
    // weights of this thread's 4 channels: wp[j][p] = (w[c0+2p][j], w[c0+2p+1][j])
    uint64_t wp[4][2];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float4 a = *reinterpret_cast<const float4*>(&wsm[u - ua][j][cu]);
      wp[j][0] = f2(a.x, a.y);
      wp[j][1] = f2(a.z, a.w);
    }
    const uint2* trow = reinterpret_cast<const uint2*>(&tile[stage][0][0]) + lane;  // slot s: trow[32 * s]
    uint64_t acc[TPT][2];
#pragma unroll
    for (int i = 0; i < TPT; ++i) acc[i][0] = acc[i][1] = f2(0.f, 0.f);
    if (fast) {
      // slot 3 + (r0 + i) - d = r0 + i + j for tap j = 3 - d: the rows r0 .. r0+10, each unpacked once
#pragma unroll
      for (int e = 0; e < TPT + 3; ++e) {
        const uint2 xv = trow[32 * (r0 + e)];
        const uint64_t x2[2] = {unpack2(xv.x), unpack2(xv.y)};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int i = e - j;  // the token for which row e is tap j
          if (i < 0 || i >= TPT) continue;
          acc[i][0] = f2fma(wp[j][0], x2[0], acc[i][0]);
          acc[i][1] = f2fma(wp[j][1], x2[1], acc[i][1]);
        }
      }
    } else {
      // general path, token by token, taps in order 0..3; each token's sums enter at the top of acc, which shifts
      // down one token per step (static register indices: the loop is not unrolled)
#pragma unroll 1
      for (int i = 0; i < TPT; ++i) {
        const int row = r0 + i;
        const int4 m = smeta[row];
        const bool valid = tbeg + row < Tf && m.x >= m.y && m.x >= 0;
        uint64_t a0 = f2(0.f, 0.f), a1 = a0;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int d = 3 - j, src = m.x - d;
          if (!valid || src < 0) continue;
          uint2 xv;
          if (d == 0 || ((tmask >> (3 * i + d - 1)) & 1u)) {
            xv = trow[32 * (3 + row - d)];
          } else {
            const uint16_t* rp = src >= m.y ? qkv + (long long)(m.z + src) * SX : cache + (long long)(m.w + src) * C;
            xv = __ldg(reinterpret_cast<const uint2*>(rp + c0));
          }
          a0 = f2fma(wp[j][0], unpack2(xv.x), a0);
          a1 = f2fma(wp[j][1], unpack2(xv.y), a1);
        }
#pragma unroll
        for (int ii = 0; ii + 1 < TPT; ++ii) acc[ii][0] = acc[ii + 1][0], acc[ii][1] = acc[ii + 1][1];
        acc[TPT - 1][0] = a0;
        acc[TPT - 1][1] = a1;
      }
    }
    // y = bf16(acc); gate; s = bf16(gate)
    uint32_t sp[TPT][2];  // s as packed bf16 pairs
    float ymin = INFINITY;
    uint64_t y2[TPT][2];
#pragma unroll
    for (int i = 0; i < TPT; ++i)
#pragma unroll
      for (int p = 0; p < 2; ++p) {
        y2[i][p] = unpack2(pack2(acc[i][p]));
        float a, b;
        f2get(y2[i][p], a, b);
        asm("min.f32 %0, %1, %2, %3;" : "=f"(ymin) : "f"(ymin), "f"(a), "f"(b));
      }
    if (!(ymin > -87.0f)) {  // some y <= -87 (or nan): expf and IEEE division for this thread's values
#pragma unroll
      for (int i = 0; i < TPT; ++i)
#pragma unroll
        for (int p = 0; p < 2; ++p) {
          float a, b;
          f2get(y2[i][p], a, b);
          sp[i][p] = pack_bf16(silu_f(a), silu_f(b));
        }
    } else {
#pragma unroll
      for (int i = 0; i < TPT; ++i)
#pragma unroll
        for (int p = 0; p < 2; ++p) sp[i][p] = pack2(silu2(y2[i][p]));
    }
    if (u < nqk) {
      // per-token sum of s^2 over the 128 channels (32 lanes x 4): reduce-scatter over lane bits 4, 3, 2 (token
      // 4*b4 + 2*b3 + b2 stays with this lane), then a butterfly over bits 1, 0; every lane then fetches the 8 norm
      // factors from lanes 4t
      float s8[TPT];
#pragma unroll
      for (int i = 0; i < TPT; ++i) {
        const uint64_t sa2 = unpack2(sp[i][0]), sb2 = unpack2(sp[i][1]);
        const uint64_t ss = f2fma(sb2, sb2, f2mul(sa2, sa2));
        float sa, sb;
        f2get(ss, sa, sb);
        s8[i] = sa + sb;
      }
      float s4[4], s2v[2];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float send = b4 ? s8[i] : s8[i + 4], keep = b4 ? s8[i + 4] : s8[i];
        s4[i] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
      }
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const float send = b3 ? s4[i] : s4[i + 2], keep = b3 ? s4[i + 2] : s4[i];
        s2v[i] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
      }
      float s1;
      {
        const float send = b2 ? s2v[0] : s2v[1], keep = b2 ? s2v[1] : s2v[0];
        s1 = keep + __shfl_xor_sync(0xffffffffu, send, 4);
      }
      s1 += __shfl_xor_sync(0xffffffffu, s1, 2);
      s1 += __shfl_xor_sync(0xffffffffu, s1, 1);
      const float rs = rsqrtf(__fadd_rn(eps, s1));
      const int nh = REP * KD / 128, hq = u % nq;
      uint16_t* dst = (u < nq ? q : k) + (long long)(tbeg + r0) * (nh * 128) + REP * hq * 128 + cu;
#pragma unroll
      for (int i = 0; i < TPT; ++i, dst += nh * 128) {
        const float rstd = __shfl_sync(0xffffffffu, rs, 4 * i);
        if (i >= nrows) continue;
        const uint64_t r2 = f2(rstd, rstd);
        const uint2 ov = make_uint2(pack2(f2mul(unpack2(sp[i][0]), r2)), pack2(f2mul(unpack2(sp[i][1]), r2)));
        __stcs(reinterpret_cast<uint2*>(dst), ov);
        if (REP == 2) __stcs(reinterpret_cast<uint2*>(dst + 128), ov);
      }
    } else if (!SKIP_V) {
      uint16_t* dst = v + (long long)(tbeg + r0) * VD + (c0 - 2 * KD);
#pragma unroll
      for (int i = 0; i < TPT; ++i, dst += VD)
        if (i < nrows) __stcs(reinterpret_cast<uint2*>(dst), make_uint2(sp[i][0], sp[i][1]));
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
  if (SX % 8 || C % 8 ||
      (((uintptr_t)qkv | (uintptr_t)cache | (uintptr_t)w | (uintptr_t)q | (uintptr_t)k | (uintptr_t)v) & 15))
    return -1;
  if (nunits <= 0) return 0;
  const int tblocks = (Tf + CONV_TB - 1) / CONV_TB;
  if (tblocks > 65535) return -1;
  dim3 grid((nunits + CONV_UPC - 1) / CONV_UPC, tblocks);
  const int u1 = u0 + nunits;
  const uint16_t* a = (const uint16_t*)qkv;
  const uint16_t* cc = (const uint16_t*)cache;
  const int4* mt = (const int4*)meta;
  const uint16_t* ww = (const uint16_t*)w;
  uint16_t *qq = (uint16_t*)q, *kk = (uint16_t*)k, *vv = (uint16_t*)v;
  if (rep == 1 && !skip_v) conv_kernel<1, false><<<grid, 256, 0, st>>>(a, SX, cc, C, mt, ww, qq, kk, vv, Tf, eps, KD, VD, u0, u1);
  else if (rep == 1) conv_kernel<1, true><<<grid, 256, 0, st>>>(a, SX, cc, C, mt, ww, qq, kk, vv, Tf, eps, KD, VD, u0, u1);
  else if (!skip_v) conv_kernel<2, false><<<grid, 256, 0, st>>>(a, SX, cc, C, mt, ww, qq, kk, vv, Tf, eps, KD, VD, u0, u1);
  else conv_kernel<2, true><<<grid, 256, 0, st>>>(a, SX, cc, C, mt, ww, qq, kk, vv, Tf, eps, KD, VD, u0, u1);
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
