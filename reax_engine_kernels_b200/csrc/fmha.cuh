// Fused attention forward for sm_100a (tcgen05 + TMEM + TMA), head dim 128 or 256.
//
// Semantics (libreax_fmha_post/reax_fmha_v11.cu:6-13, :204-221, :295-450, :451-531):
//   per (batch b, kv head h), rows r < M:  O[r] = softmax(scale * Q[r] K^T + mask_or_bias[r]) V
//   qpos mode: key j visible iff j <= qpos[b*qpBs + r/G] (and j < N); bias mode: + bf16 bias[b,h,r,j].
//   Rows with no visible key produce 0.  POST (qpos mode only): out[inv[b*Lq + r/G]][(h*G + r%G)*D + d] =
//   bf16(bf16(O) * bf16(sigmoid(gate))), gate = qg[R*qg_rs + (h*G + r%G)*2D + D + d]; rows with inv < 0 skipped.
//
// One CTA = 128 query rows of one (b, h); 192 threads:
//   warp 0      TMA producer: the Q tile once, then K and V blocks of 128 keys (D/64 boxes of 64 columns, 128-byte
//               swizzle) into KST / VST-deep rings;
//   warp 1      TMEM owner + MMA issuer: S_j = Q K_j^T (M=128, N=128, K=D) into one of two TMEM score buffers,
//               then O += P_j V_j (M=128, N=D, K=128) with P read from TMEM (the bf16 P_j overwrites S_j) and V as
//               an MN-major shared-memory operand.  Issue order S0 S1 PV0 S2 PV1 ... keeps the tensor core busy
//               with S_{j+1} while the softmax works on S_j;
//   warps 2..5  softmax (thread = row, warp w owns TMEM lanes 32*(w%4)..+31): online softmax in the log2 domain
//               with the exact running max per 128-key block (the point where the reference rounds P to bf16),
//               P written back as bf16 with tcgen05.st, O rescaled in TMEM when a row's max grows, then the epilogue.
// Key blocks past the tile's last visible key are skipped; tiles are dispatched longest-first.
#pragma once
#include "common.cuh"

#include <type_traits>

namespace reax {

enum FmhaMode { FMHA_BIAS = 0, FMHA_QPOS = 1, FMHA_QPOS_POST = 2 };

struct FmhaParams {
  const uint16_t* bias;  // bf16 bits (bias mode)
  const int* qpos;
  int G;
  long long qpBs;
  uint16_t* o;
  float scale;       // softmax scale
  float scale_log2;  // scale * log2(e)
  int q_hc, q_bc, k_hc, k_bc, v_hc, v_bc;  // 0 where a stride-0 (broadcast) head / batch dim was folded
  int bias_vec;                            // 1: every bias row starts 16-byte aligned (vector loads)
  int M, N;
  long long bsB, bsH, bsM;
  long long osB, osH, osM;
  const int* inv;
  int Lq;
  const uint16_t* qg;
  long long qg_rs;
  uint16_t* outp;
  long long out_rs;
  int num_mtiles;
  int H, B;          // kv heads, batches
  int group_units;   // (batch, head) units per dispatch group (see cta_work)
};

// One CTA's (query tile, head, batch) from a 1-D grid.  The (batch, head) units are taken in groups of
// group_units; inside a group every unit's longest (latest) query tile comes first, then the next longest of every
// unit, and so on, so the hardware's in-order dispatch approximates longest-processing-time-first scheduling of the
// causal tiles across units.  A group's K/V (group_units x N keys) stays small enough to be shared through L2 by
// the CTAs running at the same time.
__device__ __forceinline__ void cta_work(const FmhaParams& p, int& mtile, int& h, int& b) {
  const int idx = (int)blockIdx.x;
  const int HB = p.H * p.B;
  const int per_group = p.num_mtiles * p.group_units;
  const int g = idx / per_group;
  const int r = idx - g * per_group;
  const int gu = min(p.group_units, HB - g * p.group_units);  // units in this group (the last may be smaller)
  const int mt = r / gu;
  const int unit = g * p.group_units + (r - mt * gu);
  mtile = p.num_mtiles - 1 - mt;
  h = unit % p.H;
  b = unit / p.H;
}

template <int D>
struct FmhaCfg {
  static constexpr int BM = 128, BN = 128;
  static constexpr int NB64 = D / 64;                  // 64-column boxes per row
  static constexpr uint32_t Q_BYTES = BM * D * 2;
  static constexpr uint32_t KV_BYTES = BN * D * 2;
  static constexpr int KST = D == 128 ? 2 : 1;
  static constexpr int VST = D == 128 ? 2 : 1;
  static constexpr uint32_t S_COL = 0;                 // S buffers at TMEM columns 0 and 128
  static constexpr uint32_t O_COL = 256;               // O accumulator at columns 256 .. 256+D
  static constexpr uint32_t TMEM_COLS = 512;
  static constexpr int SMEM = 1024 + Q_BYTES + (KST + VST) * KV_BYTES + 256;
};

// 2^x for a pair x <= 0 on the FMA pipe (relieves the MUFU unit, which alone would take as long as the tensor core
// per key block).  Cody-Waite split x = n + f with n = round(x) (adding 1.5 * 2^23 leaves n in the low mantissa bits)
// and |f| <= 1/2; 2^f by a degree-5 polynomial fitted for this project by reweighted least squares on [-1/2, 1/2]
// (max relative error 2^-22 in fp32 Horner form); 2^n added to the exponent field.  x < -126 (including -inf) gives
// 0, as MUFU ex2.approx.ftz does (its results below 2^-126 flush to zero); the lanes computed for such x are discarded.
__device__ __forceinline__ void exp2_fma_pair(uint64_t x2, float& r0, float& r1) {
  constexpr float MAGIC = 12582912.0f;
  float x0, x1;
  f2get(x2, x0, x1);
  const bool z0 = x0 < -126.0f, z1 = x1 < -126.0f;
  const uint64_t xc = x2;
  const uint64_t j = f2add(xc, f2(MAGIC, MAGIC));
  const uint64_t n = f2add(j, f2(-MAGIC, -MAGIC));
  const uint64_t f = f2fma(n, f2(-1.0f, -1.0f), xc);
  uint64_t pp = f2(1.327646896e-03f, 1.327646896e-03f);
  pp = f2fma(pp, f, f2(9.675540961e-03f, 9.675540961e-03f));
  pp = f2fma(pp, f, f2(5.550713465e-02f, 5.550713465e-02f));
  pp = f2fma(pp, f, f2(2.402212024e-01f, 2.402212024e-01f));
  pp = f2fma(pp, f, f2(6.931469440e-01f, 6.931469440e-01f));
  pp = f2fma(pp, f, f2(1.000000119e+00f, 1.000000119e+00f));
  float j0, j1, p0, p1;
  f2get(j, j0, j1);
  f2get(pp, p0, p1);
  r0 = z0 ? 0.f : __int_as_float(__float_as_int(p0) + (__float_as_int(j0) << 23));
  r1 = z1 ? 0.f : __int_as_float(__float_as_int(p1) + (__float_as_int(j1) << 23));
}

// Pairs of a fully visible block whose 2^x runs on the FMA pipe (exp2_fma_pair): every kPolyStride-th pair of keys.
// MUFU ex2 issues 16 results per clock per SM and the polynomial costs about five FMA-pipe cycles per result, so a
// few spread pairs let the two pipes work side by side.
constexpr int kPolyStride = 8;

// S_j row of this thread (tcgen05.ld) -> s[]: FOLD: the raw fp32 accumulators; otherwise the reference's log2-domain
// scores x = (acc * scale) * log2(e) (bias mode: (acc * scale + bias) * log2(e)), each product rounded to fp32.
// Keys outside the row's visibility are -inf.  Returns true when every key of the block is visible (qpos mode).
template <int MODE, bool FOLD>
__device__ __forceinline__ bool load_scores(const FmhaParams& p, uint32_t sbuf, int j, int row, int qlim, int b, int h,
                                            float (&s)[128]) {
  constexpr int BN = 128;
  constexpr float kLog2e = 1.4426950408889634074f;
  {
    uint32_t r[128];
    __syncwarp();         // tcgen05.ld/st are warp-collective (.sync.aligned): reconverge after the per-lane wait loop
    tmem_ld128(sbuf, r);  // the whole 128-key row of S_j, one round trip
#pragma unroll
    for (int i = 0; i < 128; ++i) s[i] = __uint_as_float(r[i]);
  }
  const int k0 = j * BN;
  bool full = false;
  if (MODE == FMHA_BIAS) {
    const bool live = row < p.M;
    const uint16_t* brow = p.bias + (long long)b * p.bsB + (long long)h * p.bsH + (long long)(live ? row : 0) * p.bsM + k0;
#pragma unroll
    for (int c = 0; c < 16; ++c) {
      uint4 bv = make_uint4(0, 0, 0, 0);
      const int kc = k0 + 8 * c;
      if (p.bias_vec && live && kc + 8 <= p.N) {
        bv = *reinterpret_cast<const uint4*>(brow + 8 * c);
      } else if (live && kc < p.N) {  // unaligned rows or the ragged row end: element loads, never past N-1
        uint16_t t8[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        for (int e = 0; e < 8 && kc + e < p.N; ++e) t8[e] = brow[8 * c + e];
        bv = make_uint4(t8[0] | ((uint32_t)t8[1] << 16), t8[2] | ((uint32_t)t8[3] << 16), t8[4] | ((uint32_t)t8[5] << 16),
                        t8[6] | ((uint32_t)t8[7] << 16));
      }
      const uint32_t w4[4] = {bv.x, bv.y, bv.z, bv.w};
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const int i = 8 * c + e;
        const float bb = (e & 1) ? bf_hi(w4[e >> 1]) : bf_lo(w4[e >> 1]);
        s[i] = (live && k0 + i < p.N) ? __fmul_rn(__fadd_rn(__fmul_rn(s[i], p.scale), bb), kLog2e) : -INFINITY;
      }
    }
  } else {
    full = k0 + BN - 1 <= qlim;
    if (!FOLD) {
      const uint64_t sc2 = f2(p.scale, p.scale), lg2 = f2(kLog2e, kLog2e);
#pragma unroll
      for (int i = 0; i < 128; i += 2) {
        const uint64_t x2 = f2mul(f2mul(f2(s[i], s[i + 1]), sc2), lg2);
        f2get(x2, s[i], s[i + 1]);
      }
    }
    if (!full) {
#pragma unroll
      for (int i = 0; i < 128; ++i) s[i] = k0 + i <= qlim ? s[i] : -INFINITY;
    }
  }
  return full;
}

// Block max in the log2 domain: a tree of independent 3-input maxima (one chain would serialise 64 dependent
// instructions); FOLD: the max of the raw accumulators scaled once (x is monotone in acc for scale > 0).
template <bool FOLD>
__device__ __forceinline__ float block_max(const FmhaParams& p, const float (&s)[128]) {
  float m8[8];
#pragma unroll
  for (int a = 0; a < 8; ++a) m8[a] = fmaxf(s[a], s[a + 8]);
#pragma unroll
  for (int i = 16; i < 128; i += 16)
#pragma unroll
    for (int a = 0; a < 8; a += 2) {
      m8[a] = max3f(m8[a], s[i + a], s[i + a + 8]);
      m8[a + 1] = max3f(m8[a + 1], s[i + a + 1], s[i + a + 9]);
    }
  const float mraw = fmaxf(max3f(m8[0], m8[1], m8[2]), max3f(max3f(m8[3], m8[4], m8[5]), m8[6], m8[7]));
  return FOLD ? __fmul_rn(mraw, p.scale_log2) : mraw;
}

// 2^d for a pair of exponent arguments: d = acc * c - m (FOLD) or x - m
template <bool FOLD, bool POLY>
__device__ __forceinline__ void exp_pair(float s0, float s1, uint64_t c2, uint64_t nmu2, float& a, float& b) {
  const uint64_t d2 = FOLD ? f2fma(f2(s0, s1), c2, nmu2) : f2add(f2(s0, s1), nmu2);
  if (POLY) {
    exp2_fma_pair(d2, a, b);
  } else {
    float d0, d1;
    f2get(d2, d0, d1);
    a = ex2_approx(d0);
    b = ex2_approx(d1);
  }
}

// One 128-key block of the online softmax for this thread's row (thread = TMEM lane = query row), one-tile kernel:
// S_j (fp32, TMEM) -> log2-domain scores -> exact running max -> P_j = bf16(2^(x - m)) written back over S_j,
// running sum of the unrounded probabilities, O (TMEM) rescaled when the row's max grew.  Returns false when a bounded
// wait gave up.  The rounding point of the reference kept exactly is P = bf16(2^(x - m)) at the exact running max m.
// Scores: FOLD (qpos mode, scale > 0): x = acc * c with c = fp32(scale * log2(e)); x is monotone in acc, so the row max
// is taken on the raw accumulators and each exponent argument is one FMA, d = acc * c - m.  Otherwise the reference's
// own chain x = (acc * scale) * log2(e) (bias mode: (acc * scale + bias) * log2(e)), each product rounded to fp32.
// The two score forms differ by a few fp32 ulps of x, the size of the accumulation-order differences of the dot
// product itself.
template <int D, int MODE, bool FOLD, int RCH = 128>
__device__ __forceinline__ bool softmax_block(const FmhaParams& p, uint32_t sbuf, uint32_t obuf, int j, int row, int qlim,
                                              int b, int h, float& m_run, float& l, uint32_t pv_done,
                                              volatile int* abort_flag) {
  float s[128];
  const bool full = load_scores<MODE, FOLD>(p, sbuf, j, row, qlim, b, h, s);
  const float mx = block_max<FOLD>(p, s);
  // exact running max (the reference's rounding point for P): on a new max, l and O scale by 2^(m_old - m_new)
  const bool grow = mx > m_run;
  const float m_new = grow ? mx : m_run;
  const bool rescale = grow && m_run != -INFINITY;
  const float alpha = rescale ? exp2f(m_run - m_new) : 1.0f;
  l = rescale ? __fmul_rn(l, alpha) : l;
  const float mu = m_new == -INFINITY ? 0.f : m_new;  // a row with nothing visible yet: every p is 0
  const uint64_t nmu2 = f2(-mu, -mu), c2 = f2(p.scale_log2, p.scale_log2);
  uint64_t sum4[4] = {f2(0.f, 0.f), f2(0.f, 0.f), f2(0.f, 0.f), f2(0.f, 0.f)};  // independent partial sums
  uint32_t pr[64];
  auto run = [&](auto poly_tag) {
    constexpr bool POLY = decltype(poly_tag)::value;
#pragma unroll
    for (int i = 0; i < 64; ++i) {
      float a, bq;
      if (POLY && i % kPolyStride == 0)
        exp_pair<FOLD, true>(s[2 * i], s[2 * i + 1], c2, nmu2, a, bq);
      else
        exp_pair<FOLD, false>(s[2 * i], s[2 * i + 1], c2, nmu2, a, bq);
      sum4[i & 3] = f2add(sum4[i & 3], f2(a, bq));  // the normaliser sums the unrounded probabilities
      pr[i] = pack_bf16(a, bq);
    }
  };
  if (MODE != FMHA_BIAS && full) run(std::true_type{});
  else run(std::false_type{});
  __syncwarp();         // the bias loads branch per lane (live / dead rows): reconverge before the collective store
  tmem_st64(sbuf, pr);  // P_j (bf16 pairs) over the first 64 columns of S_j, one round trip
  float s0, s1, s2, s3, s4, s5, s6, s7;
  f2get(sum4[0], s0, s1);
  f2get(sum4[1], s2, s3);
  f2get(sum4[2], s4, s5);
  f2get(sum4[3], s6, s7);
  l += ((s0 + s1) + (s2 + s3)) + ((s4 + s5) + (s6 + s7));
  if (j > 0) {
    // Observe PV_{j-1} at every block, not only when rescaling: an mbarrier parity wait is only meaningful while the
    // barrier is at most one phase away, so a thread must not skip phases of pv_done (a thread that waited for phase
    // j+1 while phase j-1 was still open would be released by the parity of phase j-1).  Placed after P_j is
    // written, so PV_{j-1} normally completed meanwhile.
    if (!mbar_wait_warp(pv_done, (uint32_t)(j - 1) & 1u, abort_flag, ST_TIMEOUT_ATTN)) return false;
    tc_fence_after();
  }
  if (__any_sync(0xffffffffu, rescale) && j > 0) {
    // O holds PV_0..PV_{j-1} (complete, observed above): scale this warp's rows in place (lanes whose max did not
    // move use alpha = 1), RCH columns per round trip (128 where the register budget allows)
    __syncwarp();
    const uint64_t al2 = f2(alpha, alpha);
#pragma unroll 1
    for (int c = 0; c < D / RCH; ++c) {
      uint32_t r[RCH];
      if constexpr (RCH == 128) tmem_ld128(obuf + (uint32_t)(c * RCH), r);
      else tmem_ld64(obuf + (uint32_t)(c * RCH), r);
#pragma unroll
      for (int i = 0; i < RCH; i += 2) {
        const uint64_t o2 = f2mul(f2(__uint_as_float(r[i]), __uint_as_float(r[i + 1])), al2);
        float o0, o1;
        f2get(o2, o0, o1);
        r[i] = __float_as_uint(o0);
        r[i + 1] = __float_as_uint(o1);
      }
      if constexpr (RCH == 128) tmem_st128(obuf + (uint32_t)(c * RCH), r);
      else tmem_st64(obuf + (uint32_t)(c * RCH), r);
    }
  }
  m_run = m_new;
  return true;
}

// Pass 2 of the two-tile softmax for this thread's row: P = bf16(2^(acc * c - m)) for the 128 keys of S (TMEM),
// streamed in 16-key chunks (the next chunk's load in flight while one is computed; tcgen05.wait::ld waits for every
// earlier load, so each wait follows the computation it overlaps) and written back over S, 8 packed words per chunk
// (P chunk c covers S columns 8c..8c+7, all read by then); sum4 accumulates the unrounded probabilities.
__device__ __forceinline__ void exp_pass(uint32_t sbuf, uint64_t c2, uint64_t nmu2, uint64_t (&sum4)[4]) {
  uint32_t sb[2][16];
  tmem_ld16_nowait(sbuf, sb[0]);
  tmem_wait_ld16(sb[0]);
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    uint32_t(&sc)[16] = sb[c & 1];
    if (c < 7) tmem_ld16_nowait(sbuf + (uint32_t)(16 * (c + 1)), sb[(c + 1) & 1]);
    uint32_t pr[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      float a, bq;
      if ((8 * c + i) % kPolyStride == 0)
        exp_pair<true, true>(__uint_as_float(sc[2 * i]), __uint_as_float(sc[2 * i + 1]), c2, nmu2, a, bq);
      else
        exp_pair<true, false>(__uint_as_float(sc[2 * i]), __uint_as_float(sc[2 * i + 1]), c2, nmu2, a, bq);
      sum4[i & 3] = f2add(sum4[i & 3], f2(a, bq));
      pr[i] = pack_bf16(a, bq);
    }
    tmem_st8_nowait(sbuf + (uint32_t)(8 * c), pr);
    if (c < 7) tmem_wait_ld16(sb[(c + 1) & 1]);
  }
}

// The two-tile kernel's softmax block (head dim 128, qpos mode with the folded score form).  Same arithmetic as
// softmax_block, split in two so the O rescale leaves this warp's critical path: pass 1 reads the row of S_j for the
// max, updates the running max and normaliser and publishes this row's alpha = 2^(m_old - m_new) (plus the warp's
// "some row grew" flag) for the other tile's warp of the same TMEM lane quarter, which rescales O (help_rescale) while
// this warp computes exponents; pass 2 (exp_pass) streams S_j again and writes P_j over it.  A block with masked keys
// (at most the two diagonal blocks of a tile) writes -inf over them in pass 1, so pass 2 is one loop for every block.
template <int MODE>
__device__ __forceinline__ void softmax_block2(const FmhaParams& p, uint32_t sbuf, int j, int row, int qlim, int b,
                                               int h, float& m_run, float& l, float* alpha_slot, int* flag_slot,
                                               uint32_t alpha_bar) {
  static_assert(MODE != FMHA_BIAS, "qpos modes only");
  float mx;
  {
    float s[128];
    const bool full = load_scores<MODE, true>(p, sbuf, j, row, qlim, b, h, s);
    mx = block_max<true>(p, s);
    if (__any_sync(0xffffffffu, !full)) {
      uint32_t r[128];
#pragma unroll
      for (int i = 0; i < 128; ++i) r[i] = __float_as_uint(s[i]);
      tmem_st128(sbuf, r);  // masked keys as -inf (rows of the warp that see every key store their values unchanged)
    }
  }
  const bool grow = mx > m_run;
  const float m_new = grow ? mx : m_run;
  const bool rescale = grow && m_run != -INFINITY;
  const float alpha = rescale ? exp2f(m_run - m_new) : 1.0f;
  l = rescale ? __fmul_rn(l, alpha) : l;
  const float mu = m_new == -INFINITY ? 0.f : m_new;
  const uint64_t nmu2 = f2(-mu, -mu), c2 = f2(p.scale_log2, p.scale_log2);
  const bool resc = __any_sync(0xffffffffu, rescale) && j > 0;  // warp-uniform
  *alpha_slot = alpha;
  if ((threadIdx.x & 31) == 0) *flag_slot = resc ? 1 : 0;
  mbar_arrive(alpha_bar);  // release: the helper reads alpha and the flag after its wait
  __syncwarp();
  uint64_t sum4[4] = {f2(0.f, 0.f), f2(0.f, 0.f), f2(0.f, 0.f), f2(0.f, 0.f)};
  exp_pass(sbuf, c2, nmu2, sum4);
  tmem_wait_st();  // P_j is in TMEM before the caller's fence and arrive
  float s0, s1, s2, s3, s4, s5, s6, s7;
  f2get(sum4[0], s0, s1);
  f2get(sum4[1], s2, s3);
  f2get(sum4[2], s4, s5);
  f2get(sum4[3], s6, s7);
  l += ((s0 + s1) + (s2 + s3)) + ((s4 + s5) + (s6 + s7));
  m_run = m_new;
}

// O rescale of the OTHER tile's rows in this warp's TMEM lane quarter for block j: waits for that tile's published
// alphas, and when some row's max grew, for PV_{j-1} of that tile (observed through its pv_done barrier; the barrier is
// then at phase j-1 or j, since PV_j needs this warp's o_ready first), scales the 128 O columns in 32-column chunks
// (one in flight while another is scaled) and signals o_ready.  Returns false when a bounded wait gave up.
__device__ __forceinline__ bool help_rescale(uint32_t obuf, int j, const float* alpha_slot, const int* flag_slot,
                                             uint32_t alpha_bar, uint32_t pv_done, uint32_t o_ready,
                                             volatile int* abort_flag) {
  if (!mbar_wait_warp(alpha_bar, (uint32_t)j & 1u, abort_flag, ST_TIMEOUT_ATTN)) return false;
  if (*reinterpret_cast<const volatile int*>(flag_slot) != 0) {  // warp-uniform: one flag per warp
    const float alpha = *reinterpret_cast<const volatile float*>(alpha_slot);
    if (!mbar_wait_warp(pv_done, (uint32_t)(j - 1) & 1u, abort_flag, ST_TIMEOUT_ATTN)) return false;
    tc_fence_after();
    __syncwarp();
    const uint64_t al2 = f2(alpha, alpha);
    uint32_t ob[2][32];
    tmem_ld32_nowait(obuf, ob[0]);
    tmem_wait_ld32(ob[0]);
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      uint32_t(&oc)[32] = ob[c & 1];
      if (c < 3) tmem_ld32_nowait(obuf + (uint32_t)(32 * (c + 1)), ob[(c + 1) & 1]);
#pragma unroll
      for (int i = 0; i < 32; i += 2) {
        const uint64_t o2 = f2mul(f2(__uint_as_float(oc[i]), __uint_as_float(oc[i + 1])), al2);
        float o0, o1;
        f2get(o2, o0, o1);
        oc[i] = __float_as_uint(o0);
        oc[i + 1] = __float_as_uint(o1);
      }
      tmem_st32_nowait(obuf + (uint32_t)(32 * c), oc);
      if (c < 3) tmem_wait_ld32(ob[(c + 1) & 1]);
    }
    tmem_wait_st();
  }
  tc_fence_before();
  mbar_arrive(o_ready);
  return true;
}

// Epilogue for this thread's row: O / l as bf16 to o (or the attn_post gate + scatter); `have` is false when the row's
// CTA had no key block (O was never written) or a wait gave up -- the row then gets zeros.
template <int D, int MODE>
__device__ __forceinline__ void attn_epilogue(const FmhaParams& p, uint32_t obuf, bool have, int row, int b, int h, float l) {
  const bool live = row < p.M;
  const float inv_l = l > 0.f ? 1.0f / l : 0.f;
  if (MODE != FMHA_QPOS_POST) {
    uint16_t* orow = p.o + (long long)b * p.osB + (long long)h * p.osH + (long long)(live ? row : 0) * p.osM;
#pragma unroll 1
    for (int c = 0; c < D / 32; ++c) {
      uint32_t r[32];
      __syncwarp();  // reconverge (per-lane wait loop, the previous pass's row-dependent stores) before tcgen05.ld
      if (have) {
        tmem_ld32(obuf + (uint32_t)(c * 32), r);
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) r[i] = 0u;
      }
      if (live) {
#pragma unroll
        for (int v = 0; v < 4; ++v) {
          uint4 o4;
          o4.x = pack_bf16(__uint_as_float(r[8 * v + 0]) * inv_l, __uint_as_float(r[8 * v + 1]) * inv_l);
          o4.y = pack_bf16(__uint_as_float(r[8 * v + 2]) * inv_l, __uint_as_float(r[8 * v + 3]) * inv_l);
          o4.z = pack_bf16(__uint_as_float(r[8 * v + 4]) * inv_l, __uint_as_float(r[8 * v + 5]) * inv_l);
          o4.w = pack_bf16(__uint_as_float(r[8 * v + 6]) * inv_l, __uint_as_float(r[8 * v + 7]) * inv_l);
          *reinterpret_cast<uint4*>(orow + c * 32 + 8 * v) = o4;
        }
      }
    }
  } else {
    const int R = live ? p.inv[(long long)b * p.Lq + row / p.G] : -1;
    const long long hq = (long long)h * p.G + row % p.G;
    const uint16_t* grow = p.qg + (long long)(R < 0 ? 0 : R) * p.qg_rs + hq * 2 * D + D;
    uint16_t* orow = p.outp + (long long)(R < 0 ? 0 : R) * p.out_rs + hq * D;
#pragma unroll 1
    for (int c = 0; c < D / 32; ++c) {
      uint32_t r[32];
      __syncwarp();  // reconverge (per-lane wait loop, the previous pass's row-dependent stores) before tcgen05.ld
      if (have) {
        tmem_ld32(obuf + (uint32_t)(c * 32), r);
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) r[i] = 0u;
      }
      if (R >= 0) {
#pragma unroll
        for (int v = 0; v < 4; ++v) {
          const uint4 g4 = *reinterpret_cast<const uint4*>(grow + c * 32 + 8 * v);
          const uint32_t gw[4] = {g4.x, g4.y, g4.z, g4.w};
          uint32_t res[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const uint32_t ob = pack_bf16(__uint_as_float(r[8 * v + 2 * e]) * inv_l, __uint_as_float(r[8 * v + 2 * e + 1]) * inv_l);
            const float s0 = 1.0f / (1.0f + expf(-bf_lo(gw[e])));
            const float s1 = 1.0f / (1.0f + expf(-bf_hi(gw[e])));
            const uint32_t sg = pack_bf16(s0, s1);
            // bf16 x bf16 product rounded once to bf16
            res[e] = pack_bf16(bf_lo(ob) * bf_lo(sg), bf_hi(ob) * bf_hi(sg));
          }
          *reinterpret_cast<uint4*>(orow + c * 32 + 8 * v) = make_uint4(res[0], res[1], res[2], res[3]);
        }
      }
    }
  }
}

template <int D, int MODE, bool FOLD>
__global__ void __launch_bounds__(192, 1)
fmha_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
            const __grid_constant__ CUtensorMap tv, const FmhaParams p) {
  using C = FmhaCfg<D>;
  constexpr int KST = C::KST, VST = C::VST, NB64 = C::NB64;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t sbase = (raw + 1023u) & ~1023u;
  const uint32_t sq = sbase;
  const uint32_t sk = sq + C::Q_BYTES;
  const uint32_t sv = sk + KST * C::KV_BYTES;
  const uint32_t bars = sv + VST * C::KV_BYTES;
  // barriers: q_full | k_full[KST] | k_empty[KST] | v_full[VST] | v_empty[VST] | s_full[2] | p_ready[2] | pv_done
  const uint32_t q_full = bars;
  auto k_full = [&](int s) { return bars + 8u * (1 + s); };
  auto k_empty = [&](int s) { return bars + 8u * (1 + KST + s); };
  auto v_full = [&](int s) { return bars + 8u * (1 + 2 * KST + s); };
  auto v_empty = [&](int s) { return bars + 8u * (1 + 2 * KST + VST + s); };
  auto s_full = [&](int s) { return bars + 8u * (1 + 2 * KST + 2 * VST + s); };
  auto p_ready = [&](int s) { return bars + 8u * (3 + 2 * KST + 2 * VST + s); };
  const uint32_t pv_done = bars + 8u * (5 + 2 * KST + 2 * VST);
  const uint32_t drain = bars + 8u * (6 + 2 * KST + 2 * VST);
  const uint32_t misc = bars + 8u * (7 + 2 * KST + 2 * VST);  // tmem holder, abort flag, qmax reduction
  uint8_t* misc_ptr = smem_raw + (misc - raw);
  const uint32_t* holder_ptr = reinterpret_cast<const uint32_t*>(misc_ptr);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(misc_ptr + 4);
  int* qmax_red = reinterpret_cast<int*>(misc_ptr + 8);  // 4 ints

  const int warp = warp_id(), lane = lane_id();
  int mtile, h, b;
  cta_work(p, mtile, h, b);
  const int m0 = mtile * C::BM;

  // ---- per-row visibility limit (softmax threads) and the CTA's last visible key
  const int q = warp & 3;
  const int row = m0 + 32 * q + lane;  // meaningful for warps 2..5
  int qlim = -1;
  if (warp >= 2) {
    if (MODE == FMHA_BIAS) {
      qlim = row < p.M ? p.N - 1 : -1;
    } else {
      qlim = row < p.M ? p.qpos[(long long)b * p.qpBs + row / p.G] : -1;
      qlim = min(qlim, p.N - 1);
    }
    const int wmax = __reduce_max_sync(0xffffffffu, qlim);
    if (lane == 0) qmax_red[q] = wmax;
  }
  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < KST; ++s) {
      mbar_init(k_full(s), 1);
      mbar_init(k_empty(s), 1);
    }
    for (int s = 0; s < VST; ++s) {
      mbar_init(v_full(s), 1);
      mbar_init(v_empty(s), 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(s_full(s), 1);
      mbar_init(p_ready(s), 128);
    }
    mbar_init(pv_done, 1);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tq);
    tma_prefetch_desc(&tk);
    tma_prefetch_desc(&tv);
  }
  if (warp == 1) {
    tmem_alloc(misc, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *holder_ptr;
  const int cta_qmax = max(max(qmax_red[0], qmax_red[1]), max(qmax_red[2], qmax_red[3]));
  const int nkb_all = (p.N + C::BN - 1) / C::BN;
  const int nkb = cta_qmax < 0 ? 0 : min(nkb_all, cta_qmax / C::BN + 1);

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0 && nkb > 0) {
      mbar_arrive_expect_tx(q_full, C::Q_BYTES);
#pragma unroll
      for (int c = 0; c < NB64; ++c) tma_load_4d(sq + c * (C::BM * 128), &tq, q_full, c * 64, m0, h * p.q_hc, b * p.q_bc);
      uint32_t kph = 0, vph = 0;
      int ks = 0, vs = 0;
      CopyLedger led;  // the Q copy's barrier is slot 0, K stages 1..KST, V stages 1+KST..
      led.arm(0, 0);
      bool ok = true;
      for (int j = 0; j < nkb && ok; ++j) {
        if (!mbar_wait(k_empty(ks), kph ^ 1u, abort_flag, ST_TIMEOUT_ATTN)) { ok = false; break; }
        mbar_arrive_expect_tx(k_full(ks), C::KV_BYTES);
        const uint32_t kdst = sk + ks * C::KV_BYTES;
#pragma unroll
        for (int c = 0; c < NB64; ++c) tma_load_4d(kdst + c * (C::BN * 128), &tk, k_full(ks), c * 64, j * C::BN, h * p.k_hc, b * p.k_bc);
        led.arm(1 + ks, kph);
        if (++ks == KST) { ks = 0; kph ^= 1u; }
        if (!mbar_wait(v_empty(vs), vph ^ 1u, abort_flag, ST_TIMEOUT_ATTN)) { ok = false; break; }
        mbar_arrive_expect_tx(v_full(vs), C::KV_BYTES);
        const uint32_t vdst = sv + vs * C::KV_BYTES;
#pragma unroll
        for (int c = 0; c < NB64; ++c) tma_load_4d(vdst + c * (C::BN * 128), &tv, v_full(vs), c * 64, j * C::BN, h * p.v_hc, b * p.v_bc);
        led.arm(1 + KST + vs, vph);
        if (++vs == VST) { vs = 0; vph ^= 1u; }
      }
      if (!ok) record_status(ST_TIMEOUT_ATTN);
      // teardown: never leave the CTA while a copy into its shared memory may still be in flight
      led.drain([&](int slot) { return slot == 0 ? q_full : slot <= KST ? k_full(slot - 1) : v_full(slot - 1 - KST); });
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0 && nkb > 0) {
      constexpr uint32_t IDESC_S = idesc_bf16(128, C::BN);
      constexpr uint32_t IDESC_PV = idesc_bf16(128, D, /*b_mn_major=*/1);
      bool ok = mbar_wait(q_full, 0, abort_flag, ST_TIMEOUT_ATTN);
      uint32_t kph = 0, vph = 0;
      int ks = 0, vs = 0;
      auto issue_s = [&](int j) -> bool {
        // S_j overwrites the TMEM buffer holding P_{j-2}; PV_{j-2} was issued earlier by this thread and one thread's
        // MMAs execute in issue order.  The completion wait below is kept anyway: PV_{j-1} is already queued behind
        // PV_{j-2}, so it costs the tensor core nothing here.
        if (j >= 2 && !mbar_wait(pv_done, (uint32_t)(j - 2) & 1u, abort_flag, ST_TIMEOUT_ATTN)) return false;
        if (!mbar_wait(k_full(ks), kph, abort_flag, ST_TIMEOUT_ATTN)) return false;
        tc_fence_after();
        const uint32_t kbase = sk + ks * C::KV_BYTES;
        const uint32_t d_tmem = tmem + C::S_COL + (uint32_t)((j & 1) * 128);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (uint32_t)((kk >> 2) * (C::BM * 128) + (kk & 3) * 32);
          mma_bf16_ss(d_tmem, sw128_desc(sq + off), sw128_desc(kbase + (uint32_t)((kk >> 2) * (C::BN * 128) + (kk & 3) * 32)),
                      IDESC_S, kk > 0);
        }
        mma_commit(k_empty(ks));
        mma_commit(s_full(j & 1));
        if (++ks == KST) { ks = 0; kph ^= 1u; }
        return true;
      };
      auto issue_pv = [&](int j) -> bool {
        if (!mbar_wait(p_ready(j & 1), (uint32_t)(j >> 1) & 1u, abort_flag, ST_TIMEOUT_ATTN)) return false;
        if (!mbar_wait(v_full(vs), vph, abort_flag, ST_TIMEOUT_ATTN)) return false;
        tc_fence_after();
        const uint32_t vbase = sv + vs * C::KV_BYTES;
        const uint32_t a_tmem = tmem + C::S_COL + (uint32_t)((j & 1) * 128);
#pragma unroll
        for (int kk = 0; kk < C::BN / 16; ++kk)
          mma_bf16_ts(tmem + C::O_COL, a_tmem + (uint32_t)(kk * 8),
                      sw128_desc(vbase + (uint32_t)(kk * 2048), /*lbo=*/C::BN * 128, /*sbo=*/1024), IDESC_PV,
                      (j > 0 || kk > 0) ? 1u : 0u);
        mma_commit(v_empty(vs));
        mma_commit(pv_done);
        if (++vs == VST) { vs = 0; vph ^= 1u; }
        return true;
      };
      if (ok) ok = issue_s(0);
      for (int j = 1; j < nkb && ok; ++j) {
        ok = issue_s(j);
        if (ok) ok = issue_pv(j - 1);
      }
      if (ok) ok = issue_pv(nkb - 1);
      mma_commit(drain);
      const long long t0 = clock64();
      while (!mbar_try_wait(drain, 0)) {
        if (clock64() - t0 > REAX_DRAIN_LIMIT) { record_status(ST_TIMEOUT_DRAIN); break; }
      }
    }
  } else {
    // ------------------------------------------------------------------ softmax + epilogue (thread = row)
    const uint32_t lane_base = tmem + ((uint32_t)(32 * q) << 16);
    float m_run = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < nkb && ok; ++j) {
      if (!mbar_wait_warp(s_full(j & 1), (uint32_t)(j >> 1) & 1u, abort_flag, ST_TIMEOUT_ATTN)) { ok = false; break; }
      tc_fence_after();
      const uint32_t sbuf = lane_base + C::S_COL + (uint32_t)((j & 1) * 128);
      if (!softmax_block<D, MODE, FOLD>(p, sbuf, lane_base + C::O_COL, j, row, qlim, b, h, m_run, l, pv_done,
                                        abort_flag)) {
        ok = false;
        break;
      }
      tc_fence_before();
      mbar_arrive(p_ready(j & 1));
    }
    if (ok && nkb > 0) {
      if (!mbar_wait_warp(pv_done, (uint32_t)(nkb - 1) & 1u, abort_flag, ST_TIMEOUT_ATTN)) ok = false;
      tc_fence_after();
    }
    attn_epilogue<D, MODE>(p, lane_base + C::O_COL, ok && nkb > 0, row, b, h, l);
  }
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}


// Two query tiles per CTA (head dim 128): 256 query rows share every K/V block, 320 threads:
//   warp 0 TMA producer, warp 1 MMA issuer, warps 2..5 softmax of tile 0, warps 6..9 softmax of tile 1.
// TMEM (512 columns): S0 [0,128) S1 [128,256) O0 [256,384) O1 [384,512); P_t overwrites S_t as bf16.
// Issue order per key block j:  S0_j | PV1_{j-1} | S1_j | PV0_j  -- while softmax 0 works on S0_j the tensor core runs
// PV1_{j-1} and S1_j, and while softmax 1 works on S1_j it runs PV0_j and S0_{j+1}: each softmax has two MMAs of
// cover (S_t,j follows PV_t,j-1 on the same TMEM columns without a wait: one thread's MMAs execute in issue order).
// K_j is released after S1_j, V_j after PV1_j.
template <int MODE, bool FOLD>
__global__ void __launch_bounds__(320, 1)
fmha2_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
             const __grid_constant__ CUtensorMap tv, const FmhaParams p) {
  constexpr int D = 128, BM = 128, BN = 128, NB64 = 2;
  constexpr uint32_t QT = BM * D * 2, KVB = BN * D * 2;
  constexpr int KST = 2, VST = 2;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t sbase = (raw + 1023u) & ~1023u;
  const uint32_t sq = sbase;                     // Q0, Q1
  const uint32_t sk = sq + 2 * QT;
  const uint32_t sv = sk + KST * KVB;
  const uint32_t bars = sv + VST * KVB;
  const uint32_t q_full = bars;
  auto k_full = [&](int s) { return bars + 8u * (1 + s); };
  auto k_empty = [&](int s) { return bars + 8u * (3 + s); };
  auto v_full = [&](int s) { return bars + 8u * (5 + s); };
  auto v_empty = [&](int s) { return bars + 8u * (7 + s); };
  auto s_full = [&](int t) { return bars + 8u * (9 + t); };
  auto p_ready = [&](int t) { return bars + 8u * (11 + t); };
  auto pv_done = [&](int t) { return bars + 8u * (13 + t); };
  const uint32_t drain = bars + 8u * 15;
  auto o_ready = [&](int t) { return bars + 8u * (16 + t); };                  // O of tile t rescaled (128 lanes)
  auto alpha_bar = [&](int t, int q) { return bars + 8u * (18 + 4 * t + q); };  // alphas of tile t, quarter q
  const uint32_t misc = bars + 256u;
  uint8_t* misc_ptr = smem_raw + (misc - raw);
  const uint32_t* holder_ptr = reinterpret_cast<const uint32_t*>(misc_ptr);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(misc_ptr + 4);
  int* qmax_red = reinterpret_cast<int*>(misc_ptr + 8);                        // 8 ints
  float* alpha_s = reinterpret_cast<float*>(misc_ptr + 64);                    // [tile][slot][128 rows]
  int* flag_s = reinterpret_cast<int*>(misc_ptr + 64 + 2 * 2 * 128 * 4);       // [tile][slot][4 quarters]

  const int warp = warp_id(), lane = lane_id();
  int mtile, h, b;
  cta_work(p, mtile, h, b);
  const int m0 = mtile * 2 * BM;
  const int t = warp >= 2 ? (warp - 2) >> 2 : 0;  // softmax tile of this warp
  const int q = warp & 3;
  const int row = m0 + BM * t + 32 * q + lane;
  int qlim = -1;
  if (warp >= 2) {
    if (MODE == FMHA_BIAS) {
      qlim = row < p.M ? p.N - 1 : -1;
    } else {
      qlim = row < p.M ? p.qpos[(long long)b * p.qpBs + row / p.G] : -1;
      qlim = min(qlim, p.N - 1);
    }
    const int wmax = __reduce_max_sync(0xffffffffu, qlim);
    if (lane == 0) qmax_red[warp - 2] = wmax;
  }
  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s2 = 0; s2 < 2; ++s2) {
      mbar_init(k_full(s2), 1);
      mbar_init(k_empty(s2), 1);
      mbar_init(v_full(s2), 1);
      mbar_init(v_empty(s2), 1);
      mbar_init(s_full(s2), 1);
      mbar_init(p_ready(s2), 128);
      mbar_init(pv_done(s2), 1);
      mbar_init(o_ready(s2), 128);
      for (int q2 = 0; q2 < 4; ++q2) mbar_init(alpha_bar(s2, q2), 32);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tq);
    tma_prefetch_desc(&tk);
    tma_prefetch_desc(&tv);
  }
  if (warp == 1) {
    tmem_alloc(misc, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *holder_ptr;
  int cta_qmax = -1;
#pragma unroll
  for (int i = 0; i < 8; ++i) cta_qmax = max(cta_qmax, qmax_red[i]);
  const int nkb_all = (p.N + BN - 1) / BN;
  const int nkb = cta_qmax < 0 ? 0 : min(nkb_all, cta_qmax / BN + 1);

  if (warp == 0) {
    if (lane == 0 && nkb > 0) {
      mbar_arrive_expect_tx(q_full, 2 * QT);
#pragma unroll
      for (int tt = 0; tt < 2; ++tt)
#pragma unroll
        for (int c = 0; c < NB64; ++c)
          tma_load_4d(sq + tt * QT + c * (BM * 128), &tq, q_full, c * 64, m0 + BM * tt, h * p.q_hc, b * p.q_bc);
      uint32_t kph = 0, vph = 0;
      int ks = 0, vs = 0;
      CopyLedger led;  // slot 0: Q, 1..2: K stages, 3..4: V stages
      led.arm(0, 0);
      for (int j = 0; j < nkb; ++j) {
        if (!mbar_wait(k_empty(ks), kph ^ 1u, abort_flag, ST_TIMEOUT_ATTN)) break;
        mbar_arrive_expect_tx(k_full(ks), KVB);
#pragma unroll
        for (int c = 0; c < NB64; ++c)
          tma_load_4d(sk + ks * KVB + c * (BN * 128), &tk, k_full(ks), c * 64, j * BN, h * p.k_hc, b * p.k_bc);
        led.arm(1 + ks, kph);
        if (++ks == KST) { ks = 0; kph ^= 1u; }
        if (!mbar_wait(v_empty(vs), vph ^ 1u, abort_flag, ST_TIMEOUT_ATTN)) break;
        mbar_arrive_expect_tx(v_full(vs), KVB);
#pragma unroll
        for (int c = 0; c < NB64; ++c)
          tma_load_4d(sv + vs * KVB + c * (BN * 128), &tv, v_full(vs), c * 64, j * BN, h * p.v_hc, b * p.v_bc);
        led.arm(1 + KST + vs, vph);
        if (++vs == VST) { vs = 0; vph ^= 1u; }
      }
      // teardown: never leave the CTA while a copy into its shared memory may still be in flight
      led.drain([&](int slot) { return slot == 0 ? q_full : slot <= KST ? k_full(slot - 1) : v_full(slot - 1 - KST); });
    }
  } else if (warp == 1) {
    if (lane == 0 && nkb > 0) {
      constexpr uint32_t IDESC_S = idesc_bf16(128, BN);
      constexpr uint32_t IDESC_PV = idesc_bf16(128, D, /*b_mn_major=*/1);
      bool ok = mbar_wait(q_full, 0, abort_flag, ST_TIMEOUT_ATTN);
      auto issue_s = [&](int tt, int j) {
        const int ks = j & 1;
        const uint32_t kbase = sk + ks * KVB, qbase = sq + tt * QT;
        const uint32_t d_tmem = tmem + (uint32_t)(tt * 128);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (uint32_t)((kk >> 2) * (BM * 128) + (kk & 3) * 32);
          mma_bf16_ss(d_tmem, sw128_desc(qbase + off), sw128_desc(kbase + (uint32_t)((kk >> 2) * (BN * 128) + (kk & 3) * 32)),
                      IDESC_S, kk > 0);
        }
        mma_commit(s_full(tt));
      };
      auto issue_pv = [&](int tt, int j) {
        const uint32_t vbase = sv + (j & 1) * KVB;
        const uint32_t a_tmem = tmem + (uint32_t)(tt * 128);
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk)
          mma_bf16_ts(tmem + 256u + (uint32_t)(tt * 128), a_tmem + (uint32_t)(kk * 8),
                      sw128_desc(vbase + (uint32_t)(kk * 2048), /*lbo=*/BN * 128, /*sbo=*/1024), IDESC_PV,
                      (j > 0 || kk > 0) ? 1u : 0u);
        mma_commit(pv_done(tt));
      };
      auto wait_k = [&](int j) { return mbar_wait(k_full(j & 1), (uint32_t)(j >> 1) & 1u, abort_flag, ST_TIMEOUT_ATTN); };
      auto wait_v = [&](int j) { return mbar_wait(v_full(j & 1), (uint32_t)(j >> 1) & 1u, abort_flag, ST_TIMEOUT_ATTN); };
      auto wait_p = [&](int tt, int j) {
        if (!mbar_wait(p_ready(tt), (uint32_t)j & 1u, abort_flag, ST_TIMEOUT_ATTN)) return false;
        if (FOLD && !mbar_wait(o_ready(tt), (uint32_t)j & 1u, abort_flag, ST_TIMEOUT_ATTN)) return false;
        tc_fence_after();
        return true;
      };
      if (ok) ok = wait_k(0);
      if (ok) {
        tc_fence_after();
        issue_s(0, 0);
        issue_s(1, 0);
        mma_commit(k_empty(0));
        ok = wait_p(0, 0) && wait_v(0);
        if (ok) issue_pv(0, 0);
      }
      // S_t,j overwrites the TMEM buffer PV_t,j-1 read P_t,j-1 from; both are issued by this thread and tcgen05.mma
      // operations of one thread are executed in issue order, so no completion wait sits between them
      for (int j = 1; j < nkb && ok; ++j) {
        if (!(ok = wait_k(j))) break;
        tc_fence_after();
        issue_s(0, j);
        if (!(ok = wait_p(1, j - 1))) break;
        issue_pv(1, j - 1);
        mma_commit(v_empty((j - 1) & 1));
        issue_s(1, j);
        mma_commit(k_empty(j & 1));
        if (!(ok = wait_p(0, j) && wait_v(j))) break;
        issue_pv(0, j);
      }
      if (ok && wait_p(1, nkb - 1)) {
        issue_pv(1, nkb - 1);
        mma_commit(v_empty((nkb - 1) & 1));
      }
      mma_commit(drain);
      const long long t0 = clock64();
      while (!mbar_try_wait(drain, 0)) {
        if (clock64() - t0 > REAX_DRAIN_LIMIT) { record_status(ST_TIMEOUT_DRAIN); break; }
      }
    }
  } else {
    const uint32_t lane_base = tmem + ((uint32_t)(32 * q) << 16);
    const uint32_t sbuf = lane_base + (uint32_t)(t * 128);
    const uint32_t obuf = lane_base + 256u + (uint32_t)(t * 128);
    float m_run = -INFINITY, l = 0.f;
    bool ok = true;
    if constexpr (FOLD) {
      // tile 1's warps rescale tile 0's O for block j before their own block j; tile 0's warps rescale tile 1's O
      // after theirs (each is idle then, waiting for its next S)
      const int u = 1 - t;
      const uint32_t obuf_u = lane_base + 256u + (uint32_t)(u * 128);
      for (int j = 0; j < nkb && ok; ++j) {
        const int slot = j & 1;
        auto help = [&]() {
          return help_rescale(obuf_u, j, alpha_s + (u * 2 + slot) * 128 + 32 * q + lane, flag_s + (u * 2 + slot) * 4 + q,
                              alpha_bar(u, q), pv_done(u), o_ready(u), abort_flag);
        };
        if (t == 1 && !(ok = help())) break;
        if (!mbar_wait_warp(s_full(t), (uint32_t)j & 1u, abort_flag, ST_TIMEOUT_ATTN)) { ok = false; break; }
        tc_fence_after();
        softmax_block2<MODE>(p, sbuf, j, row, qlim, b, h, m_run, l, alpha_s + (t * 2 + slot) * 128 + 32 * q + lane,
                             flag_s + (t * 2 + slot) * 4 + q, alpha_bar(t, q));
        tc_fence_before();
        mbar_arrive(p_ready(t));
        if (t == 0 && !(ok = help())) break;
      }
    } else {
      for (int j = 0; j < nkb && ok; ++j) {
        if (!mbar_wait_warp(s_full(t), (uint32_t)j & 1u, abort_flag, ST_TIMEOUT_ATTN)) { ok = false; break; }
        tc_fence_after();
        // 168 registers a thread at 320 threads: the O rescale in 64-column round trips
        if (!softmax_block<D, MODE, FOLD, 64>(p, sbuf, obuf, j, row, qlim, b, h, m_run, l, pv_done(t), abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_before();
        mbar_arrive(p_ready(t));
      }
    }
    if (ok && nkb > 0) {
      if (!mbar_wait_warp(pv_done(t), (uint32_t)(nkb - 1) & 1u, abort_flag, ST_TIMEOUT_ATTN)) ok = false;
      tc_fence_after();
    }
    attn_epilogue<D, MODE>(p, obuf, ok && nkb > 0, row, b, h, l);
  }
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace reax

namespace reax_host {

struct FmhaArgs {
  const void *q, *k, *v, *bias;
  const int* qpos;
  int G;
  long long qpBs;
  void* o;
  float scale;
  int B, H, M, N;
  long long qsB, qsH, qsM, ksB, ksH, ksM, vsB, vsH, vsM, bsB, bsH, bsM, osB, osH, osM;
  const int* inv;
  int Lq;
  const void* qg;
  long long qg_rs;
  void* outp;
  long long out_rs;
};

// [B, H, rows, D] strided bf16 tensor -> 4-D tensor map with boxes of 64 x 128 rows (stride-0 batch/head dims are
// folded to extent 1 so broadcast layouts stay legal).
inline bool fmha_map(CUtensorMap* m, const void* base, int D, int rows, int H, int B, long long sRow, long long sH,
                     long long sB) {
  const uint64_t dims[4] = {(uint64_t)D, (uint64_t)rows, (uint64_t)(sH == 0 ? 1 : H), (uint64_t)(sB == 0 ? 1 : B)};
  const uint64_t strides[3] = {(uint64_t)sRow * 2, (uint64_t)(sH == 0 ? sRow * rows : sH) * 2,
                               (uint64_t)(sB == 0 ? (sH == 0 ? sRow * rows : sH * H) : sB) * 2};
  const uint32_t box[4] = {64, 128, 1, 1};
  return make_map_bf16(m, base, 4, dims, strides, box);
}

inline bool fmha_al(long long s) { return (s % 8) == 0; }

// argument checks shared by the launchers: 16-byte alignment of every row start (TMA and the vector epilogue)
template <int MODE>
inline bool fmha_args_ok(const FmhaArgs& a) {
  using namespace reax;
  if (a.N < 0 || a.G <= 0 || a.H > 65535 || a.B > 65535) return false;
  if (!fmha_al(a.qsB) || !fmha_al(a.qsH) || !fmha_al(a.qsM) || !fmha_al(a.ksB) || !fmha_al(a.ksH) || !fmha_al(a.ksM) ||
      !fmha_al(a.vsB) || !fmha_al(a.vsH) || !fmha_al(a.vsM))
    return false;
  if (((uintptr_t)a.q | (uintptr_t)a.k | (uintptr_t)a.v) & 15) return false;
  if (MODE != FMHA_QPOS_POST && (!fmha_al(a.osB) || !fmha_al(a.osH) || !fmha_al(a.osM) || ((uintptr_t)a.o & 15)))
    return false;
  if (MODE == FMHA_QPOS_POST && (!fmha_al(a.qg_rs) || !fmha_al(a.out_rs) || (((uintptr_t)a.qg | (uintptr_t)a.outp) & 15)))
    return false;
  return true;
}

template <int MODE>
inline reax::FmhaParams fmha_params(const FmhaArgs& a, int num_mtiles) {
  using namespace reax;
  FmhaParams p;
  p.bias = static_cast<const uint16_t*>(a.bias);
  p.qpos = a.qpos;
  p.G = a.G;
  p.qpBs = a.qpBs;
  p.o = static_cast<uint16_t*>(a.o);
  p.scale = a.scale;
  p.bias_vec = MODE == FMHA_BIAS && fmha_al(a.bsM) && fmha_al(a.bsH) && fmha_al(a.bsB) && (((uintptr_t)a.bias & 15) == 0);
  p.scale_log2 = a.scale * 1.4426950408889634f;
  // stride-0 (broadcast) head / batch dims are folded to extent 1 in the tensor maps and indexed at 0
  p.q_hc = a.qsH != 0;
  p.q_bc = a.qsB != 0;
  p.k_hc = a.ksH != 0;
  p.k_bc = a.ksB != 0;
  p.v_hc = a.vsH != 0;
  p.v_bc = a.vsB != 0;
  p.M = a.M;
  p.N = a.N;
  p.bsB = a.bsB;
  p.bsH = a.bsH;
  p.bsM = a.bsM;
  p.osB = a.osB;
  p.osH = a.osH;
  p.osM = a.osM;
  p.inv = a.inv;
  p.Lq = a.Lq;
  p.qg = static_cast<const uint16_t*>(a.qg);
  p.qg_rs = a.qg_rs;
  p.outp = static_cast<uint16_t*>(a.outp);
  p.out_rs = a.out_rs;
  p.num_mtiles = num_mtiles;
  p.H = a.H;
  p.B = a.B;
  p.group_units = a.H * a.B < 8 ? a.H * a.B : 8;
  return p;
}

// qpos-mode scores take the folded form x = acc * fp32(scale * log2(e)) when that is a positive finite number
template <int MODE>
inline bool fmha_fold(const FmhaArgs& a) {
  const float c = a.scale * 1.4426950408889634f;
  return MODE != reax::FMHA_BIAS && a.scale > 0.f && c > 0.f && c <= 3.0e38f;
}

template <int D, int MODE, bool FOLD>
inline int launch_fmha_k(const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv, const reax::FmhaParams& p,
                         int H, int B, cudaStream_t stream) {
  using namespace reax;
  static SmemAttr attr;
  constexpr int SMEM = FmhaCfg<D>::SMEM;
  static_assert(SMEM <= 232448, "smem");
  if (ensure_smem(attr, fmha_kernel<D, MODE, FOLD>, SMEM) != cudaSuccess) return (int)cudaErrorInvalidValue;
  const long long ctas = (long long)p.num_mtiles * H * B;
  if (ctas > 0x7fffffffLL) return (int)cudaErrorInvalidValue;
  fmha_kernel<D, MODE, FOLD><<<(unsigned)ctas, 192, SMEM, stream>>>(mq, mk, mv, p);
  return (int)cudaGetLastError();
}

template <int D, int MODE>
inline int launch_fmha(const FmhaArgs& a, cudaStream_t stream) {
  using namespace reax;
  if (a.B <= 0 || a.H <= 0 || a.M <= 0) return 0;
  if (!fmha_args_ok<MODE>(a)) return -2;
  CUtensorMap mq, mk, mv;
  const int nrows_kv = a.N > 0 ? a.N : 1;
  if (!fmha_map(&mq, a.q, D, a.M, a.H, a.B, a.qsM, a.qsH, a.qsB)) return -2;
  if (!fmha_map(&mk, a.k, D, nrows_kv, a.H, a.B, a.ksM, a.ksH, a.ksB)) return -2;
  if (!fmha_map(&mv, a.v, D, nrows_kv, a.H, a.B, a.vsM, a.vsH, a.vsB)) return -2;
  const FmhaParams p = fmha_params<MODE>(a, (a.M + 127) / 128);
  if (MODE != FMHA_BIAS && fmha_fold<MODE>(a)) return launch_fmha_k<D, MODE, MODE != FMHA_BIAS>(mq, mk, mv, p, a.H, a.B, stream);
  return launch_fmha_k<D, MODE, false>(mq, mk, mv, p, a.H, a.B, stream);
}

// head dim 128, two query tiles per CTA (used when the 256-row CTAs still fill the GPU)
constexpr int kFmha2Smem = 1024 + 2 * (128 * 128 * 2) + 4 * (128 * 128 * 2) + 256 + 64 + 2 * 2 * 128 * 4 + 64;
static_assert(kFmha2Smem <= 232448, "smem");

template <int MODE, bool FOLD>
inline int launch_fmha2_k(const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv, const reax::FmhaParams& p,
                          int H, int B, cudaStream_t stream) {
  using namespace reax;
  static SmemAttr attr;
  if (ensure_smem(attr, fmha2_kernel<MODE, FOLD>, kFmha2Smem) != cudaSuccess) return (int)cudaErrorInvalidValue;
  const long long ctas = (long long)p.num_mtiles * H * B;
  if (ctas > 0x7fffffffLL) return (int)cudaErrorInvalidValue;
  fmha2_kernel<MODE, FOLD><<<(unsigned)ctas, 320, kFmha2Smem, stream>>>(mq, mk, mv, p);
  return (int)cudaGetLastError();
}

template <int MODE>
inline int launch_fmha2(const FmhaArgs& a, cudaStream_t stream) {
  using namespace reax;
  // the caller (launch_fmha_hd) has validated the arguments through the same checks as launch_fmha
  CUtensorMap mq, mk, mv;
  const int nrows_kv = a.N > 0 ? a.N : 1;
  if (!fmha_map(&mq, a.q, 128, a.M, a.H, a.B, a.qsM, a.qsH, a.qsB)) return -2;
  if (!fmha_map(&mk, a.k, 128, nrows_kv, a.H, a.B, a.ksM, a.ksH, a.ksB)) return -2;
  if (!fmha_map(&mv, a.v, 128, nrows_kv, a.H, a.B, a.vsM, a.vsH, a.vsB)) return -2;
  const FmhaParams p = fmha_params<MODE>(a, (a.M + 255) / 256);
  if (MODE != FMHA_BIAS && fmha_fold<MODE>(a)) return launch_fmha2_k<MODE, MODE != FMHA_BIAS>(mq, mk, mv, p, a.H, a.B, stream);
  return launch_fmha2_k<MODE, false>(mq, mk, mv, p, a.H, a.B, stream);
}

template <int MODE>
inline int launch_fmha_hd(const FmhaArgs& a, int hd, cudaStream_t st) {
  if (hd == 128) {
    int dev = 0;
    cudaGetDevice(&dev);
    const long long ctas2 = (long long)((a.M + 255) / 256) * a.H * a.B;
    if (a.B > 0 && a.H > 0 && a.M > 0 && ctas2 >= 2LL * device_sms(dev) && fmha_args_ok<MODE>(a))
      return launch_fmha2<MODE>(a, st);
    return launch_fmha<128, MODE>(a, st);
  }
  if (hd == 256) return launch_fmha<256, MODE>(a, st);
  return -3;
}

}  // namespace reax_host

// ------------------------------------------------------------------------------------------------
// exported entry points (reax_fmha_v11.cu:566-590 argument lists), defined once per including library
// ------------------------------------------------------------------------------------------------
#define REAX_DEFINE_FMHA_EXPORTS()                                                                                      \
  REAX_API int reax_fmha_b_hd(const void* q, const void* k, const void* v, const void* bias, void* o, float scale, int B,  \
                              int H, int M, int N, long long qsB, long long qsH, long long qsM, long long ksB,             \
                              long long ksH, long long ksM, long long vsB, long long vsH, long long vsM, long long bsB,   \
                              long long bsH, long long bsM, long long osB, long long osH, long long osM, int head_dim,    \
                              void* stream) {                                                                              \
    if (!bias) return -1;                                                                                                  \
    reax_host::FmhaArgs a{q,   k,   v,   bias, nullptr, 1,   0,   o,   scale, B,   H,      M,       N,   qsB, qsH, qsM,    \
                          ksB, ksH, ksM, vsB,  vsH,     vsM, bsB, bsH, bsM,   osB, osH,    osM,     nullptr, 0, nullptr,  \
                          0,   nullptr, 0};                                                                                \
    return reax_host::launch_fmha_hd<reax::FMHA_BIAS>(a, head_dim, (cudaStream_t)stream);                                 \
  }                                                                                                                        \
  REAX_API int reax_fmha_b(const void* q, const void* k, const void* v, const void* bias, void* o, float scale, int B,     \
                           int H, int M, int N, long long qsB, long long qsH, long long qsM, long long ksB, long long ksH, \
                           long long ksM, long long vsB, long long vsH, long long vsM, long long bsB, long long bsH,       \
                           long long bsM, long long osB, long long osH, long long osM, void* stream) {                     \
    return reax_fmha_b_hd(q, k, v, bias, o, scale, B, H, M, N, qsB, qsH, qsM, ksB, ksH, ksM, vsB, vsH, vsM, bsB, bsH, bsM, \
                          osB, osH, osM, 256, stream);                                                                     \
  }                                                                                                                        \
  REAX_API int reax_fmha_q_hd(const void* q, const void* k, const void* v, const int* qpos, int G, long long qpBs,         \
                              void* o, float scale, int B, int H, int M, int N, long long qsB, long long qsH,             \
                              long long qsM, long long ksB, long long ksH, long long ksM, long long vsB, long long vsH,   \
                              long long vsM, long long osB, long long osH, long long osM, int head_dim, void* stream) {   \
    reax_host::FmhaArgs a{q,   k,   v,   nullptr, qpos, G,   qpBs, o,   scale, B,   H,   M,       N,   qsB, qsH, qsM,     \
                          ksB, ksH, ksM, vsB,     vsH,  vsM, 0,    0,   0,     osB, osH, osM,     nullptr, 0, nullptr,    \
                          0,   nullptr, 0};                                                                                \
    return reax_host::launch_fmha_hd<reax::FMHA_QPOS>(a, head_dim, (cudaStream_t)stream);                                 \
  }                                                                                                                        \
  REAX_API int reax_fmha_q(const void* q, const void* k, const void* v, const int* qpos, int G, long long qpBs, void* o,   \
                           float scale, int B, int H, int M, int N, long long qsB, long long qsH, long long qsM,           \
                           long long ksB, long long ksH, long long ksM, long long vsB, long long vsH, long long vsM,       \
                           long long osB, long long osH, long long osM, void* stream) {                                    \
    return reax_fmha_q_hd(q, k, v, qpos, G, qpBs, o, scale, B, H, M, N, qsB, qsH, qsM, ksB, ksH, ksM, vsB, vsH, vsM, osB,  \
                          osH, osM, 256, stream);                                                                          \
  }

#define REAX_DEFINE_FMHA_QP_EXPORT()                                                                                    \
  REAX_API int reax_fmha_qp(const void* q, const void* k, const void* v, const int* qpos, int G, long long qpBs,           \
                            float scale, int B, int H, int M, int N, long long qsB, long long qsH, long long qsM,          \
                            long long ksB, long long ksH, long long ksM, long long vsB, long long vsH, long long vsM,      \
                            const int* inv, int Lq, const void* qg, long long qg_rs, void* outp, long long out_rs,        \
                            void* stream) {                                                                                \
    reax_host::FmhaArgs a{q,   k,   v,   nullptr, qpos, G,   qpBs, nullptr, scale, B,  H,     M,    N,     qsB, qsH, qsM,  \
                          ksB, ksH, ksM, vsB,     vsH,  vsM, 0,    0,       0,     0,  0,     0,    inv,   Lq,  qg,        \
                          qg_rs, outp, out_rs};                                                                            \
    return reax_host::launch_fmha<256, reax::FMHA_QPOS_POST>(a, (cudaStream_t)stream);                                   \
  }
