// Chunked gated delta rule (WY form, 64-token chunks) on the 5th-generation tensor core, sm_100a: reax_howu,
// howu3_skip, howu3_dense, and reax_howu_norm (the same kernel with its rows scattered, then an in-place gated RMSNorm
// pass).
//
// Semantics (libreax_howu/reax_howu.cu:124-347), per (sequence, value head hv, key head kh = hv / (HV/H)), chunk of
// nval <= 64 tokens, state h[128 k][128 v] (fp32):
//   vb = bf16(beta v);  kb = bf16(bf16(beta k) 2^g);  u = A vb;  w = bf16(A kb)     (A: lower 16x16 blocks, or all)
//   Aq[t][s] = bf16((q_t . k_s) 2^(g_t - g_s)) for s <= t (valid), else 0
//   Hb = bf16(h);  x = bf16(u) - w Hb;  vn = bf16(x);  vdec = bf16(x 2^(g_last - g_t))
//   o = bf16(scale (Aq vn) + scale 2^(g_t) (q Hb));   h <- h 2^(g_last) + k^T vdec
// Every bf16 rounding point above is kept; the fp32 sums inside the products run in the tensor core's order.
//
// One CTA per (sequence, value head, 64-column slice of the state; the recurrence is independent per value column),
// serial over the chunks, 544 threads in three roles: warps 0-7 the chain (the epilogues on the recurrence; warp w reads
// TMEM lane quarter w % 4, column half w / 4), warp 8 one MMA-issuing thread, warps 9-16 helpers (loads of the next
// chunk's q, k, v, A by cp.async into tiles double-buffered by chunk parity, the kb / vb operands, the w epilogue).
// Per chunk c the issuer runs three MMA groups, in this order B(c), C(c), A(c+1):
//   A(c)  [w | u] = A [kb | vb] (one N = 192 MMA per k step; doneA: the helpers turn w into a bf16 operand tile) and
//         q k^T (doneQ: the chain's Aq epilogue: masked, decayed, bf16)            (M = 64: row t of an accumulator
//         sits in TMEM lane 32(t/16) + t%16)
//   B(c)  w Hb and q Hb, interleaved (doneB: the chain's S5, x = bf16(u) - w Hb -> vn, vdec as bf16 operand tiles)
//   C(c)  h += k^T vdec (M = 128: key dims in TMEM lanes 0..127, k read as an MN-major operand) and Aq vn (doneC: the
//         chain's S7, o staged and stored, Hb = bf16(h) published and h scaled by the next chunk's 2^(g_last))
// so the next chunk's first products run while the chain finishes o and Hb.
// The state lives in TMEM for the whole sequence.  Operand tiles are 128-byte-swizzled row-major (row r, 16-byte chunk
// c of a 64-column block at r*128 + ((c ^ (r & 7)) << 4); 128-column tiles are two blocks 8192 bytes apart): the
// canonical K-major layout when the row is an M/N index and the MN-major layout when the row is the K index.
#pragma once
#include "common.cuh"
#include "gate_table.cuh"

namespace reax {

struct HowuTcSmem {
  uint8_t kr[2][16384];  // raw k [64 tokens][128 dims] of chunk c in kr[c % 2]
  uint8_t kbv[2][24576];  // chunk c in kbv[c % 2]: kb [64 tokens][128 dims], then v -> vb [64 tokens][64 columns]
                          // (one MN-major operand of N = 192 for u and w together)
  uint8_t q[2][16384];   // [64 tokens][128 dims], chunk c in q[c % 2]
  uint8_t w[16384];      // bf16(A kb) [64 tokens][128 dims]
  uint8_t hb[16384];     // bf16(h) [128 dims][64 value columns]
  uint8_t a[2][8192];    // A [64][64], chunk c in a[c % 2]
  uint8_t aq[8192];     // Aq [64][64]
  uint8_t vn[8192];     // vn [64 tokens][64 columns]
  uint8_t vd[8192];     // vdec [64 tokens][64 columns]
  uint8_t ost[8192];    // o of a chunk, stored to global memory while the next chunk's first MMAs run
  float g[2][64], eg[2][64], beta[2][64], da[2][64];  // per chunk parity
  int f2s[2][64];                                      // output row of each token (SCATTER), per chunk parity
  unsigned long long bar[7];  // doneA, doneB, doneC, doneQ (MMA commits), rdyA, rdyB, rdyC (operands ready)
  uint32_t tmem;
  int abort;
};
constexpr int kHowuTcSmemBytes = (int)sizeof(HowuTcSmem) + 1024;  // + slack: tiles start on 1024-byte boundaries
constexpr uint32_t HT_W = 0, HT_U = 128, HT_AQ = 192, HT_OI = 256, HT_H = 320, HT_VW = 384, HT_CI = 448;  // TMEM columns

// byte offset of bf16 element (r, c) in a swizzled tile of 64-column blocks
__device__ __forceinline__ uint32_t ht_off(int r, int c) {
  return (uint32_t)((c >> 6) * 8192 + r * 128 + ((((c >> 3) & 7) ^ (r & 7)) << 4) + (c & 7) * 2);
}
// K-step kk (16 elements) of a K-major operand whose K runs along the row (64-element blocks 8192 bytes apart)
__device__ __forceinline__ uint64_t ht_kdesc(uint32_t tile, int kk) {
  return sw128_desc(tile + (uint32_t)((kk >> 2) * 8192 + (kk & 3) * 32));
}
// K-step kk (16 rows) of an MN-major operand whose K runs down the rows (the M/N index along the row)
__device__ __forceinline__ uint64_t ht_mndesc(uint32_t tile, int kk) {
  return sw128_desc(tile + (uint32_t)(kk * 2048), /*lbo=*/8192, /*sbo=*/1024);
}
__device__ __forceinline__ void ht_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n\t"
      "tcgen05.wait::ld.sync.aligned;\n"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
}

// AND of a predicate over the NTHREADS threads of named barrier ID (which they all reach)
template <int ID, int NTHREADS>
__device__ __forceinline__ bool named_bar_and(bool p) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred pi, po;\n\t"
      "setp.ne.u32 pi, %1, 0;\n\t"
      "bar.red.and.pred po, %2, %3, pi;\n\t"
      "selp.u32 %0, 1, 0, po;\n\t}\n"
      : "=r"(r)
      : "r"((uint32_t)p), "n"(ID), "n"(NTHREADS)
      : "memory");
  return r != 0;
}

// Warps 0-7 (256 threads): elementwise work and epilogues, synchronised among themselves by named barrier 1.
// Warp 8: its lane 0 issues every MMA.  Warps 9-12: load (cp.async) the next chunk's tiles and scalars as soon as G1
// of the current chunk has completed.  Hand-offs by mbarriers: rdy[0..2] (256 arrivals: operands of G1 / G2 / G3 ready),
// done[0..3] (MMA commits: u, w / q k^T, q Hb / w Hb / Aq vn, h), landed (256 arrivals: each loader thread once for its
// scalar stores and once, by cp.async.mbarrier.arrive, when its copies have completed).
// Roles (17 warps).  Warps 0-7 ("chain", named barrier 1): the Aq epilogue and the epilogues on the recurrence —
// x = bf16(u) - w Hb -> vn, vdec; o; Hb and the 2^(g_last) rescale of h for the next chunk.  Warp 8: its lane 0 issues
// every MMA.  Warps 9-16 ("helpers", named barrier 2): loads, the chunk's derived operands (scalars, vb, kb) and the
// w epilogue.  Per chunk c the MMA thread issues  B(c) = {q Hb, w Hb},  C(c) = {Aq vn, h += k^T vdec},  then
// A(c+1) = {u, w} and {q k^T} of the next chunk (two commits, so the w epilogue need not wait for q k^T), so the next
// chunk's first products run while the chain warps finish o and Hb.  q, raw k, kb, v and A are double-buffered by chunk parity, so the next chunk's copies start as soon as the
// previous chunk's last MMA group has completed.  Hand-offs by mbarriers: doneA/Q/B/C (commits), rdyA (helpers: the
// chunk's operands are ready), rdyB (chain: Hb ready and h rescaled; helpers: w tile ready), rdyC (chain: Aq, vn,
// vdec ready).
// SCATTER: row t of o goes to output row f2s[t] (skipped when negative) — the first pass of the norm entry point.
template <bool SKIPA, bool SCATTER>
__global__ void __launch_bounds__(544, 1)
howu_tc_kernel(const uint16_t* __restrict__ q, const uint16_t* __restrict__ k, const uint16_t* __restrict__ v,
               const uint16_t* __restrict__ beta, const uint16_t* __restrict__ Ag, const float* __restrict__ g,
               uint16_t* __restrict__ o, const long long* __restrict__ cu, float scale, int NSEQ, int H, int HV,
               const int* __restrict__ f2s) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  HowuTcSmem& S = *reinterpret_cast<HowuTcSmem*>(smem_raw + (((raw + 1023u) & ~1023u) - raw));
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, gq = lane >> 2, tq = lane & 3;
  const int sl = (int)(blockIdx.x & 1), bx = (int)(blockIdx.x >> 1), c_lo = 64 * sl;
  // last sequence first, like the reference's dispatch
  const int n = NSEQ - 1 - bx / HV, hv = bx % HV, kh = hv / (HV / H);
  const long long bos = cu[n], T = cu[n + 1] - bos;

  if (warp == 0) {
    tmem_alloc(smem_u32(&S.tmem), 512);
    tmem_relinquish();
  }
  const uint32_t bar_base = smem_u32(&S.bar[0]);
  const uint32_t doneA = bar_base, doneB = bar_base + 8, doneC = bar_base + 16, doneQ = bar_base + 48;
  const uint32_t rdyA = bar_base + 24, rdyB = bar_base + 32, rdyC = bar_base + 40;
  if (tid == 0) {
    mbar_init(doneA, 1);
    mbar_init(doneB, 1);
    mbar_init(doneC, 1);
    mbar_init(doneQ, 1);
    mbar_init(rdyA, 256);
    mbar_init(rdyB, 512);
    mbar_init(rdyC, 256);
    fence_mbar_init();
    S.abort = 0;
  }
  const uint32_t skr0 = smem_u32(S.kr[0]), skb0 = smem_u32(S.kbv[0]), sq0 = smem_u32(S.q[0]),
                 sa0 = smem_u32(S.a[0]), sw = smem_u32(S.w), shb = smem_u32(S.hb), saq = smem_u32(S.aq),
                 svn = smem_u32(S.vn), svd = smem_u32(S.vd), sost = smem_u32(S.ost);
  // chunk c's tiles
  auto krt = [&](int c) { return skr0 + 16384u * (uint32_t)(c & 1); };
  auto kbt = [&](int c) { return skb0 + 24576u * (uint32_t)(c & 1); };
  auto qt = [&](int c) { return sq0 + 16384u * (uint32_t)(c & 1); };
  auto vt = [&](int c) { return kbt(c) + 16384u; };
  auto at = [&](int c) { return sa0 + 8192u * (uint32_t)(c & 1); };
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = S.tmem;
  const int nchunks = (int)((T + 63) / 64);
  const int qd = warp & 3;                              // TMEM lane quarter of this warp
  const uint32_t tq_lane = (uint32_t)(32 * qd) << 16;  // ... in a TMEM address
  const int ra = 16 * qd + gq, rb = ra + 8;            // the two token rows of this thread in the M = 64 epilogues
  // 16 rows (16qd + gq, + 8) x 16 columns of an M = 64 accumulator, m16n8 fragment layout
  auto ld64 = [&](uint32_t col, float (&x)[8]) {
    uint32_t r[8];
    tmem_ld_16x256b_x2(tmem + tq_lane + col, r);
#pragma unroll
    for (int e = 0; e < 8; ++e) x[e] = __uint_as_float(r[e]);
  };
  // stores a fragment pair (row, columns c, c + 1) into a bf16 tile
  auto st_pair = [&](uint32_t tile, int r, int c, float a, float b) {
    asm volatile("st.shared.b32 [%0], %1;" ::"r"(tile + ht_off(r, c)), "r"(pack_bf16(a, b)) : "memory");
  };

  if (warp == 8) {
    // ================================================================ MMA issuer
    if (lane == 0 && nchunks > 0) {
      constexpr uint32_t I64N = idesc_bf16(64, 64, 1), I192N = idesc_bf16(64, 192, 1), I64K = idesc_bf16(64, 64),
                         IH = idesc_bf16(128, 64, 1, 1);
      uint32_t last_bar = 0, last_ph = 0;  // the last commit issued and its phase
      auto issue_a = [&](int c) {  // u = A vb, w = A kb (doneA: the w epilogue starts), then q k^T of chunk c (doneQ)
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)  // [w | u] = A [kb | vb]: columns 0..127 w, 128..191 u
          mma_bf16_ss(tmem + HT_W, ht_kdesc(at(c), kk), ht_mndesc(kbt(c), kk), I192N, kk > 0);
        mma_commit(doneA);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) mma_bf16_ss(tmem + HT_AQ, ht_kdesc(qt(c), kk), ht_kdesc(krt(c), kk), I64K, kk > 0);
        mma_commit(doneQ);
        last_bar = doneQ;
        last_ph = (uint32_t)c & 1u;
      };
      bool ok = mbar_wait(rdyA, 0, &S.abort, ST_TIMEOUT_HOWU);
      if (ok) {
        tc_fence_after();
        issue_a(0);
      }
      for (int c = 0; c < nchunks && ok; ++c) {
        const uint32_t ph = (uint32_t)c & 1u;
        // B(c): q Hb, w Hb
        if (!(ok = mbar_wait(rdyB, ph, &S.abort, ST_TIMEOUT_HOWU))) break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          mma_bf16_ss(tmem + HT_VW, ht_kdesc(sw, kk), ht_mndesc(shb, kk), I64N, kk > 0);
          mma_bf16_ss(tmem + HT_OI, ht_kdesc(qt(c), kk), ht_mndesc(shb, kk), I64N, kk > 0);
        }
        mma_commit(doneB);
        last_bar = doneB;
        last_ph = ph;
        // C(c): Aq vn; h += k^T vdec (k as the MN-major A operand: M = 128 key dims, K = 64 tokens)
        if (!(ok = mbar_wait(rdyC, ph, &S.abort, ST_TIMEOUT_HOWU))) break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          mma_bf16_ss(tmem + HT_H, ht_mndesc(krt(c), kk), ht_mndesc(svd, kk), IH, (c > 0 || kk > 0) ? 1u : 0u);
          mma_bf16_ss(tmem + HT_CI, ht_kdesc(saq, kk), ht_mndesc(svn, kk), I64N, kk > 0);
        }
        mma_commit(doneC);
        last_bar = doneC;
        // A(c+1)
        if (c + 1 < nchunks) {
          if (!(ok = mbar_wait(rdyA, ph ^ 1u, &S.abort, ST_TIMEOUT_HOWU))) break;
          tc_fence_after();
          issue_a(c + 1);
        }
      }
      // every MMA issued has completed before the TMEM is released (bounded: after a give-up it may never)
      if (last_bar) {
        const long long tw = clock64();
        while (!mbar_try_wait(last_bar, last_ph) && clock64() - tw < REAX_DRAIN_LIMIT) {
        }
      }
    }
  } else if (warp >= 9) {
    // ================================================================ helpers (warps 9-16, 256 threads)
    const int hid = tid - 288, hh = (warp - 9) >> 2;  // helper index; column half of its epilogue work
    auto wait_all = [&](uint32_t b, uint32_t parity) {
      return named_bar_and<2, 256>(mbar_wait(b, parity, &S.abort, ST_TIMEOUT_HOWU));
    };
    // chunk c's q, raw k, v (this slice's 64 columns), A (zero where SKIPA skips it) into its parity's tiles, rows past
    // the chunk zero-filled.  Thread hid owns a fixed 16-byte column and rows of one residue mod 8 (q, k: column
    // hid % 16, rows hid / 16 + 16e; v, A: column hid % 8, rows hid / 8 + 32e), so the swizzled offsets are fixed.
    const int qc = hid & 15, qr = hid >> 4, vc = hid & 7, vr = hid >> 3;
    const uint32_t q_off = (uint32_t)((qc >> 3) * 8192 + qr * 128 + (((qc & 7) ^ (qr & 7)) << 4));
    const uint32_t v_off = (uint32_t)(vr * 128 + ((vc ^ (vr & 7)) << 4));
    const long long qstride = 16LL * H * 128, vstride = 32LL * HV * 128, astride = 32LL * HV * 64;
    auto copy_chunk = [&](int c) {
      const long long tok0 = bos + 64LL * c;
      const int nv = (int)min(64LL, T - 64LL * c);
      const uint16_t* qs = q + ((tok0 + qr) * H + kh) * 128 + 8 * qc;
      const uint16_t* ks = k + ((tok0 + qr) * H + kh) * 128 + 8 * qc;
      const uint32_t qd0 = qt(c) + q_off, kd0 = krt(c) + q_off;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const bool ok = qr + 16 * e < nv;
        cp_async16(qd0 + 2048u * e, ok ? qs + qstride * e : q, ok);
        cp_async16(kd0 + 2048u * e, ok ? ks + qstride * e : k, ok);
      }
      const uint16_t* vs = v + ((tok0 + vr) * HV + hv) * 128 + c_lo + 8 * vc;
      const uint16_t* as = Ag + ((tok0 + vr) * HV + hv) * 64 + 8 * vc;
      const uint32_t vd0 = vt(c) + v_off, ad0 = at(c) + v_off;
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int r = vr + 32 * e;
        const bool ok = r < nv;
        cp_async16(vd0 + 4096u * e, ok ? vs + vstride * e : v, ok);
        const bool oka = ok && !(SKIPA && (vc >> 1) > (r >> 4));
        cp_async16(ad0 + 4096u * e, oka ? as + astride * e : Ag, oka);
      }
      cp_async_commit();
    };
    // once chunk c's copies have landed: its scalars, vb = bf16(beta v) in place and kb = bf16(bf16(beta k) 2^g);
    // then rdyA
    auto prepare = [&](int c) {
      const int nv = (int)min(64LL, T - 64LL * c), p = c & 1;
      if (hid < 64) {
        const long long tok = bos + 64LL * c + min(hid, nv - 1);
        const float g0 = g[tok * HV + hv];
        const uint16_t b0 = beta[tok * HV + hv];
        const float gv = hid < nv ? g0 : 0.f;
        S.g[p][hid] = gv;
        S.eg[p][hid] = exp2f(gv);
        S.beta[p][hid] = hid < nv ? __uint_as_float((uint32_t)b0 << 16) : 0.f;
        if (SCATTER) S.f2s[p][hid] = hid < nv ? f2s[bos + 64LL * c + hid] : -1;
      }
      cp_async_wait<0>();
      named_bar_sync<2, 256>();  // every helper's copies and scalars are visible
      if (hid < 64) S.da[p][hid] = hid < nv ? exp2f(S.g[p][nv - 1] - S.g[p][hid]) : 0.f;
      const uint32_t kr = krt(c), kb = kbt(c), vv = vt(c);
#pragma unroll
      for (int e = 0; e < 6; ++e) {
        const int id = hid + 256 * e;  // 0..511 v chunks, 512..1535 k chunks
        const bool isv = id < 512;
        const int j = isv ? id : id - 512, r = isv ? (j >> 3) : (j >> 4), cc = isv ? (j & 7) : (j & 15);
        const uint32_t off = (uint32_t)((cc >> 3) * 8192 + r * 128 + (((cc & 7) ^ (r & 7)) << 4));
        const float b = S.beta[p][r];
        uint4 x = ld_shared_v4((isv ? vv : kr) + off);
        uint32_t* xp = reinterpret_cast<uint32_t*>(&x);
        if (isv) {
#pragma unroll
          for (int i = 0; i < 4; ++i) xp[i] = pack_bf16(bf_lo(xp[i]) * b, bf_hi(xp[i]) * b);
          st_shared_v4(vv + off, x);
        } else {
          const float eg = S.eg[p][r];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const uint32_t t = pack_bf16(bf_lo(xp[i]) * b, bf_hi(xp[i]) * b);
            xp[i] = pack_bf16(bf_lo(t) * eg, bf_hi(t) * eg);
          }
          st_shared_v4(kb + off, x);
        }
      }
      fence_proxy_async_smem();
      mbar_arrive(rdyA);
    };

    if (nchunks > 0) {
      copy_chunk(0);
      prepare(0);
      if (nchunks > 1) copy_chunk(1);  // chunk 1's tiles are untouched so far
    }
    for (int c = 0; c < nchunks; ++c) {
      const uint32_t ph = (uint32_t)c & 1u;
      // chunk c + 1's tiles were last read by chunk c - 1's MMA groups, all complete once C(c - 1) is
      if (c >= 1 && c + 1 < nchunks) {
        if (!wait_all(doneC, ph ^ 1u)) break;
        copy_chunk(c + 1);
      }
      // ---- A(c) complete: w -> bf16 operand tile (rdyB)
      if (!wait_all(doneA, ph)) break;
      tc_fence_after();
#pragma unroll
      for (int hc = 0; hc < 4; ++hc) {
        const int cb = 64 * hh + 16 * hc;
        float x[8];
        ld64(HT_W + cb, x);
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) {
          const int c0 = cb + 8 * nt + 2 * tq;
          st_pair(sw, ra, c0, x[4 * nt], x[4 * nt + 1]);
          st_pair(sw, rb, c0, x[4 * nt + 2], x[4 * nt + 3]);
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(rdyB);
      // ---- the next chunk's derived operands, once the chain warps are past chunk c - 1 (whose scalars share the
      // parity): rdyB of chunk c complete
      if (c + 1 < nchunks) {
        if (!wait_all(rdyB, ph)) break;
        prepare(c + 1);
      }
    }
    cp_async_wait<0>();
  } else {
    // ================================================================ chain warps (0-7, 256 threads)
    const int hh = warp >> 2;  // column half
    auto wait_all = [&](uint32_t b, uint32_t parity) {
      return named_bar_and<1, 256>(mbar_wait(b, parity, &S.abort, ST_TIMEOUT_HOWU));
    };
    // Hb = 0 for the first chunk
    for (int i = tid; i < 16384 / 16; i += 256) st_shared_v4(shb + 16u * i, make_uint4(0, 0, 0, 0));
    fence_proxy_async_smem();
    if (nchunks > 0) mbar_arrive(rdyB);
    for (int c = 0; c < nchunks; ++c) {
      const uint32_t ph = (uint32_t)c & 1u;
      const long long t0 = 64LL * c;
      const int nval = (int)min(64LL, T - t0), p = c & 1;
      const bool more = c + 1 < nchunks;
      // 2^(g_last) of the next chunk, for the rescale of h after this chunk (loaded now, used at the end)
      float gnext = 0.f;
      if (more) gnext = g[(bos + t0 + 64 + min(64LL, T - t0 - 64) - 1) * HV + hv];
      // ---- Aq = bf16((q k^T) 2^(g_t - g_s)) on and below the diagonal (valid rows and keys), else 0
      if (!wait_all(doneQ, ph)) break;
      tc_fence_after();
      {
        const float gA = S.g[p][ra], gB = S.g[p][rb];
#pragma unroll
        for (int hc = 0; hc < 2; ++hc) {
          const int cb = 32 * hh + 16 * hc;
          if (cb > 16 * qd + 15) {  // 16x16 tile above the diagonal: zero (warp-uniform)
#pragma unroll
            for (int nt = 0; nt < 2; ++nt) {
              st_pair(saq, ra, cb + 8 * nt + 2 * tq, 0.f, 0.f);
              st_pair(saq, rb, cb + 8 * nt + 2 * tq, 0.f, 0.f);
            }
            continue;
          }
          float x[8];
          ld64(HT_AQ + cb, x);
#pragma unroll
          for (int nt = 0; nt < 2; ++nt) {
            const int s0 = cb + 8 * nt + 2 * tq;
            float y[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const int t = e < 2 ? ra : rb, s = s0 + (e & 1);
              y[e] = (s <= t && t < nval && s < nval) ? x[4 * nt + e] * exp2f((e < 2 ? gA : gB) - S.g[p][s]) : 0.f;
            }
            st_pair(saq, ra, s0, y[0], y[1]);
            st_pair(saq, rb, s0, y[2], y[3]);
          }
        }
      }
      // ---- S5: x = bf16(u) - w Hb -> vn = bf16(x), vdec = bf16(x 2^(g_last - g_t))  (A(c) precedes B(c))
      if (!wait_all(doneB, ph)) break;
      tc_fence_after();
      {
        const float da = S.da[p][ra], db = S.da[p][rb];
#pragma unroll
        for (int hc = 0; hc < 2; ++hc) {
          const int cb = 32 * hh + 16 * hc;
          float u[8], x[8];
          ld64(HT_U + cb, u);
          ld64(HT_VW + cb, x);
#pragma unroll
          for (int nt = 0; nt < 2; ++nt) {
            const int c0 = cb + 8 * nt + 2 * tq;
            const uint32_t u0 = pack_bf16(u[4 * nt], u[4 * nt + 1]), u1 = pack_bf16(u[4 * nt + 2], u[4 * nt + 3]);
            const float x0 = bf_lo(u0) - x[4 * nt], x1 = bf_hi(u0) - x[4 * nt + 1];
            const float x2 = bf_lo(u1) - x[4 * nt + 2], x3 = bf_hi(u1) - x[4 * nt + 3];
            st_pair(svn, ra, c0, x0, x1);
            st_pair(svn, rb, c0, x2, x3);
            st_pair(svd, ra, c0, x0 * da, x1 * da);
            st_pair(svd, rb, c0, x2 * db, x3 * db);
          }
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(rdyC);
      // ---- S7: o = bf16(scale (Aq vn) + scale 2^g (q Hb)) -> staging tile -> global; Hb = bf16(h); h *= 2^(g_last)
      // of the next chunk
      if (!wait_all(doneC, ph)) break;
      tc_fence_after();
      {
        const float ea = S.eg[p][ra], eb = S.eg[p][rb];
#pragma unroll
        for (int hc = 0; hc < 2; ++hc) {
          const int cb = 32 * hh + 16 * hc;
          float x[8], y[8];
          ld64(HT_CI + cb, x);
          ld64(HT_OI + cb, y);
#pragma unroll
          for (int nt = 0; nt < 2; ++nt) {
            const int c0 = cb + 8 * nt + 2 * tq;
            float r[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) r[e] = __fmaf_rn(x[4 * nt + e], scale, (y[4 * nt + e] * (e < 2 ? ea : eb)) * scale);
            st_pair(sost, ra, c0, r[0], r[1]);
            st_pair(sost, rb, c0, r[2], r[3]);
          }
        }
        uint32_t r[32];
        ht_ld32(tmem + tq_lane + HT_H + 32 * hh, r);
        const int d = 32 * qd + lane;  // key dim of this thread's TMEM lane
#pragma unroll
        for (int c4 = 0; c4 < 4; ++c4) {
          uint4 wv;
          wv.x = pack_bf16(__uint_as_float(r[8 * c4]), __uint_as_float(r[8 * c4 + 1]));
          wv.y = pack_bf16(__uint_as_float(r[8 * c4 + 2]), __uint_as_float(r[8 * c4 + 3]));
          wv.z = pack_bf16(__uint_as_float(r[8 * c4 + 4]), __uint_as_float(r[8 * c4 + 5]));
          wv.w = pack_bf16(__uint_as_float(r[8 * c4 + 6]), __uint_as_float(r[8 * c4 + 7]));
          st_shared_v4(shb + ht_off(d, 32 * hh + 8 * c4), wv);
        }
        if (more) {
          const float gl = exp2f(gnext);
#pragma unroll
          for (int e = 0; e < 32; ++e) r[e] = __float_as_uint(__uint_as_float(r[e]) * gl);
          tmem_st32_nowait(tmem + tq_lane + HT_H + 32 * hh, r);
          tmem_wait_st();
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      if (more) mbar_arrive(rdyB);  // the next chunk's Hb is ready and h rescaled
      named_bar_sync<1, 256>();      // the staging tile is complete
      // o rows < nval: 64 rows x 8 chunks of 16 bytes
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int id = tid + 256 * e, r = id >> 3, c8 = id & 7;
        const long long orow = SCATTER ? (long long)S.f2s[p][r] : bos + t0 + r;
        if (r < nval && orow >= 0)
          *reinterpret_cast<uint4*>(o + (orow * HV + hv) * 128 + c_lo + 8 * c8) =
              ld_shared_v4(sost + (uint32_t)(r * 128 + ((c8 ^ (r & 7)) << 4)));
      }
    }
  }

  // ---- teardown
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// Second pass of the norm entry point (libreax_howu/reax_howu_norm_v3.cu:347-374), in place on the rows the first pass
// scattered: out[f2s[t]][hv] = bf16( bf16(nw * bf16(o * rsqrt(sum(o^2) factor + eps))) * silu(z) ), with o the bf16
// row already in out.  A warp per token: one f2s load, then the token's heads 8 rows at a time (each lane holds 4
// values of 8 rows of o and of z: 16 loads in flight per lane), so the HBM stream is not broken by a dependent f2s load
// per row.  The sum of squares keeps the reference's order: per lane (x0^2 + x1^2) + x2^2 + x3^2 without contraction,
// then the shuffle tree over offsets 16, 8, 4, 2, 1 (every lane ends with lane 0's value).  The gate z is a bf16 input,
// so silu(z) -- the reference's fp32 quotient z / (1 + expf(-z)) with IEEE division -- is read from gtab, a table of
// that exact value for all 65536 bf16 patterns (gate_table.cuh); the values
// that occur sit in a few KB of it, which stay in L1 (this kernel uses no shared memory).  The token count is read
// from cu[N] on the device (the entry point does not pass it), so the grid strides over tokens.
constexpr int GN_ROWS = 8;  // heads a warp has in flight at once
__global__ void __launch_bounds__(256)
howu_gnorm_kernel(uint16_t* __restrict__ out, const int* __restrict__ f2s, const uint16_t* __restrict__ zg, long long ZS,
                  const uint16_t* __restrict__ nw, float eps, float factor, const long long* __restrict__ cu, int N,
                  int HV, const float* __restrict__ gtab) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const long long t_lo = cu[0], t_hi = cu[N];
  const uint2 wv = __ldg(reinterpret_cast<const uint2*>(nw + 4 * lane));
  const float wn[4] = {bf_lo(wv.x), bf_hi(wv.x), bf_lo(wv.y), bf_hi(wv.y)};
  for (long long t = t_lo + (long long)blockIdx.x * 8 + warp; t < t_hi; t += (long long)gridDim.x * 8) {
    const int sr = f2s[t];
    if (sr < 0) continue;  // warp-uniform
    uint16_t* orow = out + (long long)sr * HV * 128 + 4 * lane;
    const uint16_t* zrow = zg + (long long)sr * ZS + 4 * lane;
    for (int h0 = 0; h0 < HV; h0 += GN_ROWS) {
      uint2 xv[GN_ROWS], zv[GN_ROWS];
#pragma unroll
      for (int i = 0; i < GN_ROWS; ++i) {
        if (h0 + i < HV) {
          xv[i] = *reinterpret_cast<const uint2*>(orow + (long long)(h0 + i) * 128);
          zv[i] = __ldg(reinterpret_cast<const uint2*>(zrow + (long long)(h0 + i) * 128));
        }
      }
#pragma unroll
      for (int i = 0; i < GN_ROWS; ++i) {
        if (h0 + i >= HV) break;  // warp-uniform
        const float x[4] = {bf_lo(xv[i].x), bf_hi(xv[i].x), bf_lo(xv[i].y), bf_hi(xv[i].y)};
        float ss = __fadd_rn(__fadd_rn(__fadd_rn(__fmul_rn(x[0], x[0]), __fmul_rn(x[1], x[1])), __fmul_rn(x[2], x[2])),
                             __fmul_rn(x[3], x[3]));
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, off));
        const float rr = rsqrtf(__fadd_rn(__fmul_rn(ss, factor), eps));
        const uint32_t y01 = pack_bf16(__fmul_rn(x[0], rr), __fmul_rn(x[1], rr));
        const uint32_t y23 = pack_bf16(__fmul_rn(x[2], rr), __fmul_rn(x[3], rr));
        const uint32_t w01 = pack_bf16(__fmul_rn(wn[0], bf_lo(y01)), __fmul_rn(wn[1], bf_hi(y01)));
        const uint32_t w23 = pack_bf16(__fmul_rn(wn[2], bf_lo(y23)), __fmul_rn(wn[3], bf_hi(y23)));
        const uint32_t r01 = pack_bf16(__fmul_rn(bf_lo(w01), __ldg(gtab + (zv[i].x & 0xffffu))),
                                       __fmul_rn(bf_hi(w01), __ldg(gtab + (zv[i].x >> 16))));
        const uint32_t r23 = pack_bf16(__fmul_rn(bf_lo(w23), __ldg(gtab + (zv[i].y & 0xffffu))),
                                       __fmul_rn(bf_hi(w23), __ldg(gtab + (zv[i].y >> 16))));
        *reinterpret_cast<uint2*>(orow + (long long)(h0 + i) * 128) = make_uint2(r01, r23);
      }
    }
  }
}

}  // namespace reax

namespace reax_host {
template <bool SKIPA, bool SCATTER>
inline int howu_tc_launch(const void* q, const void* k, const void* v, const void* beta, const void* A, const void* g,
                          void* o, const void* cu, float scale, int N, int H, int HV, void* stream,
                          const void* f2s = nullptr) {
  static SmemAttr attr;
  if (N <= 0 || HV <= 0) return 0;
  if (H <= 0 || HV % H) return -1;
  if ((((uintptr_t)q | (uintptr_t)k | (uintptr_t)v | (uintptr_t)A | (uintptr_t)o) & 15)) return -1;
  if (2LL * N * HV > 0x7fffffffLL) return -1;
  if (ensure_smem(attr, reax::howu_tc_kernel<SKIPA, SCATTER>, reax::kHowuTcSmemBytes) != cudaSuccess)
    return (int)cudaErrorInvalidValue;
  reax::howu_tc_kernel<SKIPA, SCATTER><<<2 * N * HV, 544, reax::kHowuTcSmemBytes, (cudaStream_t)stream>>>(
      (const uint16_t*)q, (const uint16_t*)k, (const uint16_t*)v, (const uint16_t*)beta, (const uint16_t*)A,
      (const float*)g, (uint16_t*)o, (const long long*)cu, scale, N, H, HV, (const int*)f2s);
  return (int)cudaGetLastError();
}

// reax_howu_norm: the delta rule with its output rows scattered to out[f2s[t]] (bf16 o), then the gated RMSNorm in
// place on those rows.  f2s is a scatter index: two tokens with the same non-negative f2s would race in the reference
// and would be normalised twice here.
inline int howu_norm_tc_launch(const void* q, const void* k, const void* v, const void* beta, const void* A,
                               const void* g, void* out, const void* cu, float scale, int N, int H, int HV, void* stream,
                               const void* f2s, const void* z, long long ZS, const void* nw, float eps, float factor) {
  if (N <= 0 || HV <= 0) return 0;
  if (!f2s || !z || !nw || (((uintptr_t)z | (uintptr_t)nw) & 7) || ZS % 4) return -1;
  const float* gtab = gate_table((cudaStream_t)stream);
  if (gtab == nullptr) return -2;
  const int rc = howu_tc_launch<true, true>(q, k, v, beta, A, g, out, cu, scale, N, H, HV, stream, f2s);
  if (rc) return rc;
  int dev = 0;
  cudaGetDevice(&dev);
  reax::howu_gnorm_kernel<<<8 * device_sms(dev), 256, 0, (cudaStream_t)stream>>>(
      (uint16_t*)out, (const int*)f2s, (const uint16_t*)z, ZS, (const uint16_t*)nw, eps, factor, (const long long*)cu, N,
      HV, gtab);
  return (int)cudaGetLastError();
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
