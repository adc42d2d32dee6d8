// reax_oracle.cpp -- TEST INFRASTRUCTURE, not product code.
//
// fp64 CPU restatement of the REAX engine kernel set, written from the semantics of the reference .cu sources
// (each function cites the reference lines it follows).  Long reductions (dot products, sums of squares,
// softmax sums, the chunk recurrence) run in double precision; every rounding point the reference makes
// explicit (bf16 storage of intermediates, fp32 partial storage) is kept, because those roundings are part of
// the computed function.  Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg use this
// library, and only as the checker.
//
// Parity of this restatement is pinned against the reference kernels themselves: tests/golden/ holds outputs of
// the reference sources compiled for sm_100a (oracle/_ref) and run on a B200, and the CPU test suite checks
// this oracle against them.
//
// All tensors are host arrays; bf16 values are uint16_t bit patterns.  Work is split over `oracle_threads`
// std::threads (oracle_set_threads, default: all hardware threads).
#include <math.h>
#include <stdint.h>
#include <string.h>

#include <algorithm>
#include <atomic>
#include <functional>
#include <thread>
#include <vector>

#define ORACLE_API extern "C" __attribute__((visibility("default")))

namespace {

int g_threads = 0;

int nthreads() {
  if (g_threads > 0) return g_threads;
  unsigned h = std::thread::hardware_concurrency();
  return h ? (int)h : 1;
}

// dynamic parallel loop over [0, n)
void parallel_for(long long n, const std::function<void(long long)>& fn) {
  const int nt = (int)std::min<long long>(nthreads(), std::max<long long>(n, 1));
  if (nt <= 1) {
    for (long long i = 0; i < n; ++i) fn(i);
    return;
  }
  std::atomic<long long> next(0);
  std::vector<std::thread> th;
  for (int t = 0; t < nt; ++t)
    th.emplace_back([&] {
      for (;;) {
        const long long i = next.fetch_add(1);
        if (i >= n) break;
        fn(i);
      }
    });
  for (auto& x : th) x.join();
}

inline float bf2f(uint16_t b) {
  uint32_t u = (uint32_t)b << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}
// round-to-nearest-even float -> bf16 (NaN kept quiet)
inline uint16_t f2bf(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40);
  u += 0x7fffu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}
// double -> bf16 with a single rounding (round to nearest even on the exact value).  Rounding to float first
// is exact enough unless the float lands exactly on a bf16 midpoint that d itself is not on; then the side
// of the midpoint d lies on decides.
inline uint16_t d2bf(double d) {
  if (d != d) return 0x7fc0;
  const float f = (float)d;
  uint32_t u;
  memcpy(&u, &f, 4);
  if ((u & 0xffffu) == 0x8000u && (double)f != d) {
    const uint16_t lo = (uint16_t)(u >> 16);  // truncated magnitude, same sign
    return fabs(d) > fabs((double)f) ? (uint16_t)(lo + 1) : lo;
  }
  return f2bf(f);
}
inline float bfr(float x) { return bf2f(f2bf(x)); }
inline double bfd(double x) { return (double)bf2f(d2bf(x)); }

double dot_bf16(const uint16_t* a, const uint16_t* b, long long n) {
  double s = 0.0;
  for (long long k = 0; k < n; ++k) s += (double)bf2f(a[k]) * (double)bf2f(b[k]);
  return s;
}
double dot_f(const float* a, const float* b, long long n) {
  double s0 = 0, s1 = 0, s2 = 0, s3 = 0;
  long long k = 0;
  for (; k + 4 <= n; k += 4) {
    s0 += (double)a[k] * (double)b[k];
    s1 += (double)a[k + 1] * (double)b[k + 1];
    s2 += (double)a[k + 2] * (double)b[k + 2];
    s3 += (double)a[k + 3] * (double)b[k + 3];
  }
  for (; k < n; ++k) s0 += (double)a[k] * (double)b[k];
  return (s0 + s1) + (s2 + s3);
}
void to_float(const uint16_t* src, float* dst, long long n) {
  for (long long i = 0; i < n; ++i) dst[i] = bf2f(src[i]);
}

inline double silu_d(double g) { return g / (1.0 + exp(-g)); }

}  // namespace

ORACLE_API void oracle_set_threads(int n) { g_threads = n; }
ORACLE_API int oracle_threads() { return nthreads(); }

// ------------------------------------------------------------------------------------------------
// gate/up GEMM + SiLU*mul -- libreax_gv/gateup_vis2.cu:1-7 (math), :54-68 (epilogue), :182 (layouts)
//   G = sum_k x[m,k] w[8j+i,k], U = sum_k x[m,k] w[8j+4+i,k]; g = bf16(G), u = bf16(U);
//   out[m, 4j+i] = bf16( bf16(silu(g)) * u )
// The bf16 roundings of G and U depend on where the exact sum falls; any fp32 accumulation (the reference's
// mma.sync chain, a tcgen05 MMA) can land on the other side of a bf16 rounding boundary when the exact value is
// within its accumulation error of it, and silu amplifies that for large |g|.  When lo/hi are given they
// receive the smallest / largest output over the roundings of G and U reachable within +-band*sum_k|x w|
// (the test suite passes band = 2^-19, a safe bound on fp32 accumulation of these sizes) and over both roundings of silu(g) reachable
// within a relative 2^-20 (an fp32 expf + division lands within a few fp32 ulps of the exact value); elsewhere
// lo = hi = out.
// Rows [m0, m1) only, so a bounded sample of a large problem can be timed.
// ------------------------------------------------------------------------------------------------
ORACLE_API void oracle_gv_rows(const uint16_t* x, const uint16_t* w, uint16_t* out, uint16_t* lo, uint16_t* hi, int M,
                               int N2, int K, int m0, int m1, double band) {
  (void)M;
  const int rows = m1 - m0;
  if (rows <= 0 || N2 <= 0) return;
  std::vector<float> xf((size_t)rows * K), xa((size_t)rows * K);
  to_float(x + (size_t)m0 * K, xf.data(), (long long)rows * K);
  for (size_t i = 0; i < xf.size(); ++i) xa[i] = fabsf(xf[i]);
  const int ngroups = N2 / 4;
  auto f = [](double g, double u) { return (double)bf2f(d2bf((double)bf2f(d2bf(silu_d(g))) * u)); };
  // one task per 4-feature group: its 8 weight rows are converted once and reused for every row
  parallel_for(ngroups, [&](long long j) {
    std::vector<float> wf((size_t)8 * K), wa((size_t)8 * K);
    to_float(w + (size_t)j * 8 * K, wf.data(), 8LL * K);
    for (size_t i = 0; i < wf.size(); ++i) wa[i] = fabsf(wf[i]);
    for (int r = 0; r < rows; ++r) {
      const float* xr = xf.data() + (size_t)r * K;
      for (int i = 0; i < 4; ++i) {
        const double G = dot_f(xr, wf.data() + (size_t)i * K, K);
        const double U = dot_f(xr, wf.data() + (size_t)(4 + i) * K, K);
        const double g = bf2f(d2bf(G)), u = bf2f(d2bf(U));
        const size_t o = (size_t)(m0 + r) * N2 + 4 * j + i;
        const double y = f(g, u);
        out[o] = d2bf(y);
        if (lo && hi) {
          const float* xar = xa.data() + (size_t)r * K;
          const double dg = band * dot_f(xar, wa.data() + (size_t)i * K, K);
          const double du = band * dot_f(xar, wa.data() + (size_t)(4 + i) * K, K);
          const double gs[2] = {bf2f(d2bf(G - dg)), bf2f(d2bf(G + dg))};
          const double us[2] = {bf2f(d2bf(U - du)), bf2f(d2bf(U + du))};
          double mn = y, mx = y;
          for (double gg : gs)
            for (double uu : us)
              for (double e : {1.0 - 0x1p-20, 1.0 + 0x1p-20}) {
                const double sg = (double)bf2f(d2bf(silu_d(gg) * e));
                const double c = (double)bf2f(d2bf(sg * uu));
                mn = std::min(mn, c);
                mx = std::max(mx, c);
              }
          lo[o] = d2bf(mn);
          hi[o] = d2bf(mx);
        }
      }
    }
  });
}
ORACLE_API void oracle_gv(const uint16_t* x, const uint16_t* w, uint16_t* out, int M, int N2, int K) {
  oracle_gv_rows(x, w, out, nullptr, nullptr, M, N2, K, 0, M, 0.0);
}

// ------------------------------------------------------------------------------------------------
// plain GEMM -- libreax_plain/gemm_plain2.cu:1-3, :21-23:  D[m, n] (ld ldd) = bf16( sum_k X[m,k] W[n,k] )
// ------------------------------------------------------------------------------------------------
ORACLE_API void oracle_gemm(const uint16_t* x, const uint16_t* w, uint16_t* d, int M, int N, int K, int ldd) {
  parallel_for(M, [&](long long m) {
    for (int n = 0; n < N; ++n) d[(size_t)m * ldd + n] = d2bf(dot_bf16(x + (size_t)m * K, w + (size_t)n * K, K));
  });
}

// ------------------------------------------------------------------------------------------------
// sliced GEMM -- libreax_slices/gemm_slices_v2.cu:1-8, :26-28:
//   P[s][m, n] = sum_{k < kps} X[m, s*kps + k] W[n, s*kps + k], stored once as fp32 or bf16, P[s] at s*M*N
// ------------------------------------------------------------------------------------------------
ORACLE_API void oracle_slices(int part_fp32, const uint16_t* x, const uint16_t* w, void* p, int M, int N, int kps, int S,
                              int K) {
  parallel_for((long long)S * M, [&](long long sm) {
    const int s = (int)(sm / M), m = (int)(sm % M);
    for (int n = 0; n < N; ++n) {
      const double v = dot_bf16(x + (size_t)m * K + (size_t)s * kps, w + (size_t)n * K + (size_t)s * kps, kps);
      const size_t idx = ((size_t)s * M + m) * N + n;
      if (part_fp32)
        static_cast<float*>(p)[idx] = (float)v;
      else
        static_cast<uint16_t*>(p)[idx] = d2bf(v);
    }
  });
}

// ------------------------------------------------------------------------------------------------
// attention forward -- libreax_fmha_post/reax_fmha_v11.cu:6-13 (semantics), :204-221 (visibility), :295-450 (online
// softmax over 128-key blocks), :451-531 (epilogues), :583 (qp entry)
//   per row: x_j = (scale * Q.K_j + bias_j) * log2(e) for visible keys (qpos mode: j <= qpos[b*qpBs + r/G]; bias
//   mode: bf16 bias[b,h,r,j]); keys are consumed in blocks of 128 in order with the exact running max m (the max
//   over the visible keys of all blocks so far):  on a new max, l and O are scaled by 2^(m_old - m_new);
//   p_j = 2^(x_j - m);  l += p_j (unrounded);  O += bf16(p_j) * V_j.  The bf16 rounding of p before the P.V product
//   is a rounding point of the reference (its probabilities feed a bf16 tensor-core product), so it is kept here.
//   O = O / l (rows with no visible key: 0), stored as bf16 -- or, post (qpos mode): outp[R*out_rs + (h*G + r%G)*D + d]
//   = bf16(bf16(O) * bf16(sigmoid(gate))), R = inv[b*Lq + r/G] (skip R < 0), gate = qg[R*qg_rs + (h*G + r%G)*2D + D + d].
// Rows r in [r0, r1) only (a bounded sample for timing); r1 = M for the full problem.
// lo / hi (optional, same layout as the output): the interval of results reachable when a probability lies within
// a relative `band` of a bf16 rounding midpoint -- a GPU computes the scores with fp32 dot products whose last-bit
// differences (accumulation order) can put p on either side of such a midpoint, so both roundings are legitimate there.
// In post mode the interval also spans the two later rounding points, bf16(O) and bf16(sigmoid(gate)).
// ------------------------------------------------------------------------------------------------
ORACLE_API void oracle_fmha(int mode, int D, const uint16_t* q, const uint16_t* k, const uint16_t* v, const uint16_t* bias,
                            const int* qpos, int G, long long qpBs, uint16_t* o, float scale, int B, int H, int M, int N,
                            long long qsB, long long qsH, long long qsM, long long ksB, long long ksH, long long ksM,
                            long long vsB, long long vsH, long long vsM, long long bsB, long long bsH, long long bsM,
                            long long osB, long long osH, long long osM, int post, const int* inv, int Lq,
                            const uint16_t* qg, long long qg_rs, uint16_t* outp, long long out_rs, int r0, int r1,
                            uint16_t* lo, uint16_t* hi, double band) {
  const long long rows = (long long)B * H * (r1 - r0);
  const double LOG2E = 1.4426950408889634074;
  parallel_for(rows, [&](long long idx) {
    const int r = r0 + (int)(idx % (r1 - r0));
    const int h = (int)((idx / (r1 - r0)) % H);
    const int b = (int)(idx / ((long long)(r1 - r0) * H));
    const uint16_t* Q = q + b * qsB + h * qsH + (long long)r * qsM;
    std::vector<float> qf(D);
    for (int d = 0; d < D; ++d) qf[d] = bf2f(Q[d]);
    const int lim = mode == 1 ? qpos[(long long)b * qpBs + r / G] : N - 1;
    std::vector<double> acc(D, 0.0), x(128), dlo(D, 0.0), dhi(D, 0.0);
    double m = -INFINITY, l = 0.0;
    for (int k0 = 0; k0 < N; k0 += 128) {
      const int k1 = std::min(N, k0 + 128);
      double bm = -INFINITY;
      for (int j = k0; j < k1; ++j) {
        double s = -INFINITY;
        if (j <= lim) {
          const uint16_t* Kj = k + b * ksB + h * ksH + (long long)j * ksM;
          double a = 0;
          for (int d = 0; d < D; ++d) a += (double)qf[d] * (double)bf2f(Kj[d]);
          s = a * (double)scale;
          if (mode == 0) s += (double)bf2f(bias[b * bsB + h * bsH + (long long)r * bsM + j]);
          s *= LOG2E;
        }
        x[j - k0] = s;
        bm = std::max(bm, s);
      }
      if (bm > m) {
        const double alpha = m == -INFINITY ? 0.0 : exp2(m - bm);
        l *= alpha;
        for (int d = 0; d < D; ++d) {
          acc[d] *= alpha;
          dlo[d] *= alpha;
          dhi[d] *= alpha;
        }
        m = bm;
      }
      if (m == -INFINITY) continue;
      for (int j = k0; j < k1; ++j) {
        if (x[j - k0] == -INFINITY) continue;
        const double pj = exp2(x[j - k0] - m);
        l += pj;
        const double pb = bfd(pj);
        const uint16_t* Vj = v + b * vsB + h * vsH + (long long)j * vsM;
        for (int d = 0; d < D; ++d) acc[d] += pb * (double)bf2f(Vj[d]);
        if (lo) {
          const double p1 = bfd(pj * (1.0 - band)), p2 = bfd(pj * (1.0 + band));
          const double alt = p1 != pb ? p1 : p2;  // the other rounding, when p is that close to a midpoint
          if (alt != pb)
            for (int d = 0; d < D; ++d) {
              const double dv = (alt - pb) * (double)bf2f(Vj[d]);
              if (dv < 0) dlo[d] += dv; else dhi[d] += dv;
            }
        }
      }
    }
    if (post) {
      const int R = inv[(long long)b * Lq + r / G];
      if (R < 0) return;
      const long long hq = (long long)h * G + r % G;
      for (int d = 0; d < D; ++d) {
        const double gate = bf2f(qg[(long long)R * qg_rs + hq * 2 * D + D + d]);
        const double sg = bf2f(d2bf(1.0 / (1.0 + exp(-gate))));
        auto f = [&](double a) { return d2bf((double)bf2f(d2bf(l > 0 ? a / l : 0.0)) * sg); };
        const long long oi = (long long)R * out_rs + hq * D + d;
        outp[oi] = f(acc[d]);
        if (lo) {
          // two more rounding points follow P here: bf16(O) and bf16(sigmoid(gate)).  Where the exact O (over the
          // P interval) or the exact sigmoid lies within a relative `band` of a bf16 midpoint, a GPU computing them
          // in fp32 may round either way, and the product's own rounding follows; the interval takes every such
          // combination (away from midpoints both candidates coincide and this is the P interval alone).
          const double sig = 1.0 / (1.0 + exp(-gate));
          const double sgs[2] = {bf2f(d2bf(sig * (1.0 - band))), bf2f(d2bf(sig * (1.0 + band)))};
          double vlo = INFINITY, vhi = -INFINITY;
          uint16_t blo = 0, bhi = 0;
          for (const double a : {acc[d] + dlo[d], acc[d] + dhi[d]})
            for (const double e : {1.0 - band, 1.0 + band}) {
              const double ob = bf2f(d2bf(l > 0 ? a / l * e : 0.0));
              for (const double s : sgs) {
                const uint16_t c = d2bf(ob * s);
                const double cv = bf2f(c);
                if (cv < vlo) vlo = cv, blo = c;
                if (cv > vhi) vhi = cv, bhi = c;
              }
            }
          lo[oi] = blo;
          hi[oi] = bhi;
        }
      }
    } else {
      const long long ob = b * osB + h * osH + (long long)r * osM;
      for (int d = 0; d < D; ++d) {
        o[ob + d] = d2bf(l > 0 ? acc[d] / l : 0.0);
        if (lo) {
          lo[ob + d] = d2bf(l > 0 ? (acc[d] + dlo[d]) / l : 0.0);
          hi[ob + d] = d2bf(l > 0 ? (acc[d] + dhi[d]) / l : 0.0);
        }
      }
    }
  });
}

// ------------------------------------------------------------------------------------------------
// reduce + residual + RMSNorm -- libreax_howu/reax_rarn_final.cu:36-89
//   d = sum_s part[s] (serial: bf16 after the first term and after every add, else one bf16 rounding at the end)
//   h = bf16(res + d) -> h_out;  out = bf16( h * rsqrt(sum(h^2) * factor + eps) * (1 + w) )
// ------------------------------------------------------------------------------------------------
ORACLE_API void oracle_rarn(const uint16_t* part, int S, int serial, long long pstride, const uint16_t* res, const uint16_t* w,
                            uint16_t* h_out, uint16_t* out, int n, int D, float eps, float factor) {
  parallel_for(n, [&](long long row) {
    std::vector<double> h(D);
    double ss = 0;
    for (int c = 0; c < D; ++c) {
      const long long o = row * D + c;
      double d;
      if (serial) {
        float f = bf2f(part[o]);
        for (int s = 1; s < S; ++s) f = bfr(f + bf2f(part[s * pstride + o]));
        d = f;
      } else {
        double t = 0;
        for (int s = 0; s < S; ++s) t += (double)bf2f(part[s * pstride + o]);
        d = bfd(t);
      }
      h[c] = bfd((double)bf2f(res[o]) + d);
      h_out[o] = d2bf(h[c]);
      ss += h[c] * h[c];
    }
    const double r = 1.0 / sqrt(ss * (double)factor + (double)eps);
    for (int c = 0; c < D; ++c) out[row * D + c] = d2bf(h[c] * r * (1.0 + (double)bf2f(w[c])));
  });
}

// ------------------------------------------------------------------------------------------------
// depthwise causal conv + SiLU (+ L2 norm) -- libreax_howu/reax_conv_v2.cu:60-150, :164-189
//   tap j of token t (meta = pos, y, z, w): src = pos - 3 + j; skipped if src < 0; x = qkv[(z+src)*SX + c] if
//   src >= y else cache[(w+src)*C + c].  acc = sum_j wt[c][j] * x;  y = bf16(acc);  s = bf16(y / (1 + exp(-y))).
//   Units of 128 channels: u < KD/128 -> q, u < 2KD/128 -> k (both L2-normalised: s / sqrt(eps + sum s^2),
//   written rep times), else v (channels 2KD.., written when !skip_v).  units_lo/units_hi select a unit range
//   (reax_conv_v uses the value units only).
// ------------------------------------------------------------------------------------------------
ORACLE_API void oracle_conv(const uint16_t* qkv, long long SX, const uint16_t* cache, int C, const int* meta, const uint16_t* w,
                            uint16_t* q, uint16_t* k, uint16_t* v, int Tf, float eps, int KD, int VD, int rep, int skip_v,
                            int units_lo, int units_hi) {
  const int nqk = 2 * KD / 128;
  const int nunits = units_hi - units_lo;
  parallel_for((long long)Tf * nunits, [&](long long idx) {
    const int t = (int)(idx / nunits), u = units_lo + (int)(idx % nunits);
    if (u >= nqk && skip_v) return;
    const int* m = meta + (long long)t * 4;
    double s[128];
    for (int cc = 0; cc < 128; ++cc) {
      const int c = u * 128 + cc;
      double acc = 0;
      for (int j = 0; j < 4; ++j) {
        const int src = m[0] - 3 + j;
        if (src < 0) continue;
        const double x = src >= m[1] ? bf2f(qkv[(long long)(m[2] + src) * SX + c]) : bf2f(cache[(long long)(m[3] + src) * C + c]);
        acc += (double)bf2f(w[(long long)c * 4 + j]) * x;
      }
      const double y = bfd(acc);
      s[cc] = bfd(silu_d(y));
    }
    if (u < nqk) {
      double ss = 0;
      for (int cc = 0; cc < 128; ++cc) ss += s[cc] * s[cc];
      const double rstd = 1.0 / sqrt((double)eps + ss);
      const int nh = rep * KD / 128, hq = u % (KD / 128);
      uint16_t* dst = (u < KD / 128 ? q : k) + (long long)t * (nh * 128) + (long long)rep * hq * 128;
      for (int cc = 0; cc < 128; ++cc) {
        const uint16_t b = d2bf(s[cc] * rstd);
        dst[cc] = b;
        if (rep == 2) dst[128 + cc] = b;
      }
    } else {
      uint16_t* dst = v + (long long)t * VD + (u * 128 - 2 * KD);
      for (int cc = 0; cc < 128; ++cc) dst[cc] = d2bf(s[cc]);
    }
  });
}

// ------------------------------------------------------------------------------------------------
// chunked KKT + triangular inverse -- libreax_howu/reax_kkt.cu:85-104 (inputs), :133-159 (decay, mask, beta),
// :160-245 (inverse), :246-260 (write set)
//   per chunk (seq n, chunk c: tokens bos+64c .. +nval) and value head hv (key head hv/2):
//   L[r][s] = beta[r] * (k_r . k_s) * 2^(g[r] - g[s]) for s < r < nval;  A = (I + L)^-1 (exact, fp64);
//   written: rows r < nval, columns s < 16*(r/16 + 1) (16x16 blocks on and below the diagonal), as bf16.
// ------------------------------------------------------------------------------------------------
ORACLE_API void oracle_kkt(const uint16_t* k, const float* g, const uint16_t* beta, uint16_t* A, const long long* cu,
                           const long long* cidx, int NT, int H, int HV) {
  parallel_for((long long)NT * HV, [&](long long idx) {
    const int ci = (int)(idx / HV), hv = (int)(idx % HV);
    const int kh = hv / (HV / H);
    const long long i_n = cidx[2 * ci], i_t = cidx[2 * ci + 1];
    const long long bos = cu[i_n], T = cu[i_n + 1] - bos;
    const long long t0 = i_t * 64;
    const int nval = (int)std::min<long long>(64, T - t0);
    if (nval <= 0) return;
    double L[64][64] = {};
    for (int r = 0; r < nval; ++r) {
      const long long tr = bos + t0 + r;
      const double br = bf2f(beta[tr * HV + hv]);
      const double gr = g[tr * HV + hv];
      for (int s = 0; s < r; ++s) {
        const long long ts = bos + t0 + s;
        const double kk = dot_bf16(k + (tr * H + kh) * 128, k + (ts * H + kh) * 128, 128);
        L[r][s] = br * kk * exp2(gr - (double)g[ts * HV + hv]);
      }
    }
    // X = (I + L)^-1 by forward substitution, column by column
    double X[64][64] = {};
    for (int c = 0; c < nval; ++c) {
      X[c][c] = 1.0;
      for (int r = c + 1; r < nval; ++r) {
        double acc = 0;
        for (int s = c; s < r; ++s) acc += L[r][s] * X[s][c];
        X[r][c] = -acc;
      }
    }
    for (int r = 0; r < nval; ++r) {
      const int cols = 16 * (r / 16 + 1);
      uint16_t* row = A + ((bos + t0 + r) * HV + hv) * 64;
      for (int s = 0; s < cols; ++s) row[s] = d2bf(X[r][s]);
    }
  });
}

// ------------------------------------------------------------------------------------------------
// chunked gated delta rule (+ gated RMSNorm) -- libreax_howu/reax_howu.cu:124-347 (chunk recurrence, rounding
// points), libreax_howu/reax_howu_norm_v3.cu:347-374 (norm epilogue)
//   per (seq, value head hv; key head kh = hv / (HV/H)), chunk of nval <= 64 tokens, state h[128 k][128 v]:
//     vb = bf16(beta*v);  kb = bf16(bf16(beta*k) * 2^g);  u = bf16(A vb);  w = bf16(A kb)
//     Aq[t][s] = bf16( (q_t.k_s) * 2^(g_t - g_s) ) for s <= t (valid), else 0
//     H = bf16(h);  x = u - w H;  vn = bf16(x);  vdec = bf16(x * 2^(g_last - g_t))
//     o = bf16( scale * (Aq vn) + scale * 2^(g_t) * (q H) )
//     h = h * 2^(g_last) + k^T vdec
//   dense != 0 uses all of A's 64x64 block (its upper blocks as stored); otherwise only blocks j <= i.
//   norm != 0: out[f2s[t]][hv] = bf16( bf16(nw * bf16(o * rsqrt(sum(o^2)*factor + eps))) * silu(z) ),
//              z = zg[f2s[t]*ZS + hv*128 + :], rows with f2s < 0 skipped; else o[t][hv] = o.
// ------------------------------------------------------------------------------------------------
ORACLE_API void oracle_howu(const uint16_t* q, const uint16_t* k, const uint16_t* v, const uint16_t* beta, const uint16_t* Ag,
                            const float* g, uint16_t* o, const long long* cu, float scale, int N, int H, int HV, int dense,
                            int norm, const int* f2s, const uint16_t* zg, long long ZS, const uint16_t* nw, float eps,
                            float factor) {
  parallel_for((long long)N * HV, [&](long long idx) {
    const int n = (int)(idx / HV), hv = (int)(idx % HV);
    const int kh = hv / (HV / H);
    const long long bos = cu[n], T = cu[n + 1] - bos;
    std::vector<double> h(128 * 128, 0.0);
    std::vector<double> Hb(128 * 128);
    for (long long t0 = 0; t0 < T; t0 += 64) {
      const int nv = (int)std::min<long long>(64, T - t0);
      static thread_local double Av[64][64], vb[64][128], kb[64][128], uu[64][128], ww[64][128], aq[64][64], kr[64][128],
          qr[64][128], gg[64], xx[64][128], vn[64][128], vd[64][128];
      for (int r = 0; r < 64; ++r) {
        const bool ok = r < nv;
        const long long t = bos + t0 + r;
        gg[r] = ok ? (double)g[t * HV + hv] : 0.0;
        const double b = ok ? (double)bf2f(beta[t * HV + hv]) : 0.0;
        const double eg = exp2(gg[r]);
        for (int c = 0; c < 64; ++c) Av[r][c] = ok ? (double)bf2f(Ag[(t * HV + hv) * 64 + c]) : 0.0;
        for (int c = 0; c < 128; ++c) {
          const double vv = ok ? (double)bf2f(v[(t * HV + hv) * 128 + c]) : 0.0;
          kr[r][c] = ok ? (double)bf2f(k[(t * H + kh) * 128 + c]) : 0.0;
          qr[r][c] = ok ? (double)bf2f(q[(t * H + kh) * 128 + c]) : 0.0;
          vb[r][c] = bfd(b * vv);
          kb[r][c] = bfd(bfd(b * kr[r][c]) * eg);
        }
      }
      for (int r = 0; r < 64; ++r) {
        const int jmax = dense ? 64 : 16 * (r / 16 + 1);
        for (int c = 0; c < 128; ++c) {
          double su = 0, sw = 0;
          for (int s = 0; s < jmax; ++s) {
            su += Av[r][s] * vb[s][c];
            sw += Av[r][s] * kb[s][c];
          }
          uu[r][c] = bfd(su);
          ww[r][c] = bfd(sw);
        }
        for (int s = 0; s < 64; ++s) {
          double z = 0;
          if (s <= r && r < nv && s < nv) {
            double d = 0;
            for (int c = 0; c < 128; ++c) d += qr[r][c] * kr[s][c];
            z = bfd(d * exp2(gg[r] - gg[s]));
          }
          aq[r][s] = z;
        }
      }
      for (int i = 0; i < 128 * 128; ++i) Hb[i] = bfd(h[i]);
      const double glast = gg[nv - 1];
      for (int r = 0; r < 64; ++r) {
        const double da = r < nv ? exp2(glast - gg[r]) : 0.0;
        for (int c = 0; c < 128; ++c) {
          double vw = 0;
          for (int kk = 0; kk < 128; ++kk) vw += ww[r][kk] * Hb[kk * 128 + c];
          xx[r][c] = uu[r][c] - vw;
          vn[r][c] = bfd(xx[r][c]);
          vd[r][c] = bfd(xx[r][c] * da);
        }
      }
      // outputs of this chunk
      for (int r = 0; r < nv; ++r) {
        const long long t = bos + t0 + r;
        double orow[128];
        const double ea = exp2(gg[r]);
        for (int c = 0; c < 128; ++c) {
          double ci = 0, oi = 0;
          for (int s = 0; s <= r; ++s) ci += aq[r][s] * vn[s][c];
          for (int kk = 0; kk < 128; ++kk) oi += qr[r][kk] * Hb[kk * 128 + c];
          orow[c] = bfd(ci * scale + oi * ea * scale);
        }
        if (!norm) {
          for (int c = 0; c < 128; ++c) o[(t * HV + hv) * 128 + c] = d2bf(orow[c]);
        } else {
          const int sr = f2s[t];
          if (sr < 0) continue;
          double ss = 0;
          for (int c = 0; c < 128; ++c) ss += orow[c] * orow[c];
          const double rr = 1.0 / sqrt(ss * (double)factor + (double)eps);
          for (int c = 0; c < 128; ++c) {
            const double y = bfd(orow[c] * rr);
            const double y2 = bfd((double)bf2f(nw[c]) * y);
            const double z = bf2f(zg[(long long)sr * ZS + (long long)hv * 128 + c]);
            o[((long long)sr * HV + hv) * 128 + c] = d2bf(y2 * silu_d(z));
          }
        }
      }
      // state update
      const double gl = exp2(glast);
      for (int kk = 0; kk < 128; ++kk)
        for (int c = 0; c < 128; ++c) {
          double a = h[kk * 128 + c] * gl;
          for (int r = 0; r < 64; ++r) a += kr[r][kk] * vd[r][c];
          h[kk * 128 + c] = a;
        }
    }
  });
}
