/*
 * reax_abi.h -- the C ABI of the five REAX engine kernel libraries, built for B200 (sm_100a).
 *
 * Every entry point below keeps the exact name, argument order and argument meaning of the
 * sm_120 reference library it replaces, so an engine that dlopen()s libreax_*.so and binds these
 * symbols by name runs unchanged.  Each declaration cites the reference definition it replaces
 * (path inside the reference project : line).
 *
 * Conventions shared by every entry point (same as the reference):
 *   - all tensor pointers are caller-owned DEVICE pointers; the libraries allocate nothing;
 *   - `stream` is a cudaStream_t passed as void*; work is enqueued asynchronously on it;
 *   - the int return value reports argument-validation and launch errors only, never device
 *     completion: 0 = success, small positive / negative codes = validation failures (listed per
 *     function), any other value = a cudaError_t cast to int;
 *   - bf16 = IEEE bfloat16 stored as 16-bit words; "row-major [R, C]" means element (r, c) at r*C + c.
 *
 * Additions that do not exist in the reference are grouped at the end and marked EXTENSION.
 */
#ifndef REAX_ABI_H
#define REAX_ABI_H

#ifdef __cplusplus
extern "C" {
#endif

/* ======================= libreax_gv.so : gate/up GEMM with fused SiLU*mul ======================= */

/* Number of tile configurations accepted by reax_gv (20).      replaces libreax_gv/gateup_vis2.cu:172 */
int reax_gv_ncfg(void);
/* Name of configuration c, or "?" when c is out of range.      replaces libreax_gv/gateup_vis2.cu:173-181 */
const char* reax_gv_cfgname(int c);
/* out[m, 4j+i] = bf16( bf16(silu(bf16 G)) * bf16 U ),  G = sum_k x[m,k] w[8j+i,k],  U = sum_k x[m,k] w[8j+4+i,k]
 * x [M, K] row-major bf16; w [2*N2, K] row-major bf16 with gate/up rows interleaved in groups of 4;
 * out [M, N2] row-major bf16.  Returns 1 if K % 8 or N2 % 4, 9 for an unknown cfg, 3 on launch error.
 *                                                              replaces libreax_gv/gateup_vis2.cu:183-208 */
int reax_gv(int cfg, const void* x, const void* w, void* out, int M, int N2, int K, void* stream);
/* reax_gv for callers that cannot allocate device memory (an engine that reserves all GPU memory for its own arena,
 * a serving loop that cannot afford a cudaMalloc mid-step): the same computation and bits, with the split kernel's
 * scratch in a static ~20 MiB array that every GPU loading the library holds until exit; allocates nothing.
 * The array serves GPUs with at most 160 SMs (returns 5 on a larger one, launching nothing).  All calls share it:
 * calls that overlap on the GPU race.  The first call on a device sets up (symbol address, SiLU table, waiting on
 * `stream`); make it before any stream capture.  Other return codes as reax_gv.
 *                                                              no counterpart in the reference */
int reax_gv_noalloc(int cfg, const void* x, const void* w, void* out, int M, int N2, int K, void* stream);

/* ========================== libreax_plain.so : plain GEMM D = X W^T ============================= */

/* 15 configurations.                                           replaces libreax_plain/gemm_plain2.cu:32 */
int reax_gemm_ncfg(void);
/*                                                              replaces libreax_plain/gemm_plain2.cu:33-36 */
const char* reax_gemm_cfgname(int c);
/* D[M, N] (leading dimension ldd elements) = X[M, K] W[N, K]^T, fp32 accumulation, bf16 output.
 * Returns 1 when the shape/alignment is not implementable (K % 8, ldd < N), 9 for an unknown cfg,
 * 4 on launch error.                                           replaces libreax_plain/gemm_plain2.cu:20-29,37-57 */
int reax_gemm(int cfg, const void* x, const void* w, void* d, int M, int N, int K, int ldd, void* stream);

/* ====================== libreax_slices.so : split-K partials as one batched GEMM ================ */

/* 16 configurations (the SLICE_CFGS table).                    replaces libreax_slices/gemm_slices_v2.cu:56 */
int reax_slices_ncfg(void);
/*                                                              replaces libreax_slices/gemm_slices_v2.cu:57-64 */
const char* reax_slices_cfgname(int c);
/* P[s][m, n] = sum_{k in [s*kps, (s+1)*kps)} X[m, k] W[n, k]  for s < S, stored as fp32 (part_fp32 != 0)
 * or bf16; P[s] starts at p + s*M*N (elements), leading dimension N.  X [M, K], W [N, K] row-major.
 * Returns 1 when not implementable (K % 8, kps % 8, S*kps > K), 9 for an unknown cfg, 4 on launch error.
 *                                                              replaces libreax_slices/gemm_slices_v2.cu:25-34,65-84 */
int reax_slices(int cfg, int part_fp32, const void* x, const void* w, void* p, int M, int N, int kps, int S,
                int K, void* stream);

/* ============================ libreax_howu.so : linear-attention layer ========================== */

/* Chunked gated delta rule output (WY form, 64-token chunks), one program per (sequence, value head).
 * q, k [T][H][128] bf16; v, o [T][HV][128] bf16; beta [T][HV] bf16; A [T][HV][64] bf16 (from reax_kkt);
 * g [T][HV] fp32 (log2-domain chunk-local cumulative decay); cu [N+1] int64 sequence offsets.
 * howu3_dense reads the whole 64x64 A block (its never-written upper blocks must be zero);
 * howu3_skip and reax_howu read only the lower block triangle.
 *                                                              replaces libreax_howu/reax_howu.cu:363-376 */
int howu3_dense(const void* q, const void* k, const void* v, const void* beta, const void* A, const void* g,
                void* o, const void* cu, float scale, int N, int H, int HV, void* stream);
int howu3_skip(const void* q, const void* k, const void* v, const void* beta, const void* A, const void* g,
               void* o, const void* cu, float scale, int N, int H, int HV, void* stream);
/* Dynamic shared memory (bytes) one howu program uses.        replaces libreax_howu/reax_howu.cu:371 */
int howu3_smem(void);
int reax_howu(const void* q, const void* k, const void* v, const void* beta, const void* A, const void* g,
              void* o, const void* cu, float scale, int N, int H, int HV, void* stream);

/* Per 64-token chunk of each sequence and value head: A = (I + tril(beta_r (k_r . k_c) 2^(g_r - g_c), -1))^-1.
 * k [T][H][128] bf16, g [T][HV] fp32, beta [T][HV] bf16, A [T][HV][64] bf16, cu [N+1] int64,
 * cidx [NT][2] int64 = (sequence, chunk).  Only rows < chunk length and 16x16 blocks j <= i are written.
 * Returns -1 unless HV == 2*H.                                 replaces libreax_howu/reax_kkt.cu:263-271 */
int reax_kkt(const void* k, const void* g, const void* beta, void* A, const void* cu, const void* cidx, int NT,
             int H, int HV, void* stream);
/*                                                              replaces libreax_howu/reax_kkt.cu:272 */
int reax_kkt_smem(void);

/* reax_howu followed by a gated RMSNorm over each (token, value head) row of 128:
 * out[f2s[t]][hv][:] = bf16( bf16(nw * bf16(o * rsqrt(sum(o^2) * factor + eps))) * silu(z) ),
 * z = zg[f2s[t] * ZS + hv*128 + :]; tokens with f2s[t] < 0 are not written.  The first call on a device fills a
 * 256 KB table of silu(z) in the library's static device memory (a kernel on `stream`, waited for); -2 if that fails.
 *                                                              replaces libreax_howu/reax_howu_norm_v3.cu:431-435 */
int reax_howu_norm(const void* q, const void* k, const void* v, const void* beta, const void* A, const void* g,
                   void* out, const void* cu, float scale, int N, int H, int HV, void* stream, const void* f2s,
                   const void* z, long long ZS, const void* nw, float eps, float factor);

/* Reduce S bf16 partials (stride pstride elements), add the residual, RMSNorm with (1 + w):
 * d = bf16(sum_s part[s]) (serial != 0: rounded to bf16 after every add); h_out = bf16(res + d);
 * out = bf16( h * rsqrt(sum(h^2) * factor + eps) * (1 + w) ).  Rows n, width D.
 * The reference accepts only D == 2560; this build accepts any D that is a positive multiple of 128
 * (other D: -1).  S outside 2..8: -2.  n <= 0: 0 (nothing to do). replaces libreax_howu/reax_rarn_final.cu:98-106 */
int reax_rarn(const void* part, int S, int serial, long long pstride, const void* res, const void* w,
              void* h_out, void* out, int n, int D, float eps, float factor, void* stream);

/* Depthwise causal conv (4 taps) + SiLU, then L2 norm per 128-channel unit for the q and k units.
 * meta [Tf] int4 = (pos, y, z, w): tap j reads source position src = pos-3+j (skipped when src < 0), from
 * qkv[(z+src)*SX + c] when src >= y, else from cache[(w+src)*C + c].  w [channels][4] bf16.
 * q, k [Tf][rep*KD]; v [Tf][VD].  RT (rows per CTA in the reference) must be 8, 16 or 32 (else -1).
 *                                                              replaces libreax_howu/reax_conv_v2.cu:164-181 */
int reax_conv_l2(const void* qkv, long long SX, const void* cache, int C, const void* meta, const void* w,
                 void* q, void* k, void* v, int Tf, float eps, int KD, int VD, int rep, int skip_v, int RT,
                 void* stream);
/* Value channels only: v = SiLU(conv) for channels 2*KD .. 2*KD+VD.  replaces libreax_howu/reax_conv_v2.cu:183-189 */
int reax_conv_v(const void* qkv, long long SX, const void* cache, int C, const void* meta, const void* w,
                void* v, int Tf, int KD, int VD, void* stream);

/* ==================== attention forward (exported by libreax_howu.so and libreax_fmha_post.so) ==== */

/* Per (batch b, head h): O[r] = softmax(scale * Q[r] K^T + bias[b,h,r,:]) V, head dim 256.
 * Element (b, h, r, d) of Q/K/V/O/bias lives at P + b*sB + h*sH + r*sM + d (strides in elements).
 * Rows whose every score is -inf produce 0.  Returns -1 if bias is NULL.
 *                                  replaces libreax_fmha_post/reax_fmha_v11.cu:566-573 (= libreax_howu/reax_fmha_v8.cu:435-442) */
int reax_fmha_b(const void* q, const void* k, const void* v, const void* bias, void* o, float scale, int B, int H,
                int M, int N, long long qsB, long long qsH, long long qsM, long long ksB, long long ksH,
                long long ksM, long long vsB, long long vsH, long long vsM, long long bsB, long long bsH,
                long long bsM, long long osB, long long osH, long long osM, void* stream);
/* qpos mode, head dim 256: row r of batch b sees keys 0 .. qpos[b*qpBs + r/G] (G query rows per token:
 * the GQA fold, row r <-> query head h*G + r%G of token r/G).
 *                                  replaces libreax_fmha_post/reax_fmha_v11.cu:575-581 (= libreax_howu/reax_fmha_v8.cu:444-450) */
int reax_fmha_q(const void* q, const void* k, const void* v, const int* qpos, int G, long long qpBs, void* o,
                float scale, int B, int H, int M, int N, long long qsB, long long qsH, long long qsM,
                long long ksB, long long ksH, long long ksM, long long vsB, long long vsH, long long vsM,
                long long osB, long long osH, long long osM, void* stream);

/* ============================ libreax_fmha_post.so only ========================================== */

/* qpos mode with the attn_post epilogue fused (head dim 256):
 * outp[inv[b*Lq + r/G]*out_rs + (h*G + r%G)*256 + d] = bf16( bf16(O) * bf16(sigmoid(gate)) ),
 * gate = qg[R*qg_rs + (h*G + r%G)*512 + 256 + d], R = inv[b*Lq + r/G]; rows with R < 0 are skipped.
 *                                                              replaces libreax_fmha_post/reax_fmha_v11.cu:583-590 */
int reax_fmha_qp(const void* q, const void* k, const void* v, const int* qpos, int G, long long qpBs, float scale,
                 int B, int H, int M, int N, long long qsB, long long qsH, long long qsM, long long ksB,
                 long long ksH, long long ksM, long long vsB, long long vsH, long long vsM, const int* inv, int Lq,
                 const void* qg, long long qg_rs, void* outp, long long out_rs, void* stream);

/* ================================ EXTENSIONS (not in the reference) ============================= */

/* EXTENSION: reax_fmha_q / reax_fmha_b / reax_fmha_qp with a selectable head dimension (128 or 256; any other
 * value returns -3).  head_dim 256 is exactly the reference entry point.  Exported wherever the
 * head-dim-256 entry points are. */
int reax_fmha_q_hd(const void* q, const void* k, const void* v, const int* qpos, int G, long long qpBs, void* o,
                   float scale, int B, int H, int M, int N, long long qsB, long long qsH, long long qsM,
                   long long ksB, long long ksH, long long ksM, long long vsB, long long vsH, long long vsM,
                   long long osB, long long osH, long long osM, int head_dim, void* stream);
int reax_fmha_b_hd(const void* q, const void* k, const void* v, const void* bias, void* o, float scale, int B,
                   int H, int M, int N, long long qsB, long long qsH, long long qsM, long long ksB, long long ksH,
                   long long ksM, long long vsB, long long vsH, long long vsM, long long bsB, long long bsH,
                   long long bsM, long long osB, long long osH, long long osM, int head_dim, void* stream);

/* EXTENSION: device status word of the calling library.  Every bounded wait inside this library's kernels
 * that runs out records a nonzero code there (and the kernel returns early instead of hanging).
 * Reads and clears the word in one atomic step on `stream` (a code recorded by a kernel on another stream is
 * never lost between a read and a clear), synchronises `stream` and returns the code.  0 = no timeout seen.
 * Exported by all five. */
int reax_b200_status(void* stream);

#ifdef __cplusplus
}
#endif
#endif /* REAX_ABI_H */
