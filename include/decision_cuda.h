/*
 * decision_cuda.h: the C ABI of the B200 hot path of decision.js.
 *
 * This library replaces the reference's WebGPU device layer (src/gpu.ts) and its WGSL kernels
 * (src/kernels.ts, src/eg2-kernels.ts, src/encoder-kernels.ts) with sm_100a CUDA kernels. Every entry point is
 * extern "C", takes plain pointers and sizes, returns an int status (DC_OK = 0) and never throws; the message of
 * the last failure on the calling thread is dc_last_error().
 *
 * Pointers named d_* are device pointers (from dc_alloc or any CUDA allocation on the context's device); h_*
 * are host pointers. f16 tensors are IEEE binary16, row-major. Quantized weights use the reference's format
 * (scripts/export_common.py:64-97): q8 = one byte per weight, code c in [-127,127] stored as c+128; q4 = two
 * codes per byte, low nibble first, stored as c+8; one f16 scale per 32 weights along K at S[n*(K/32)+k/32].
 * A dequantized weight is f16((code - Z) * scale), rounded once.
 *
 * Kernel launches are asynchronous on the context's stream (one stream per context, as the reference has one
 * command buffer per pass); dc_sync waits, with a timeout.
 */
#ifndef DECISION_CUDA_H
#define DECISION_CUDA_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define DC_API __attribute__((visibility("default")))
#else
#define DC_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes. The reference throws Error("decision.js: ...") from the same situations: a WebGPU validation
 * error at finish (src/gpu.ts:256-261), a short range read (src/gpu.ts:66), a tensor over the device's buffer
 * limit (src/gpu.ts:76-78), a lost device (src/d1.ts:67-77). */
enum {
  DC_OK = 0,
  DC_EINVAL = 1,   /* bad argument: null handle, size, shape or dtype */
  DC_ENOMEM = 2,   /* device or host allocation failed */
  DC_ECUDA = 3,    /* a CUDA runtime error (the message names it) */
  DC_ETIMEOUT = 4, /* dc_sync gave up, or a kernel's bounded wait expired */
  DC_EFORMAT = 5,  /* manifest.json / weights.bin malformed or unsupported */
  DC_EIO = 6       /* a file could not be read in full */
};

/* Matmul epilogues. The gated ones take a fused gate|up weight of N = 2I rows laid out as alternating rows, gate
 * row i at row 2i and up row i at row 2i + 1 (N a multiple of 128; dc_load_weights stores every model's `gu` /
 * `w13` weight this way) and write Y [M, I] = f16(act(f16 gate) * f16 up), the fused form of the reference's
 * MATMUL_SWIGLU (src/kernels.ts:674-676) and of matmul followed by GELU_MUL (src/eg2-kernels.ts:166-177). */
enum {
  DC_EPI_NONE = 0,     /* Y = f16(acc) */
  DC_EPI_GLU_GELU = 1, /* Y = gelu_tanh(gate) * up */
  DC_EPI_GLU_SILU = 2  /* Y = silu(gate) * up */
};

/* Gated activations over a fused gate|up row. */
enum {
  DC_ACT_SILU = 0,     /* SILU_MUL, src/kernels.ts:49-60 */
  DC_ACT_GELU_TANH = 1, /* GELU_MUL, src/eg2-kernels.ts:166-177 */
  DC_ACT_GELU_ERF = 2   /* GELU_MUL with erf (Laya), src/encoder-kernels.ts:26-44; dc_glu only */
};

typedef struct dc_ctx dc_ctx;
typedef struct dc_model dc_model;

/* ------------------------------------------------------------------ context and memory
 * Replaces requestDevice (src/gpu.ts:38-54) and the buffer helpers storage / activations / destroy
 * (src/gpu.ts:148-174, 107-110). */

/* The message of the last failure on this thread ("" when none). Never null. The reference carries the same text in
 * the Error it throws ("decision.js: ...", src/gpu.ts:66, 78, 256-261). */
DC_API const char *dc_last_error(void);
/* A context on CUDA device `device`: its own stream, scratch and kernel state. */
DC_API int dc_init(int device, dc_ctx **out);
DC_API int dc_destroy(dc_ctx *ctx);
/* The device count visible to this process (no reference counterpart: WebGPU exposes one adapter). */
DC_API int dc_device_count(int *out);
DC_API int dc_alloc(dc_ctx *ctx, size_t bytes, void **d_out);
DC_API int dc_free(dc_ctx *ctx, void *d_ptr);
/* Host <-> device copies on the context's stream; synchronous for the host buffer (pageable or pinned). */
DC_API int dc_upload(dc_ctx *ctx, void *d_dst, const void *h_src, size_t bytes);
DC_API int dc_download(dc_ctx *ctx, void *h_dst, const void *d_src, size_t bytes);
DC_API int dc_memset(dc_ctx *ctx, void *d_dst, int value, size_t bytes);
/* Waits for every launch on the context's stream; DC_ETIMEOUT after timeout_ms (< 0: no limit). Also reports
 * a kernel's bounded-wait failure (its device error word), as finish() reports a validation error
 * (src/gpu.ts:245-261). */
DC_API int dc_sync(dc_ctx *ctx, int timeout_ms);
/* The context's cudaStream_t, for interop (e.g. wrapping it in a torch stream). No reference counterpart. */
DC_API void *dc_stream(dc_ctx *ctx);
/* on != 0 declares that the weights given to the following dc_qmatmul* calls are not written by any kernel on the
 * context's stream (written before, and the stream synchronised since): a matmul may then request its codes and
 * scales while the kernel before it is still running. The model passes (dc_forward_*) do this on their own.
 * Default off. No reference counterpart (WebGPU has no programmatic dependent launch). */
DC_API int dc_static_weights(dc_ctx *ctx, int on);

/* Failure-detection self-test (no reference counterpart): enqueues one kernel whose bounded wait, on a barrier that
 * nothing completes, expires after limit_us (1 to 2,000,000) and flags the device error word, as an expired wait in
 * any pipeline kernel does. The next dc_sync returns DC_ETIMEOUT ("bounded wait expired") and clears the word; the
 * context stays usable. Nothing faults or hangs. */
DC_API int dc_selftest_wait(dc_ctx *ctx, int limit_us);

/* Per-kernel-kind timing (the reference's __d1Profile, src/gpu.ts:29-34,185-197,248-272): when enabled, every
 * launch is bracketed by CUDA events on the context's stream. dc_profile_read syncs, then returns the summed
 * milliseconds, launch count and algorithmic flops/bytes of kind `kind` since the last reset. */
enum { DC_K_QGEMM = 0, DC_K_QGEMV = 1, DC_K_ATTN = 2, DC_K_NORM = 3, DC_K_OTHER = 4, DC_K_KINDS = 5 };
DC_API int dc_profile(dc_ctx *ctx, int enable);
DC_API int dc_profile_read(dc_ctx *ctx, int kind, double *ms, long long *launches, double *flops, double *bytes);

/* ------------------------------------------------------------------ kernels (one per recorder op)
 * Each replaces one WGSL dispatch of the reference's recorder (src/gpu.ts:177-281).
 * Pointer alignment: activations, outputs and f16 norm weights 16-byte aligned (the kernels move rows in 16-byte
 * vectors); quantized codes 16-byte for the matmuls, 8 (q8) or 4 (q4) bytes for gather/dequant; f16 scales 2-byte;
 * int32 index arrays 4-byte. Every entry point checks this on the host before any device work and returns
 * DC_EINVAL with a message naming the pointer otherwise. Buffers from cudaMalloc (256-byte aligned) always pass. */

/* Y[M,N] = X[M,K] . deq(W)[N,K]^T, f32 accumulation, f16 out (src/gpu.ts:202-226 matmul; semantics of
 * MATMUL_PORTABLE_Q8/Q4, src/kernels.ts:445-520). bits 8 or 4; K a multiple of 32. d_Wq: the codes
 * (N*K or N*K/2 bytes); d_S: f16 scales [N, K/32]. The form follows M: M <= 32 the decode form (5), and up to 64
 * tokens on small weights (N*K <= 4M codes);
 * M <= 128, and larger M whose 64-token tiles fit one wave of CTAs, form 4; then form 6 while its 192-token tiles fit one wave;
 * otherwise the 256-token prefill form (3). */
DC_API int dc_qmatmul(dc_ctx *ctx, const void *d_X, const void *d_Wq, const void *d_S, void *d_Y, int M, int N, int K,
               int bits, int epilogue);
/* dc_qmatmul forced onto one form: 0 = prefill, one CTA per output tile (tokens on the MMA's M side);
 * 1 = skinny (weights on the M side, split-K across CTAs when splits > 1; splits <= 0 picks; M <= 128);
 * 2 = prefill, persistent (one CTA per SM walking the tiles, double-buffered accumulators);
 * 3 = prefill, persistent, 128 weight rows x 256 tokens per tile, weights dequantized into shared memory (the
 * default for large M); 4 = form 6 with a token tile fitted to M (16, 32 or 64) and K split across CTAs
 * (splits <= 0 picks); 5 = decode (M <= 64): a register-level weight stream on the tensor pipe, K split
 * over a cluster of `splits` <= 8 CTAs (<= 0 picks); 6 = prefill, persistent, 192-token tiles, weights
 * dequantized into tensor memory as the MMA's A operand; 7 = prefill on CTA pairs (tcgen05 cta_group::2, 256
 * weight rows x 256 tokens per MMA, each CTA loading half the tokens). For tests and tuning; the reference's
 * matmul likewise picks among its variants (src/gpu.ts:202-226). */
DC_API int dc_qmatmul_form(dc_ctx *ctx, const void *d_X, const void *d_Wq, const void *d_S, void *d_Y, int M, int N, int K,
                    int bits, int form, int splits);
/* The skinny (split-K) form of dc_qmatmul for callers that cannot allocate device memory: a plug-in whose host
 * process owns all device memory and forbids cudaMalloc once it is running, or a latency-bound loop that cannot
 * afford cudaMalloc's implicit device synchronisation. It has no counterpart in the reference. It takes no context
 * and allocates nothing: the split-K partials (at most 16 MiB of f32: splits * M * N * 4 bytes), one counter per
 * output tile (at most 4096) and an error word sit in one static device array that every GPU loading this library
 * holds until the process exits. Runs on `stream` (a cudaStream_t, 0 for the legacy default stream) of the current
 * device. M <= 128; splits <= 0 picks a split count within the static limit; larger requests fail with DC_EINVAL and
 * a message naming the limit. The first call on a device resolves the array's device address and keeps it; make
 * that first call before any stream capture (a lookup that fails, e.g. during capture, returns DC_ECUDA, is not
 * kept, and the next call tries again). All calls share the array and it keeps the last call's contents (each
 * call zeroes the tile counters it uses): calls that overlap on the GPU, on any stream, race and corrupt each
 * other's results. A kernel whose bounded wait expires is not reported by this entry point (it has no context to
 * report through); its output is then unspecified. It launches as a plain kernel, without the programmatic
 * dependent launch and the early weight reads that dc_qmatmul uses inside a context (dc_static_weights), so at
 * the same shape it can be a few microseconds slower per call. */
DC_API int dc_qmatmul_skinny_noalloc(void *stream, const void *d_X, const void *d_Wq, const void *d_S, void *d_Y,
                                     int M, int N, int K, int bits, int splits);
/* W16[n*K+k] = deq(W)[n,k] (tileWeights without the re-layout, src/kernels.ts:528-543). */
DC_API int dc_dequant(dc_ctx *ctx, const void *d_Wq, const void *d_S, void *d_W16, int N, int K, int bits);
/* Y[M,N] = X[M,K] . W16[N,K]^T on weights dequantized to f16 beforehand (dc_dequant): matmulDirect
 * (src/kernels.ts:549-676) with the fused SwiGLU/GeGLU epilogue of dc_qmatmul (same epilogue codes, same gate|up
 * row interleave). The same operand values as dc_qmatmul on the codes (f16((code - Z) * scale)), f32
 * accumulation, f16 out; twice (q8) or four times (q4) the weight bytes, no dequantisation in the pipeline: the
 * prefill form for large M (a CTA pair per 256 x 256 tile). K a multiple of 32; X, W16 and Y 16-byte aligned. */
DC_API int dc_qmatmul_f16(dc_ctx *ctx, const void *d_X, const void *d_W16, void *d_Y, int M, int N, int K,
                          int epilogue);
/* ADD_RMSNORM (src/kernels.ts:24-46): when add, X += Yr (stored f16); O = rmsnorm(X) * W. */
DC_API int dc_add_rmsnorm(dc_ctx *ctx, void *d_X, const void *d_Yr, const void *d_W, void *d_O, int T, int H, int add,
                   float eps);
/* SANDWICH (src/eg2-kernels.ts:18-48): X = (X + rmsnorm(Y) * W1) * scale; when d_W2, O = rmsnorm(X) * W2. */
DC_API int dc_sandwich(dc_ctx *ctx, void *d_X, const void *d_Y, const void *d_W1, const void *d_W2, void *d_O, int T,
                int H, float eps, float scale);
/* QKV_NORM_ROPE (src/eg2-kernels.ts:53-96) / QK_NORM_ROPE (src/kernels.ts:87-112) for any even D <= 512, in
 * place on Z [T, (heads + 2 kv) * D]: per-head RMSNorm (q by qn, k by kn, v plainly when vnorm, else v is left
 * as is), then rotate-half RoPE on q and k at d_pos[t] with inverse frequencies theta^(-2d/D). */
DC_API int dc_qkv_norm_rope(dc_ctx *ctx, void *d_Z, const void *d_qn, const void *d_kn, const int32_t *d_pos, int T,
                     int heads, int kv, int D, float eps, float theta, int vnorm);
/* Attention (src/eg2-kernels.ts:104-163, src/kernels.ts:117-147) over Z [T, (heads + 2 kv) * D] into
 * Y [T, heads * D]: query token t reads the keys of [rng[4t], rng[4t+1]) union [rng[4t+2], rng[4t+3]) (sequence,
 * causal prefix, window, or trunk + own branch). GQA head h reads kv head h / (heads / kv). D = 64 (d1-3B,
 * src/kernels.ts:117-147), 128, 256 or 512 (EmbeddingGemma 2's full layers, src/eg2-kernels.ts:104). d_Z and d_Y
 * 16-byte aligned (DC_EINVAL otherwise). */
DC_API int dc_attention(dc_ctx *ctx, const void *d_Z, const int32_t *d_rng, void *d_Y, int T, int heads, int kv, int D,
                 float scale);
/* dc_attention forced onto one kernel: 0 = mma.sync tiles (any of the four head dims), 1 = tcgen05 (TMEM
 * accumulators, D = 64, 128 or 256; the default for those). For tests and tuning; the reference likewise builds one attention kernel per head dim and tile
 * (src/eg2-kernels.ts:104). */
DC_API int dc_attention_form(dc_ctx *ctx, const void *d_Z, const int32_t *d_rng, void *d_Y, int T, int heads, int kv,
                             int D, float scale, int form);
/* dc_attention_form over rows of `stride` halves (q | k | v heads, then anything), and with `gate` d3-lite's gated
 * attention (src/d3-kernels.ts:174-240 attention256): the q heads' gates follow the v heads in the row and
 * Y = attention * sigmoid(gate). form -1 picks as dc_attention does. stride a multiple of 8. */
DC_API int dc_attention_ex(dc_ctx *ctx, const void *d_Z, const int32_t *d_rng, void *d_Y, int T, int heads, int kv,
                           int D, float scale, long stride, int gate, int form);
/* SILU_MUL / GELU_MUL (src/kernels.ts:49-60, src/eg2-kernels.ts:166-177; recorder().swiglu, src/gpu.ts:229-234):
 * H[t,c] = f16(act(A[t,c]) * A[t,I+c]) over a fused gate|up A [T, 2I]. */
DC_API int dc_glu(dc_ctx *ctx, const void *d_A, void *d_H, int T, int I, int act);
/* GATHER_Q8 / GATHER_Q4 (src/kernels.ts:7-21, 293-296): X[t,:] = deq(E)[ids[t],:]. */
DC_API int dc_gather(dc_ctx *ctx, const int32_t *d_ids, const void *d_Eq, const void *d_Es, void *d_X, int T, int H,
              int bits);
/* POOL_PROJECT (src/eg2-kernels.ts:204-228): per sequence [seqs[2s], seqs[2s+1]) the f32 mean of X's rows,
 * then out[s,:] = mean . W^T when d_W (W [N,H] f16), else out[s,:] = mean (N = H). H a multiple of 8, at most
 * 6400 (the CTA keeps 9 H floats of partial sums in shared memory). */
DC_API int dc_pool(dc_ctx *ctx, const void *d_X, const int32_t *d_seqs, const void *d_W, float *d_out, int S, int H,
            int N);
/* LEAF_LOGITS (src/kernels.ts:150-185): at row leaves[l], the final RMSNorm, then the dot with the q4/q8
 * embedding rows ids[l*nIds + j], dequantized in f32. */
DC_API int dc_leaf_logits(dc_ctx *ctx, const void *d_X, const int32_t *d_leaves, const void *d_W, const int32_t *d_ids,
                   const void *d_Eq, const void *d_Es, float *d_out, int L, int H, int nIds, int bits, float eps);

/* SHORT_CONV (src/kernels.ts:65-84), LFM2's gated short convolution of d1-3B's conv layers: over the in-projection
 * rows Z [T, 3H] = B | C | U, Y[t,c] = f16(C[t,c] * sum_j Wc[c,j] * B[r_j,c] * U[r_j,c]) with Wc f16 [H, 3] and
 * r_j = taps[4t + j] (the tokens read by taps 0, 1, 2; -1 reads nothing), in f32. H a multiple of 8; Z, Wc, Y and
 * taps 16-byte aligned. */
DC_API int dc_short_conv(dc_ctx *ctx, const void *d_Z, const void *d_Wc, const int32_t *d_taps, void *d_Y, int T,
                         int H);
/* PLE_MIX (src/eg2-kernels.ts:181-200), EmbeddingGemma 2's per-layer-embedding gate: over rows of P values,
 * O[t,:] = f16(gelu_tanh(G[t,:]) * E[t,:] * rsqrt(mean(E[t,:]^2) + eps) * W). P a multiple of 8, at most 1024. */
DC_API int dc_ple_mix(dc_ctx *ctx, const void *d_G, const void *d_E, const void *d_W, void *d_O, int T, int P,
                      float eps);
/* READOUT (src/d3-kernels.ts:243-260), d3-lite's code readout: out[k] = X[pairs[2k]] . R[pairs[2k+1]] in f32 for
 * X f16 [T, H] and R f32 [codes, H]. A row or code out of range reads row / code 0 and flags the device error
 * word (the next dc_sync returns DC_EINVAL). H a multiple of 8; X and R 16-byte aligned. */
DC_API int dc_readout(dc_ctx *ctx, const void *d_X, const float *d_R, const int32_t *d_pairs, float *d_out, int P,
                      int H, int T, int codes);

/* The Gated DeltaNet mixer of d3-lite's linear-attention layers (src/d3-kernels.ts:23-149 gdnLayer, binding the
 * same buffers: spans, the in-projection rows, conv, A_log, dt_bias, gnorm, the output), heads of 128. Z rows of
 * `stride` f16: q | k | v (H*128 each) from 0, z (H*128) | b (H) | a (H) from `qkv`. Per sequence s, spans[4s..4s+3]
 * = a start, a length | write-a << 31, b start, b length: the sequence is span a then span b, span a's outputs
 * written only when flagged. Per token: the causal 4-tap conv (W [3*H*128, 4]) + SiLU of q, k, v; q, k
 * L2-normalised (q by 128^-1/2 more); decay = exp(-exp(A_log) softplus(a + dt_bias)), beta = sigmoid(b); the delta
 * rule on a 128 x 128 f32 state per (sequence, head); Y[t, h*128 + d] = f16(rmsnorm(o)_d * gw_d * silu(z_d)) with
 * `eps`. Y is [T, H*128]; a span outside [0, T) flags the device error word. */
DC_API int dc_gdn(dc_ctx *ctx, const void *d_Z, long stride, long qkv, int H, const void *d_W, const void *d_A_log,
                  const void *d_dt_bias, const void *d_gw, const uint32_t *d_spans, int nseq, float eps, void *d_Y,
                  int T);

/* The d1-omni / Laya decision-head kernels (src/kernels.ts:187-283), binding the reference's buffers.
 * ADD_ROWS: Xo[t,:] = f16(Xi[t,:] + E[idx[t],:]) (an index outside [0, nE) reads row 0 and flags the device error
 * word). H a multiple of 8. */
DC_API int dc_add_rows(dc_ctx *ctx, const void *d_Xi, const int32_t *d_idx, const void *d_E, void *d_Xo, int T, int H,
                       int nE);
/* BIAS_ACT: Y[t,n] = f16(act(Y[t,n] + b[n])) in place; act 0 none, 1 ReLU, 2 GELU (erf, Abramowitz-Stegun 7.1.26).
 * N a multiple of 8. */
DC_API int dc_bias_act(dc_ctx *ctx, void *d_Y, const void *d_b, int T, int N, int act);
/* ADD_LAYERNORM: with add, X += Yr (stored f16); then O = f16((X - mean) / sqrt(max(var, 0) + eps) * W + B), the
 * sums over the unrounded row, B optional (NULL: Laya's bias-free norms). H a multiple of 8, at most 2048. */
DC_API int dc_add_layernorm(dc_ctx *ctx, void *d_X, const void *d_Yr, const void *d_W, const void *d_B, void *d_O,
                            int T, int H, int add, float eps);
/* GATHER_ROWS: G[m,:] = X[rows[m],:] (a row outside [0, T) reads row 0 and flags the device error word). */
DC_API int dc_gather_rows(dc_ctx *ctx, const void *d_X, const int32_t *d_rows, void *d_G, int M, int H, int T);
/* SCORE: out[m] = Y[m,:] . w + b[0] in f32. H a multiple of 8. */
DC_API int dc_score(dc_ctx *ctx, const void *d_Y, const void *d_w, const void *d_b, float *d_out, int M, int H);
/* Q/K RoPE with an optional RMSNorm over rows of `stride` f16 holding `heads` q heads then `kv` k heads of D: with
 * norm, each head x = x / sqrt(mean(x^2) + eps) * (qn or kn); then the half-split rotation of the first `rot` dims,
 * pairs (d, d + rot/2), angle pos[t] * theta^(-2d / rot). Laya's ROPE (src/encoder-kernels.ts:5-24: D = rot = 64,
 * no norm) and d3-lite's QK_NORM_ROPE_256 (src/d3-kernels.ts:150-172: D = 256, rot = 64). rot a power of two from
 * 16 to min(D, 256). */
DC_API int dc_qk_rope(dc_ctx *ctx, void *d_Z, const void *d_qn, const void *d_kn, const int32_t *d_pos, int T,
                      int heads, int kv, int D, long stride, int rot, int norm, float eps, float theta);

/* ------------------------------------------------------------------ models (manifest.json + weights.bin)
 * Replaces loadWeights (src/gpu.ts:57-88) and the engine graphs (src/eg2-engine.ts, src/d1-3b-engine.ts). */

/* Reads `dir`/manifest.json (format "d1.js/1", scripts/export_common.py:17-61) and uploads every tensor of
 * `dir`/weights.bin to the context's device. Errors: DC_EIO on a short read, DC_EFORMAT on a bad manifest. */
DC_API int dc_load_weights(dc_ctx *ctx, const char *dir, dc_model **out);
/* The same checks as dc_load_weights (manifest parse, dtypes, shapes, byte counts, alignment, every range inside
 * weights.bin) without a device: DC_OK, DC_EFORMAT or DC_EIO. No reference counterpart (its loader checks as it
 * uploads, src/gpu.ts:57-88). */
DC_API int dc_check_weights(const char *dir);
DC_API int dc_model_free(dc_model *model);
/* The manifest's config.model ("eg2", "d1-3b", ...; with no model key, the reference's rule, src/d1.ts:63-64) and
 * config values, for the host. */
DC_API int dc_model_kind(dc_model *model, char *buf, size_t len);
DC_API int dc_model_config_f(dc_model *model, const char *key, double *out);
/* Device pointers of a tensor: data (codes for q4/q8) and scales (null otherwise); dtype 4, 8, 16 (f16), 32.
 * Fused gate|up weights (`*.gu`, `*.w13`, N a multiple of 128) are held with their rows interleaved, gate row i
 * at row 2i and up row i at row 2i + 1 (see the gated epilogues); every other tensor is held exactly as in
 * weights.bin. */
DC_API int dc_model_tensor(dc_model *model, const char *name, void **d_data, void **d_scales, int *dtype, int64_t *rows,
                    int64_t *cols);

/* Eg2Engine.embed (src/eg2-engine.ts:72-141): S packed sequences, h_ids [T], h_bounds [S, 2] = [start, end) of
 * each; h_out [S, N] f32 = the mean-pooled (projected when the model has "projection") final hidden states, before
 * the host's L2 normalisation. Layer types (sliding / full attention) carry their own head dim (64 to 512), KV
 * heads and RoPE theta; with per-layer embeddings (config "ple" > 0) every layer ends with the PLE block
 * (src/eg2-engine.ts:123-128), else the layer scalar and the next input norm go on the MLP's sandwich norm. */
DC_API int dc_forward_encoder(dc_model *model, const int32_t *h_ids, const int32_t *h_bounds, int T, int S, float *h_out);
/* D13BEngine.run (src/d1-3b-engine.ts:44-108) for decoders with attention and LFM2 short-conv ("conv") layers:
 * h_ids, h_pos [T], key ranges h_rng [T, 4] (see dc_attention), readout rows h_leaves [L] and the readout ids
 * h_leaf_ids [L, nIds]; h_out [L, nIds] f32 logits. The conv layers' taps (t-2, t-1, t within each token's
 * sequence, src/d1-3b-engine.ts:53-62) are derived on the device from the causal key ranges. */
DC_API int dc_forward_decoder(dc_model *model, const int32_t *h_ids, const int32_t *h_pos, const int32_t *h_rng, int T,
                       const int32_t *h_leaves, const int32_t *h_leaf_ids, int L, int nIds, float *h_out);

/* The same two passes on device-resident inputs and output (device pointers), asynchronous on the model's
 * context stream: nothing is copied and nothing waits (no reference counterpart: a caller that keeps its tokens
 * on the GPU). Token ids, readout rows and sequence bounds cannot be
 * checked on the host here; the kernels clamp them (no read leaves the tables) and flag them in the device
 * error word, which the next dc_sync reports as DC_EINVAL. */
DC_API int dc_forward_encoder_device(dc_model *model, const int32_t *d_ids, const int32_t *d_bounds, int T, int S,
                                     float *d_out);
DC_API int dc_forward_decoder_device(dc_model *model, const int32_t *d_ids, const int32_t *d_pos,
                                     const int32_t *d_rng, int T, const int32_t *d_leaves, const int32_t *d_leaf_ids,
                                     int L, int nIds, float *d_out);
/* D3Engine.logits (src/d3-engine.ts:67-139) on a d3-lite model (config model "d3", scripts/export-d3.py): Gated
 * DeltaNet layers and gated attention layers with 256-wide heads (q/k RMSNorm, RoPE on the first rotary_dim dims),
 * SwiGLU MLPs, the final norm, then the code readout. Per token: ids, positions and key ranges (x, y, z, w) as the
 * reference builds them (its sequence, or a shared trunk and its own branch); per sequence the two spans the
 * linear layers scan (a start, a length | write-a << 31, b start, b length); per readout pair (token row, code):
 * h_out[k] = f32 logit. Host buffers; the pass is captured and replayed as a CUDA graph like the others. */
DC_API int dc_forward_d3(dc_model *model, const int32_t *h_ids, const int32_t *h_pos, const int32_t *h_rng, int T,
                         const uint32_t *h_spans, int nseq, const int32_t *h_pairs, int P, float *h_out);
/* D1OmniEngine.logits (src/omni-engine.ts:56-141) on a d1-omni model (config head_layers, scripts/export-omni.py):
 * the LFM2 backbone (bidirectional within each sequence), the question-type embedding, the pre-norm transformer
 * head with its biases, the scorer (LayerNorm, the option markers' rows, fc + GELU, Linear(H, 1)). Per token: id,
 * position, key ranges (its sequence), conv taps (t-1, t, t+1 within the sequence, -1 outside) and question type;
 * per option its marker's token row: h_out[k] = f32 raw logit. */
DC_API int dc_forward_omni(dc_model *model, const int32_t *h_ids, const int32_t *h_pos, const int32_t *h_rng,
                           const int32_t *h_taps, int T, const int32_t *h_qtype, const int32_t *h_markers, int M,
                           float *h_out);
/* LayaEngine.logits (src/laya-engine.ts:47-141) on a Laya model (config model "laya", scripts/export-laya.py): the
 * ModernBERT encoder (bias-free LayerNorms, RoPE attention with 64-wide heads, over the whole sequence on full
 * layers and over h_win's ±window on the others, GELU-gated MLP), then d1-omni's decision head. Per token: id,
 * position, its sequence's key range, its window's key range, question type; per option its marker's token row:
 * h_out[k] = f32 raw logit. */
DC_API int dc_forward_laya(dc_model *model, const int32_t *h_ids, const int32_t *h_pos, const int32_t *h_rng,
                           const int32_t *h_win, int T, const int32_t *h_qtype, const int32_t *h_markers, int M,
                           float *h_out);
/* The EmbeddingGemma 2 typed-decision head (src/eg2-head.ts: Eg2Head.logits, run by the reference on the host after
 * the encoder pass) on the device, in f32, for a whole batch of questions at once. d_S [nS, E], d_Q [nQ, E] and
 * d_O [nO, E] hold the L2-normalised embeddings (what embed() returns) of the states, questions and option texts;
 * d_items [n_items, 6] names per question instance its state row, question row, question type (the index of its
 * type in the manifest's question_types), first option row, option count and first output index; d_logits gets
 * each option's raw logit (before the temperature and softmax the host applies, src/d1.ts:206-214). The head's
 * f32 tensors are the manifest's "host" section, uploaded with the weights; its scalars are config.head. An item
 * whose rows or type are out of range is skipped and flags the device error word. All pointers 4-byte aligned;
 * asynchronous on the model's context stream. */
DC_API int dc_eg2_head(dc_model *model, const float *d_S, int nS, const float *d_Q, int nQ, const float *d_O, int nO,
                       const int32_t *d_items, int n_items, float *d_logits);
/* The context a model was loaded on (its stream orders the device-resident passes). No reference counterpart. */
DC_API int dc_model_context(dc_model *model, dc_ctx **out);

#ifdef __cplusplus
}
#endif
#endif
