// The extern "C" kernel entry points: argument checks, then the kernel hosts. One entry point per recorder op
// of the reference (src/gpu.ts:177-281).
#include "dc_internal.h"

int ops_add_rmsnorm(dc_ctx *, void *, const void *, const void *, void *, int, int, int, float);
int ops_sandwich(dc_ctx *, void *, const void *, const void *, const void *, void *, int, int, float, float);
int ops_qkv_norm_rope(dc_ctx *, void *, const void *, const void *, const int *, int, int, int, int, float, float,
                      int);
int ops_glu(dc_ctx *, const void *, void *, int, int, int, int);
int ops_gather(dc_ctx *, const int *, const void *, const void *, void *, int, int, int, int);
int ops_dequant(dc_ctx *, const void *, const void *, void *, int, int, int);
int ops_pool(dc_ctx *, const void *, const int *, const void *, float *, int, int, int);
int ops_leaf_logits(dc_ctx *, const void *, const int *, const void *, const int *, const void *, const void *,
                    float *, int, int, int, int, float, int, int);
int attn_launch(dc_ctx *, const void *, const int *, void *, int, int, int, int, float);
int ops_wait_probe(dc_ctx *, int);
int attn_launch_form(dc_ctx *, const void *, const int *, void *, int, int, int, int, float, int);
int attn_launch_ex(dc_ctx *, const void *, const int *, void *, int, int, int, int, float, int, long, int);
int ops_short_conv(dc_ctx *, const void *, const void *, const int *, void *, int, int);
int ops_ple_mix(dc_ctx *, const void *, const void *, const void *, void *, int, int, float);
int ops_readout(dc_ctx *, const void *, const float *, const int *, float *, int, int, int, int);
int ops_gdn(dc_ctx *, const void *, long, long, int, const void *, const void *, const void *, const void *,
            const uint32_t *, int, float, void *, int);
int ops_add_rows(dc_ctx *, const void *, const int *, const void *, void *, int, int, int);
int ops_bias_act(dc_ctx *, void *, const void *, int, int, int);
int ops_add_layernorm(dc_ctx *, void *, const void *, const void *, const void *, void *, int, int, int, float);
int ops_gather_rows(dc_ctx *, const void *, const int *, void *, int, int, int);
int ops_score(dc_ctx *, const void *, const void *, const void *, float *, int, int);
int ops_qk_rope(dc_ctx *, void *, const void *, const void *, const int *, int, int, int, int, long, int, int, float,
                float);

#define DC_PRE(ctx)                 \
  do {                              \
    int rc_ = dc_use(ctx);          \
    if (rc_) return rc_;            \
  } while (0)

// Pointer alignment the kernels rely on: 16 bytes where they move rows in 16-byte vectors, the element size
// elsewhere. Checked on the host, before the context is used, so a misaligned view is DC_EINVAL, not a device fault.
static bool aln(const void *p, unsigned a) { return ((uintptr_t)p & (a - 1)) == 0; }
static bool al16(const void *p) { return aln(p, 16); }

static int check_qmm(const void *X, const void *Wq, const void *S, void *Y, int M, int N, int K, int bits) {
  DC_CHECK(X && Wq && S && Y, DC_EINVAL, "decision.js: qmatmul: null pointer");
  DC_CHECK(M > 0 && N > 0 && K > 0, DC_EINVAL, "decision.js: qmatmul: bad shape M=%d N=%d K=%d", M, N, K);
  DC_CHECK(bits == 8 || bits == 4, DC_EINVAL, "decision.js: qmatmul: bits must be 4 or 8 (got %d)", bits);
  DC_CHECK(K % 32 == 0, DC_EINVAL, "decision.js: qmatmul: K=%d is not a multiple of the 32-wide scale group", K);
  DC_CHECK(al16(X) && al16(Wq) && al16(Y), DC_EINVAL,
           "decision.js: qmatmul: X, the codes and Y must be 16-byte aligned");
  DC_CHECK(aln(S, 2), DC_EINVAL, "decision.js: qmatmul: the scales must be 2-byte aligned");
  return DC_OK;
}

static double qmm_bytes(int M, int N, int K, int bits) {
  return (double)N * K * bits / 8 + (double)N * K / 16 + 2.0 * M * K + 2.0 * M * N;
}

extern "C" int dc_qmatmul(dc_ctx *ctx, const void *X, const void *Wq, const void *S, void *Y, int M, int N, int K,
                          int bits, int epilogue) {
  int rc = check_qmm(X, Wq, S, Y, M, N, K, bits);
  if (rc) return rc;
  DC_CHECK(epilogue >= DC_EPI_NONE && epilogue <= DC_EPI_GLU_SILU, DC_EINVAL,
           "decision.js: qmatmul: unknown epilogue %d", epilogue);
  DC_CHECK(epilogue == DC_EPI_NONE || N % 128 == 0, DC_EINVAL,
           "decision.js: qmatmul: a gated epilogue needs N (=2I) a multiple of 128 (got %d)", N);
  DC_PRE(ctx);
  if (epilogue != DC_EPI_NONE) {
    dc_prof_begin(ctx, DC_K_QGEMM, 2.0 * M * N * K, qmm_bytes(M, N, K, bits) - M * N);
    rc = qgemm_launch_glu(ctx, X, Wq, S, Y, M, N, K, bits, epilogue == DC_EPI_GLU_GELU ? 1 : 2);
    dc_prof_end(ctx);
    return rc;
  }
  const int form = qgemm_pick_form(M, N, K, bits, ctx->sms);
  dc_prof_begin(ctx, (form == 1 || form == 5 || (form == 4 && M <= 128)) ? DC_K_QGEMV : DC_K_QGEMM, 2.0 * M * N * K,
                qmm_bytes(M, N, K, bits));
  rc = qgemm_launch(ctx, X, Wq, S, Y, M, N, K, bits, form, 0);
  dc_prof_end(ctx);
  return rc;
}

extern "C" int dc_qmatmul_form(dc_ctx *ctx, const void *X, const void *Wq, const void *S, void *Y, int M, int N,
                               int K, int bits, int form, int splits) {
  int rc = check_qmm(X, Wq, S, Y, M, N, K, bits);
  if (rc) return rc;
  DC_CHECK(form >= 0 && form <= 7, DC_EINVAL, "decision.js: qmatmul: form must be 0 to 7");
  DC_CHECK(form != 1 || M <= 128, DC_EINVAL, "decision.js: qmatmul: form 1 takes M <= 128 (got %d)", M);
  DC_CHECK(form != 5 || M <= 64, DC_EINVAL, "decision.js: qmatmul: the decode form takes M <= 64 (got %d)", M);
  DC_PRE(ctx);
  dc_prof_begin(ctx, (form == 1 || form == 5 || (form == 4 && M <= 128)) ? DC_K_QGEMV : DC_K_QGEMM, 2.0 * M * N * K,
                qmm_bytes(M, N, K, bits));
  rc = qgemm_launch(ctx, X, Wq, S, Y, M, N, K, bits, form, splits);
  dc_prof_end(ctx);
  return rc;
}

extern "C" int dc_qmatmul_f16(dc_ctx *ctx, const void *X, const void *W16, void *Y, int M, int N, int K,
                              int epilogue) {
  DC_CHECK(X && W16 && Y, DC_EINVAL, "decision.js: qmatmul_f16: null pointer");
  DC_CHECK(M > 0 && N > 0 && K > 0, DC_EINVAL, "decision.js: qmatmul_f16: bad shape M=%d N=%d K=%d", M, N, K);
  DC_CHECK(K % 32 == 0, DC_EINVAL, "decision.js: qmatmul_f16: K=%d is not a multiple of 32", K);
  DC_CHECK(al16(X) && al16(W16) && al16(Y), DC_EINVAL, "decision.js: qmatmul_f16: X, W16 and Y must be 16-byte aligned");
  DC_CHECK(epilogue >= DC_EPI_NONE && epilogue <= DC_EPI_GLU_SILU, DC_EINVAL,
           "decision.js: qmatmul_f16: unknown epilogue %d", epilogue);
  DC_CHECK(epilogue == DC_EPI_NONE || N % 128 == 0, DC_EINVAL,
           "decision.js: qmatmul_f16: a gated epilogue needs N (=2I) a multiple of 128 (got %d)", N);
  DC_PRE(ctx);
  dc_prof_begin(ctx, DC_K_QGEMM, 2.0 * M * N * K,
                2.0 * N * K + 2.0 * M * K + 2.0 * M * N / (epilogue == DC_EPI_NONE ? 1 : 2));
  const int act = epilogue == DC_EPI_GLU_GELU ? 1 : epilogue == DC_EPI_GLU_SILU ? 2 : 0;
  int rc = qgemm_direct_launch(ctx, X, W16, Y, M, N, K, act);
  dc_prof_end(ctx);
  return rc;
}

extern "C" int dc_dequant(dc_ctx *ctx, const void *Wq, const void *S, void *W16, int N, int K, int bits) {
  DC_CHECK(Wq && S && W16 && N > 0 && K > 0 && K % 32 == 0 && (bits == 4 || bits == 8), DC_EINVAL,
           "decision.js: dequant: bad arguments");
  DC_CHECK(aln(Wq, bits) && aln(S, 2) && al16(W16), DC_EINVAL,
           "decision.js: dequant: the codes must be %d-byte, the scales 2-byte and W16 16-byte aligned", bits);
  DC_PRE(ctx);
  dc_prof_begin(ctx, DC_K_OTHER, 0, (double)N * K * (2 + bits / 8.0));
  int rc = ops_dequant(ctx, Wq, S, W16, N, K, bits);
  dc_prof_end(ctx);
  return rc;
}

extern "C" int dc_add_rmsnorm(dc_ctx *ctx, void *X, const void *Yr, const void *W, void *O, int T, int H, int add,
                              float eps) {
  DC_CHECK(X && W && O && (!add || Yr), DC_EINVAL, "decision.js: add_rmsnorm: null pointer");
  DC_CHECK(T >= 0 && H > 0 && H % 8 == 0, DC_EINVAL, "decision.js: add_rmsnorm: H=%d must be a multiple of 8", H);
  DC_CHECK(al16(X) && al16(W) && al16(O) && (!add || al16(Yr)), DC_EINVAL,
           "decision.js: add_rmsnorm: X, Y, W and O must be 16-byte aligned");
  DC_PRE(ctx);
  if (T == 0) return DC_OK;
  dc_prof_begin(ctx, DC_K_NORM, 0, 2.0 * T * H * (add ? 4 : 2));
  int rc = ops_add_rmsnorm(ctx, X, Yr, W, O, T, H, add, eps);
  dc_prof_end(ctx);
  return rc;
}

extern "C" int dc_sandwich(dc_ctx *ctx, void *X, const void *Y, const void *W1, const void *W2, void *O, int T,
                           int H, float eps, float scale) {
  DC_CHECK(X && Y && W1 && (!W2 || O), DC_EINVAL, "decision.js: sandwich: null pointer");
  DC_CHECK(T >= 0 && H > 0 && H % 8 == 0, DC_EINVAL, "decision.js: sandwich: H=%d must be a multiple of 8", H);
  DC_CHECK(al16(X) && al16(Y) && al16(W1) && (!W2 || (al16(W2) && al16(O))), DC_EINVAL,
           "decision.js: sandwich: X, Y, W1, W2 and O must be 16-byte aligned");
  DC_PRE(ctx);
  if (T == 0) return DC_OK;
  dc_prof_begin(ctx, DC_K_NORM, 0, 2.0 * T * H * (W2 ? 4 : 3));
  int rc = ops_sandwich(ctx, X, Y, W1, W2, O, T, H, eps, scale);
  dc_prof_end(ctx);
  return rc;
}

extern "C" int dc_qkv_norm_rope(dc_ctx *ctx, void *Z, const void *qn, const void *kn, const int32_t *pos, int T,
                                int heads, int kv, int D, float eps, float theta, int vnorm) {
  DC_CHECK(Z && qn && kn && pos, DC_EINVAL, "decision.js: qkv_norm_rope: null pointer");
  DC_CHECK(T >= 0 && heads > 0 && kv > 0 && heads % kv == 0, DC_EINVAL,
           "decision.js: qkv_norm_rope: heads=%d must be a multiple of kv=%d", heads, kv);
  DC_CHECK(al16(Z) && al16(qn) && al16(kn) && aln(pos, 4), DC_EINVAL,
           "decision.js: qkv_norm_rope: Z and the norm weights must be 16-byte aligned, pos 4-byte");
  DC_PRE(ctx);
  if (T == 0) return DC_OK;
  dc_prof_begin(ctx, DC_K_NORM, 0, 4.0 * T * (heads + 2 * kv) * D);
  int rc = ops_qkv_norm_rope(ctx, Z, qn, kn, pos, T, heads, kv, D, eps, theta, vnorm);
  dc_prof_end(ctx);
  return rc;
}

extern "C" int dc_attention(dc_ctx *ctx, const void *Z, const int32_t *rng, void *Y, int T, int heads, int kv,
                            int D, float scale) {
  DC_CHECK(Z && rng && Y, DC_EINVAL, "decision.js: attention: null pointer");
  DC_CHECK(al16(Z) && al16(Y) && aln(rng, 4), DC_EINVAL,
           "decision.js: attention: Z and Y must be 16-byte aligned, the ranges 4-byte");
  DC_CHECK(T >= 0 && heads > 0 && kv > 0 && heads % kv == 0, DC_EINVAL,
           "decision.js: attention: heads=%d must be a multiple of kv=%d", heads, kv);
  DC_PRE(ctx);
  if (T == 0) return DC_OK;
  dc_prof_begin(ctx, DC_K_ATTN, 0, 0);
  int rc = attn_launch(ctx, Z, rng, Y, T, heads, kv, D, scale);
  dc_prof_end(ctx);
  return rc;
}

extern "C" int dc_attention_form(dc_ctx *ctx, const void *Z, const int32_t *rng, void *Y, int T, int heads, int kv,
                                 int D, float scale, int form) {
  DC_CHECK(Z && rng && Y, DC_EINVAL, "decision.js: attention: null pointer");
  DC_CHECK(al16(Z) && al16(Y) && aln(rng, 4), DC_EINVAL,
           "decision.js: attention: Z and Y must be 16-byte aligned, the ranges 4-byte");
  DC_CHECK(T >= 0 && heads > 0 && kv > 0 && heads % kv == 0, DC_EINVAL,
           "decision.js: attention: heads=%d must be a multiple of kv=%d", heads, kv);
  DC_CHECK(form == 0 || form == 1, DC_EINVAL, "decision.js: attention: form must be 0 or 1");
  DC_PRE(ctx);
  if (T == 0) return DC_OK;
  dc_prof_begin(ctx, DC_K_ATTN, 0, 0);
  int rc = attn_launch_form(ctx, Z, rng, Y, T, heads, kv, D, scale, form);
  dc_prof_end(ctx);
  return rc;
}

extern "C" int dc_attention_ex(dc_ctx *ctx, const void *Z, const int32_t *rng, void *Y, int T, int heads, int kv,
                               int D, float scale, long stride, int gate, int form) {
  DC_CHECK(Z && rng && Y, DC_EINVAL, "decision.js: attention: null pointer");
  DC_CHECK(al16(Z) && al16(Y) && aln(rng, 4), DC_EINVAL,
           "decision.js: attention: Z and Y must be 16-byte aligned, the ranges 4-byte");
  DC_CHECK(T >= 0 && heads > 0 && kv > 0 && heads % kv == 0, DC_EINVAL,
           "decision.js: attention: heads=%d must be a multiple of kv=%d", heads, kv);
  DC_CHECK(form >= -1 && form <= 1, DC_EINVAL, "decision.js: attention: form must be -1, 0 or 1");
  DC_CHECK(stride % 8 == 0 && stride >= (long)(gate ? 2 * heads + 2 * kv : heads + 2 * kv) * D, DC_EINVAL,
           "decision.js: attention: row stride %ld must be a multiple of 8 holding q | k | v%s", stride,
           gate ? " | gate" : "");
  DC_PRE(ctx);
  if (T == 0) return DC_OK;
  dc_prof_begin(ctx, DC_K_ATTN, 0, 0);
  int rc = attn_launch_ex(ctx, Z, rng, Y, T, heads, kv, D, scale, form, stride, gate ? 1 : 0);
  dc_prof_end(ctx);
  return rc;
}

extern "C" int dc_glu(dc_ctx *ctx, const void *A, void *Hh, int T, int I, int act) {
  DC_CHECK(A && Hh && T >= 0 && I > 0 && I % 8 == 0, DC_EINVAL, "decision.js: glu: bad arguments (I=%d)", I);
  DC_CHECK(act == DC_ACT_SILU || act == DC_ACT_GELU_TANH || act == DC_ACT_GELU_ERF, DC_EINVAL,
           "decision.js: glu: unknown activation %d", act);
  DC_CHECK(al16(A) && al16(Hh), DC_EINVAL, "decision.js: glu: A and H must be 16-byte aligned");
  DC_PRE(ctx);
  if (T == 0) return DC_OK;
  dc_prof_begin(ctx, DC_K_OTHER, 0, 6.0 * T * I);
  int rc = ops_glu(ctx, A, Hh, T, I, act, 0);
  dc_prof_end(ctx);
  return rc;
}

extern "C" int dc_gather(dc_ctx *ctx, const int32_t *ids, const void *Eq, const void *Es, void *X, int T, int H,
                         int bits) {
  DC_CHECK(ids && Eq && Es && X && T >= 0 && H > 0 && H % 32 == 0 && (bits == 4 || bits == 8), DC_EINVAL,
           "decision.js: gather: bad arguments");
  DC_CHECK(aln(ids, 4) && aln(Eq, bits) && aln(Es, 2) && al16(X), DC_EINVAL,
           "decision.js: gather: the codes must be %d-byte, the scales 2-byte and X 16-byte aligned", bits);
  DC_PRE(ctx);
  if (T == 0) return DC_OK;
  dc_prof_begin(ctx, DC_K_OTHER, 0, (double)T * H * (2 + bits / 8.0));
  int rc = ops_gather(ctx, ids, Eq, Es, X, T, H, bits, 0x7fffffff);
  dc_prof_end(ctx);
  return rc;
}

extern "C" int dc_pool(dc_ctx *ctx, const void *X, const int32_t *seqs, const void *W, float *out, int S, int H,
                       int N) {
  DC_CHECK(X && seqs && out && S >= 0 && H > 0 && H % 8 == 0 && H <= 6400, DC_EINVAL,
           "decision.js: pool: bad arguments (H a multiple of 8, at most 6400)");
  DC_CHECK(al16(X) && aln(seqs, 4) && aln(W, 2) && aln(out, 4), DC_EINVAL,
           "decision.js: pool: X must be 16-byte aligned, seqs and out 4-byte, W 2-byte");
  DC_PRE(ctx);
  if (S == 0) return DC_OK;
  dc_prof_begin(ctx, DC_K_OTHER, 0, 0);
  int rc = ops_pool(ctx, X, seqs, W, out, S, H, W ? N : H);
  dc_prof_end(ctx);
  return rc;
}

extern "C" int dc_leaf_logits(dc_ctx *ctx, const void *X, const int32_t *leaves, const void *W, const int32_t *ids,
                              const void *Eq, const void *Es, float *out, int L, int H, int nIds, int bits,
                              float eps) {
  DC_CHECK(X && leaves && W && ids && Eq && Es && out && L >= 0 && nIds >= 0 && H > 0 && H % 32 == 0 &&
               H <= 16384 && (bits == 4 || bits == 8),
           DC_EINVAL, "decision.js: leaf_logits: bad arguments");
  DC_CHECK(aln(X, 2) && aln(leaves, 4) && aln(W, 2) && aln(ids, 4) && aln(Es, 2) && aln(out, 4), DC_EINVAL,
           "decision.js: leaf_logits: misaligned pointer");
  DC_PRE(ctx);
  if (L == 0 || nIds == 0) return DC_OK;
  dc_prof_begin(ctx, DC_K_OTHER, 0, 0);
  int rc = ops_leaf_logits(ctx, X, leaves, W, ids, Eq, Es, out, L, H, nIds, bits, eps, 0x7fffffff, 0x7fffffff);
  dc_prof_end(ctx);
  return rc;
}

extern "C" int dc_short_conv(dc_ctx *ctx, const void *Z, const void *Wc, const int32_t *taps, void *Y, int T, int H) {
  DC_CHECK(Z && Wc && taps && Y && T >= 0 && H > 0 && H % 8 == 0, DC_EINVAL,
           "decision.js: short_conv: bad arguments (H=%d must be a multiple of 8)", H);
  DC_CHECK(al16(Z) && al16(Wc) && al16(Y) && al16(taps), DC_EINVAL,
           "decision.js: short_conv: Z, the taps' weights, Y and the tap table must be 16-byte aligned");
  DC_PRE(ctx);
  if (T == 0) return DC_OK;
  dc_prof_begin(ctx, DC_K_OTHER, 0, (double)T * H * 2 * 4 + (double)H * 6);
  int rc = ops_short_conv(ctx, Z, Wc, taps, Y, T, H);
  dc_prof_end(ctx);
  return rc;
}

extern "C" int dc_ple_mix(dc_ctx *ctx, const void *G, const void *E, const void *W, void *O, int T, int P, float eps) {
  DC_CHECK(G && E && W && O && T >= 0 && P > 0 && P % 8 == 0 && P <= 1024, DC_EINVAL,
           "decision.js: ple_mix: bad arguments (P=%d must be a multiple of 8, at most 1024)", P);
  DC_CHECK(al16(G) && al16(E) && al16(W) && al16(O), DC_EINVAL, "decision.js: ple_mix: pointers must be 16-byte aligned");
  DC_PRE(ctx);
  if (T == 0) return DC_OK;
  dc_prof_begin(ctx, DC_K_NORM, 0, 6.0 * T * P);
  int rc = ops_ple_mix(ctx, G, E, W, O, T, P, eps);
  dc_prof_end(ctx);
  return rc;
}

extern "C" int dc_readout(dc_ctx *ctx, const void *X, const float *R, const int32_t *pairs, float *out, int P, int H,
                          int T, int codes) {
  DC_CHECK(X && R && pairs && out && P >= 0 && H > 0 && H % 8 == 0 && T > 0 && codes > 0, DC_EINVAL,
           "decision.js: readout: bad arguments (H=%d must be a multiple of 8)", H);
  DC_CHECK(al16(X) && al16(R) && aln(pairs, 8) && aln(out, 4), DC_EINVAL,
           "decision.js: readout: X and R must be 16-byte aligned, the pairs 8-byte, out 4-byte");
  DC_PRE(ctx);
  if (P == 0) return DC_OK;
  dc_prof_begin(ctx, DC_K_OTHER, 0, 0);
  int rc = ops_readout(ctx, X, R, pairs, out, P, H, T, codes);
  dc_prof_end(ctx);
  return rc;
}

extern "C" int dc_gdn(dc_ctx *ctx, const void *Z, long stride, long qkv, int H, const void *W, const void *Alog,
                      const void *dt_bias, const void *gw, const uint32_t *spans, int nseq, float eps, void *Y, int T) {
  DC_CHECK(Z && W && Alog && dt_bias && gw && Y && (spans || nseq == 0) && H > 0 && nseq >= 0 && T >= 0, DC_EINVAL,
           "decision.js: gdn: bad arguments");
  DC_CHECK(qkv >= 3L * H * 128 && stride >= qkv + (long)H * 128 + 2L * H, DC_EINVAL,
           "decision.js: gdn: a row of stride %ld cannot hold q|k|v (%d heads of 128) from 0 and z|b|a from %ld",
           stride, H, qkv);
  DC_CHECK(aln(Z, 2) && aln(W, 2) && aln(Alog, 2) && aln(dt_bias, 2) && aln(gw, 2) && aln(Y, 2) &&
               (nseq == 0 || al16(spans)),
           DC_EINVAL, "decision.js: gdn: f16 tensors must be 2-byte aligned, the spans 16-byte");
  DC_PRE(ctx);
  if (nseq == 0) return DC_OK;
  dc_prof_begin(ctx, DC_K_OTHER, 0, 0);
  int rc = ops_gdn(ctx, Z, stride, qkv, H, W, Alog, dt_bias, gw, spans, nseq, eps, Y, T);
  dc_prof_end(ctx);
  return rc;
}

extern "C" int dc_add_rows(dc_ctx *ctx, const void *Xi, const int32_t *idx, const void *E, void *Xo, int T, int H,
                           int nE) {
  DC_CHECK(Xi && idx && E && Xo && T >= 0 && H > 0 && H % 8 == 0 && nE > 0, DC_EINVAL,
           "decision.js: add_rows: bad arguments (H=%d must be a multiple of 8)", H);
  DC_CHECK(al16(Xi) && al16(E) && al16(Xo) && aln(idx, 4), DC_EINVAL,
           "decision.js: add_rows: rows must be 16-byte aligned");
  DC_PRE(ctx);
  if (T == 0) return DC_OK;
  dc_prof_begin(ctx, DC_K_OTHER, 0, 6.0 * T * H);
  int rc = ops_add_rows(ctx, Xi, idx, E, Xo, T, H, nE);
  dc_prof_end(ctx);
  return rc;
}

extern "C" int dc_bias_act(dc_ctx *ctx, void *Y, const void *b, int T, int N, int act) {
  DC_CHECK(Y && b && T >= 0 && N > 0 && N % 8 == 0 && act >= 0 && act <= 2, DC_EINVAL,
           "decision.js: bias_act: bad arguments (N=%d must be a multiple of 8, act 0, 1 or 2)", N);
  DC_CHECK(al16(Y) && al16(b), DC_EINVAL, "decision.js: bias_act: Y and b must be 16-byte aligned");
  DC_PRE(ctx);
  if (T == 0) return DC_OK;
  dc_prof_begin(ctx, DC_K_OTHER, 0, 4.0 * T * N);
  int rc = ops_bias_act(ctx, Y, b, T, N, act);
  dc_prof_end(ctx);
  return rc;
}

extern "C" int dc_add_layernorm(dc_ctx *ctx, void *X, const void *Yr, const void *W, const void *B, void *O, int T,
                                int H, int add, float eps) {
  DC_CHECK(X && W && O && (!add || Yr) && T >= 0 && H > 0 && H % 8 == 0 && H <= 2048, DC_EINVAL,
           "decision.js: add_layernorm: bad arguments (H=%d must be a multiple of 8, at most 2048)", H);
  DC_CHECK(al16(X) && al16(W) && al16(O) && (!add || al16(Yr)) && (!B || al16(B)), DC_EINVAL,
           "decision.js: add_layernorm: rows must be 16-byte aligned");
  DC_PRE(ctx);
  if (T == 0) return DC_OK;
  dc_prof_begin(ctx, DC_K_NORM, 0, (add ? 6.0 : 4.0) * T * H);
  int rc = ops_add_layernorm(ctx, X, add ? Yr : nullptr, W, B, O, T, H, add, eps);
  dc_prof_end(ctx);
  return rc;
}

extern "C" int dc_gather_rows(dc_ctx *ctx, const void *X, const int32_t *rows, void *G, int M, int H, int T) {
  DC_CHECK(X && rows && G && M >= 0 && H > 0 && H % 8 == 0 && T > 0, DC_EINVAL,
           "decision.js: gather_rows: bad arguments (H=%d must be a multiple of 8)", H);
  DC_CHECK(al16(X) && al16(G) && aln(rows, 4), DC_EINVAL, "decision.js: gather_rows: rows must be 16-byte aligned");
  DC_PRE(ctx);
  if (M == 0) return DC_OK;
  dc_prof_begin(ctx, DC_K_OTHER, 0, 4.0 * M * H);
  int rc = ops_gather_rows(ctx, X, rows, G, M, H, T);
  dc_prof_end(ctx);
  return rc;
}

extern "C" int dc_score(dc_ctx *ctx, const void *Y, const void *w, const void *b, float *out, int M, int H) {
  DC_CHECK(Y && w && b && out && M >= 0 && H > 0 && H % 8 == 0, DC_EINVAL,
           "decision.js: score: bad arguments (H=%d must be a multiple of 8)", H);
  DC_CHECK(al16(Y) && al16(w) && aln(b, 2) && aln(out, 4), DC_EINVAL,
           "decision.js: score: Y and w must be 16-byte aligned");
  DC_PRE(ctx);
  if (M == 0) return DC_OK;
  dc_prof_begin(ctx, DC_K_OTHER, 0, 2.0 * M * H);
  int rc = ops_score(ctx, Y, w, b, out, M, H);
  dc_prof_end(ctx);
  return rc;
}

extern "C" int dc_qk_rope(dc_ctx *ctx, void *Z, const void *qn, const void *kn, const int32_t *pos, int T, int heads,
                          int kv, int D, long stride, int rot, int norm, float eps, float theta) {
  DC_CHECK(Z && pos && (!norm || (qn && kn)) && T >= 0 && heads > 0 && kv > 0, DC_EINVAL,
           "decision.js: qk_rope: bad arguments");
  DC_CHECK(D == 64 || D == 128 || D == 256 || D == 512, DC_EINVAL, "decision.js: qk_rope: D=%d (64, 128, 256 or 512)",
           D);
  DC_CHECK(rot >= 16 && rot <= D && rot <= 256 && (rot & (rot - 1)) == 0, DC_EINVAL,
           "decision.js: qk_rope: rot=%d must be a power of two from 16 to min(D, 256)", rot);
  DC_CHECK(stride >= (long)(heads + kv) * D && stride % 8 == 0, DC_EINVAL,
           "decision.js: qk_rope: row stride %ld must hold the q and k heads and be a multiple of 8", stride);
  DC_CHECK(al16(Z) && aln(pos, 4) && (!norm || (al16(qn) && al16(kn))), DC_EINVAL,
           "decision.js: qk_rope: Z and the norm weights must be 16-byte aligned");
  DC_PRE(ctx);
  if (T == 0) return DC_OK;
  dc_prof_begin(ctx, DC_K_NORM, 0, 4.0 * T * (heads + kv) * D);
  int rc = ops_qk_rope(ctx, Z, norm ? qn : nullptr, norm ? kn : nullptr, pos, T, heads, kv, D, stride, rot, norm, eps,
                       theta);
  dc_prof_end(ctx);
  return rc;
}

extern "C" int dc_selftest_wait(dc_ctx *ctx, int limit_us) {
  DC_CHECK(limit_us >= 1 && limit_us <= 2000000, DC_EINVAL,
           "decision.js: selftest_wait: limit_us must be 1 to 2000000 (got %d)", limit_us);
  DC_PRE(ctx);
  return ops_wait_probe(ctx, limit_us);
}
