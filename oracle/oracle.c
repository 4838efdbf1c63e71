/*
 * CPU oracle for the decision.js hot path: a plain-C restatement of the reference's WGSL kernels.
 *
 * TEST INFRASTRUCTURE ONLY. This library is the checker for the CUDA path (tests/, __graft_entry__.smoke(),
 * and bench.py's cpu_baseline leg). The product path never calls it and never falls back to it.
 *
 * Storage conventions follow the reference (Jacqkues/decision.js):
 *   - activations are IEEE binary16, row-major; every reduction is f32        (src/kernels.ts:1)
 *   - q8: one byte per weight, code c in [-127,127] stored as c+128            (scripts/export_common.py:90-97)
 *   - q4: two codes per byte, low nibble first, stored as c+8                   (scripts/export_common.py:64-87)
 *   - one f16 scale per 32 weights along K: S[n*(K/32) + k/32]
 *   - dequantized weight = f16((code - Z) * scale), one rounding               (src/kernels.ts:18-20,295-296)
 * Every store the WGSL makes in f16 is rounded to _Float16 here at the same point.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

typedef _Float16 h16;

static inline float hf(uint16_t b) { h16 h; memcpy(&h, &b, 2); return (float)h; }
static inline uint16_t fh(float f) { h16 h = (h16)f; uint16_t b; memcpy(&b, &h, 2); return b; }
static inline float r16(float f) { return (float)(h16)f; }

/* The code of weight (n, k) of a q8 [N,K] or q4 [N,K] matrix.
 * q8: (Wq[(n*K+k)/4] >> ((k%4)*8)) & 255, i.e. byte n*K+k            (src/kernels.ts:295)
 * q4: (Wq[(n*K+k)/8] >> ((k%8)*4)) & 15, i.e. low nibble first         (src/kernels.ts:540) */
static inline int code_at(const uint8_t *Wq, long n, long k, long K, int bits) {
  long i = n * K + k;
  if (bits == 8) return Wq[i];
  uint8_t b = Wq[i >> 1];
  return (i & 1) ? (b >> 4) : (b & 15);
}

/* f16((code - Z) * scale): the f16 subtraction is exact and the f16 product is one rounding
 * (src/kernels.ts:20, 296, 541, 690-691). */
static inline float deq_at(const uint8_t *Wq, const uint16_t *S, long n, long k, long K, int bits) {
  int z = bits == 8 ? 128 : 8;
  return r16((float)(code_at(Wq, n, k, K, bits) - z) * hf(S[n * (K / 32) + k / 32]));
}

/* tileWeights / tileWeightsPortable without the re-layout: W16[n*K + k] = deq(W)[n,k]
 * (src/kernels.ts:528-543, 682-698). */
void or_dequant(const uint8_t *Wq, const uint16_t *S, uint16_t *W16, int N, int K, int bits) {
#pragma omp parallel for schedule(static)
  for (long n = 0; n < N; n++)
    for (long k = 0; k < K; k++) W16[n * K + k] = fh(deq_at(Wq, S, n, k, K, bits));
}

/* MATMUL_PORTABLE_Q8 / _Q4 (src/kernels.ts:445-520): Y[m,n] = f16(sum_k fma(f32(X[m,k]), f32(deq W[n,k]), acc)),
 * accumulated in f32, sequentially in k order, one rounding to f16 at the store. The dequantized matrix is
 * expanded once to f32, transposed to [K,N] so the per-row loop over n vectorises; each lane still performs
 * its own fma chain in k order, so the result equals the scalar definition bit for bit. */
void or_qmatmul_order(const uint16_t *X, const uint8_t *Wq, const uint16_t *S, uint16_t *Y, int M, int N, int K,
                      int bits, int order);
void or_qmatmul(const uint16_t *X, const uint8_t *Wq, const uint16_t *S, uint16_t *Y, int M, int N, int K, int bits) {
  or_qmatmul_order(X, Wq, S, Y, M, N, K, bits, 0);
}

/* The same with the k loop in another order: 0 = ascending (the reference's), 1 = descending. A second, equally
 * valid f32 summation order: the spread between the two measures how much a deep stack's outputs move under
 * rounding-order changes alone, which is the floor for any implementation that sums in another order. */
void or_qmatmul_order(const uint16_t *X, const uint8_t *Wq, const uint16_t *S, uint16_t *Y, int M, int N, int K,
                      int bits, int order) {
  float *WT = (float *)malloc(sizeof(float) * (size_t)K * N);
#pragma omp parallel for schedule(static)
  for (long k = 0; k < K; k++)
    for (long n = 0; n < N; n++) WT[k * N + n] = deq_at(Wq, S, n, k, K, bits);
#pragma omp parallel
  {
    float *acc = (float *)malloc(sizeof(float) * (size_t)N);
#pragma omp for schedule(dynamic, 4)
    for (long m = 0; m < M; m++) {
      for (long n = 0; n < N; n++) acc[n] = 0.0f;
      for (long i = 0; i < K; i++) {
        const long k = order ? K - 1 - i : i;
        const float x = hf(X[m * K + k]);
        const float *w = WT + k * N;
        for (long n = 0; n < N; n++) acc[n] = fmaf(x, w[n], acc[n]);
      }
      for (long n = 0; n < N; n++) Y[m * N + n] = fh(acc[n]);
    }
    free(acc);
  }
  free(WT);
}

/* ADD_RMSNORM (src/kernels.ts:24-46): optionally x += y (stored f16; the sum of squares uses the unrounded
 * f32 sum), then O = f16(f32(X) * rsqrt(mean(v^2) + eps) * w). */
void or_add_rmsnorm(uint16_t *X, const uint16_t *Yr, const uint16_t *W, uint16_t *O, int T, int H, int add, float eps) {
#pragma omp parallel for schedule(static)
  for (long t = 0; t < T; t++) {
    uint16_t *x = X + t * H;
    float ss = 0.0f;
    for (long k = 0; k < H; k++) {
      float v = hf(x[k]);
      if (add) { v += hf(Yr[t * H + k]); x[k] = fh(v); }
      ss += v * v;
    }
    float inv = 1.0f / sqrtf(ss / (float)H + eps);
    for (long k = 0; k < H; k++) O[t * H + k] = fh(hf(x[k]) * inv * hf(W[k]));
  }
}

/* SANDWICH (src/eg2-kernels.ts:18-48): x = (x + rmsnorm(y) * w1) * scale, stored f16; then, when norm2,
 * O = f16(rmsnorm(f16 x) * w2), the norm taken over the stored (rounded) residual. */
void or_sandwich(uint16_t *X, const uint16_t *Y, const uint16_t *W1, const uint16_t *W2, uint16_t *O, int T, int H,
                 int norm2, float eps, float scale) {
#pragma omp parallel for schedule(static)
  for (long t = 0; t < T; t++) {
    uint16_t *x = X + t * H;
    const uint16_t *y = Y + t * H;
    float ss = 0.0f;
    for (long k = 0; k < H; k++) { float v = hf(y[k]); ss += v * v; }
    float iy = 1.0f / sqrtf(ss / (float)H + eps);
    for (long k = 0; k < H; k++) x[k] = fh((hf(x[k]) + hf(y[k]) * iy * hf(W1[k])) * scale);
    if (norm2) {
      float s2 = 0.0f;
      for (long k = 0; k < H; k++) { float a = hf(x[k]); s2 += a * a; }
      float ix = 1.0f / sqrtf(s2 / (float)H + eps);
      for (long k = 0; k < H; k++) O[t * H + k] = fh(hf(x[k]) * ix * hf(W2[k]));
    }
  }
}

/* QKV_NORM_ROPE (src/eg2-kernels.ts:53-96) and QK_NORM_ROPE (src/kernels.ts:87-112), one definition for any
 * even head dim D. Rows of Z are [heads q | kv k | kv v] heads of D. Per head: RMSNorm over D (weighted by
 * qn for q, kn for k; v is normed plainly when vnorm, else left untouched), then rotate-half RoPE on q and k:
 * pairs (d, d + D/2), angle pos * theta^(-2d/D). In place, stored f16. */
void or_qkv_norm_rope(uint16_t *Z, const uint16_t *qn, const uint16_t *kn, const int *pos, int T, int heads, int kv,
                      int D, float eps, float theta, int vnorm) {
  const int per = heads + 2 * kv;
#pragma omp parallel for schedule(static)
  for (long th = 0; th < (long)T * per; th++) {
    long t = th / per;
    int h = (int)(th % per);
    int isQ = h < heads, isK = !isQ && h < heads + kv;
    if (!isQ && !isK && !vnorm) continue;
    uint16_t *z = Z + t * per * D + (long)h * D;
    float v[1024];
    float ss = 0.0f;
    for (int d = 0; d < D; d++) { v[d] = hf(z[d]); ss += v[d] * v[d]; }
    float inv = 1.0f / sqrtf(ss / (float)D + eps);
    for (int d = 0; d < D; d++) {
      v[d] *= inv;
      if (isQ) v[d] *= hf(qn[d]);
      else if (isK) v[d] *= hf(kn[d]);
    }
    if (isQ || isK) {
      float ps = (float)pos[t];
      for (int d = 0; d < D / 2; d++) {
        float ang = ps * (1.0f / powf(theta, (float)(2 * d) / (float)D));
        float c = cosf(ang), s = sinf(ang);
        float a = v[d], b = v[d + D / 2];
        v[d] = a * c - b * s;
        v[d + D / 2] = b * c + a * s;
      }
    }
    for (int d = 0; d < D; d++) z[d] = fh(v[d]);
  }
}

/* Attention over per-token key sets (src/kernels.ts:117-147, src/eg2-kernels.ts:104-163). Each query token t
 * reads the keys in the union of two ranges [rng[4t], rng[4t+1]) and [rng[4t+2], rng[4t+3]) (the second empty
 * for plain sequences): bidirectional = its sequence, causal = [start, t+1), a tree branch = its trunk plus its
 * own branch up to itself. GQA: query head h reads kv head h / (heads/kv). Online softmax in f32, keys in
 * increasing order, q pre-scaled by `scale`, output f16(acc / l). Y is [T, heads*D]. */
/* The same over rows of `stride` halves, and with `gate` d3-lite's gated form (src/d3-kernels.ts:174-240): the q
 * heads' gates follow the v heads in the row, Y = f16(acc / l / (1 + exp(-gate))). */
void or_attention_ex(const uint16_t *Z, const int *rng, uint16_t *Y, int T, int heads, int kv, int D, float scale,
                     long stride, int gate);
void or_attention(const uint16_t *Z, const int *rng, uint16_t *Y, int T, int heads, int kv, int D, float scale) {
  or_attention_ex(Z, rng, Y, T, heads, kv, D, scale, (long)(heads + 2 * kv) * D, 0);
}
void or_attention_ex(const uint16_t *Z, const int *rng, uint16_t *Y, int T, int heads, int kv, int D, float scale,
                     long stride, int gate) {
#pragma omp parallel for schedule(dynamic, 8)
  for (long th = 0; th < (long)T * heads; th++) {
    long t = th / heads;
    int h = (int)(th % heads), kvh = h / (heads / kv);
    float q[1024], acc[1024];
    for (int d = 0; d < D; d++) { q[d] = hf(Z[t * stride + (long)h * D + d]) * scale; acc[d] = 0.0f; }
    float m = -1e30f, l = 0.0f;
    for (int r = 0; r < 2; r++) {
      int lo = rng[4 * t + 2 * r], hi = rng[4 * t + 2 * r + 1];
      for (long k = lo; k < hi; k++) {
        const uint16_t *kp = Z + k * stride + (long)(heads + kvh) * D;
        const uint16_t *vp = kp + (long)kv * D;
        float s = 0.0f;
        for (int d = 0; d < D; d++) s += q[d] * hf(kp[d]);
        float mn = fmaxf(m, s), corr = expf(m - mn), e = expf(s - mn);
        l = l * corr + e;
        for (int d = 0; d < D; d++) acc[d] = acc[d] * corr + e * hf(vp[d]);
        m = mn;
      }
    }
    for (int d = 0; d < D; d++) {
      float o = l > 0.0f ? acc[d] / l : 0.0f;
      if (gate) o = o / (1.0f + expf(-hf(Z[t * stride + (long)(heads + 2 * kv) * D + (long)h * D + d])));
      Y[t * heads * D + (long)h * D + d] = fh(o);
    }
  }
}

/* GELU, tanh approximation as the reference writes it (src/eg2-kernels.ts:9-13). */
static inline float gelu_tanh(float x) {
  float u = 0.7978845608f * (x + 0.044715f * x * x * x);
  u = fminf(fmaxf(u, -15.0f), 15.0f);
  float e = expf(2.0f * u);
  return 0.5f * x * (1.0f + (e - 1.0f) / (e + 1.0f));
}

/* The gated unit over a fused gate|up row (SILU_MUL src/kernels.ts:49-60, GELU_MUL src/eg2-kernels.ts:166-177):
 * H[t,c] = f16(act(A[t,c]) * A[t,I+c]); act 0 = SiLU, 1 = GELU (tanh). */
/* erf by Abramowitz & Stegun 7.1.26, as src/kernels.ts:202-206 writes it; GELU = 0.5 x (1 + erf(x / sqrt 2)) */
static inline float erf_as(float x) {
  const float t = 1.0f / (1.0f + 0.3275911f * fabsf(x));
  const float y = 1.0f - ((((1.061405429f * t - 1.453152027f) * t + 1.421413741f) * t - 0.284496736f) * t +
                          0.254829592f) * t * expf(-x * x);
  return x >= 0.0f ? y : -y;
}
static inline float gelu_erf_as(float x) { return 0.5f * x * (1.0f + erf_as(x * 0.70710678f)); }

void or_glu(const uint16_t *A, uint16_t *Hh, int T, int I, int act) {
#pragma omp parallel for schedule(static)
  for (long t = 0; t < T; t++)
    for (long c = 0; c < I; c++) {
      float a = hf(A[t * 2 * I + c]), b = hf(A[t * 2 * I + I + c]);
      float g = act == 0 ? a / (1.0f + expf(-a)) : act == 1 ? gelu_tanh(a) : gelu_erf_as(a);
      Hh[t * I + c] = fh(g * b);
    }
}

/* GATHER_Q8 / GATHER_Q4 (src/kernels.ts:7-21, 293-296): X[t,:] = f16 dequantized embedding row ids[t]. */
void or_gather(const int *ids, const uint8_t *Eq, const uint16_t *Es, uint16_t *X, int T, int H, int bits) {
#pragma omp parallel for schedule(static)
  for (long t = 0; t < T; t++)
    for (long k = 0; k < H; k++) X[t * H + k] = fh(deq_at(Eq, Es, ids[t], k, H, bits));
}

/* POOL_PROJECT (src/eg2-kernels.ts:204-228): per sequence [seqs[2s], seqs[2s+1]) the f32 mean of its rows;
 * then, when W [N,H] f16 is given, out[s,:] = mean . W^T in f32; else out[s,:] = mean (N = H). */
void or_pool(const uint16_t *X, const int *seqs, const uint16_t *W, float *out, int S, int H, int N) {
#pragma omp parallel for schedule(static)
  for (long s = 0; s < S; s++) {
    int a = seqs[2 * s], b = seqs[2 * s + 1];
    float mean[8192];
    for (long k = 0; k < H; k++) {
      float acc = 0.0f;
      for (long t = a; t < b; t++) acc += hf(X[t * H + k]);
      mean[k] = acc / (float)(b - a);
    }
    if (!W) { for (long k = 0; k < H; k++) out[s * H + k] = mean[k]; continue; }
    for (long o = 0; o < N; o++) {
      float d = 0.0f;
      for (long k = 0; k < H; k++) d += mean[k] * hf(W[o * H + k]);
      out[s * N + o] = d;
    }
  }
}

/* LEAF_LOGITS (src/kernels.ts:150-185): at each readout row, the final RMSNorm (f32, not rounded), then the dot
 * with the tied embedding rows of the leaf's ids, dequantized in f32 ((code - Z) * scale, no f16 rounding). */
void or_leaf_logits(const uint16_t *X, const int *leaves, const uint16_t *W, const int *ids, const uint8_t *Eq,
                    const uint16_t *Es, float *out, int L, int H, int nIds, int bits, float eps) {
  const int z = bits == 8 ? 128 : 8;
#pragma omp parallel for schedule(static)
  for (long lf = 0; lf < L; lf++) {
    const uint16_t *x = X + (long)leaves[lf] * H;
    float normed[8192];
    float ss = 0.0f;
    for (long k = 0; k < H; k++) { float v = hf(x[k]); ss += v * v; }
    float inv = 1.0f / sqrtf(ss / (float)H + eps);
    for (long k = 0; k < H; k++) normed[k] = hf(x[k]) * inv * hf(W[k]);
    for (long j = 0; j < nIds; j++) {
      long id = ids[lf * nIds + j];
      float dot = 0.0f;
      for (long k = 0; k < H; k++)
        dot += normed[k] * ((float)(code_at(Eq, id, k, H, bits) - z) * hf(Es[id * (H / 32) + k / 32]));
      out[lf * nIds + j] = dot;
    }
  }
}

/* SHORT_CONV (src/kernels.ts:65-84): over the in-projection rows Z [T, 3H] = B | C | U,
 * Y[t,c] = f16(C[t,c] * (w0 * bu(tap0) + w1 * bu(tap1) + w2 * bu(tap2))), bu(r) = B[r,c] * U[r,c] in f32 (0 for a
 * tap of -1), the weights Wc [H, 3] f16, the taps [T, 4] (tokens read by taps 0, 1, 2). */
void or_short_conv(const uint16_t *Z, const uint16_t *Wc, const int *taps, uint16_t *Y, int T, int H) {
#pragma omp parallel for schedule(static)
  for (long t = 0; t < T; t++)
    for (long c = 0; c < H; c++) {
      float conv = 0.0f;
      for (int j = 0; j < 3; j++) {
        long r = taps[4 * t + j];
        float bu = r < 0 ? 0.0f : hf(Z[r * 3 * H + c]) * hf(Z[r * 3 * H + 2 * H + c]);
        float term = hf(Wc[c * 3 + j]) * bu;
        conv = j == 0 ? term : conv + term;
      }
      Y[t * H + c] = fh(hf(Z[t * 3 * H + H + c]) * conv);
    }
}

/* PLE_MIX (src/eg2-kernels.ts:181-200): O[t,:] = f16(gelu(G[t,:]) * E[t,:] * rsqrt(mean(E^2) + eps) * W). */
void or_ple_mix(const uint16_t *G, const uint16_t *E, const uint16_t *W, uint16_t *O, int T, int P, float eps) {
#pragma omp parallel for schedule(static)
  for (long t = 0; t < T; t++) {
    float ss = 0.0f;
    for (long k = 0; k < P; k++) { float e = hf(E[t * P + k]); ss += e * e; }
    float inv = 1.0f / sqrtf(ss / (float)P + eps);
    for (long k = 0; k < P; k++)
      O[t * P + k] = fh(gelu_tanh(hf(G[t * P + k])) * hf(E[t * P + k]) * inv * hf(W[k]));
  }
}

/* READOUT (src/d3-kernels.ts:243-260): out[k] = X[pairs[2k]] . R[pairs[2k+1]] in f32 (X f16 [*, H], R f32). */
void or_readout(const uint16_t *X, const float *R, const int *pairs, float *out, int P, int H) {
#pragma omp parallel for schedule(static)
  for (long k = 0; k < P; k++) {
    const uint16_t *x = X + (long)pairs[2 * k] * H;
    const float *r = R + (long)pairs[2 * k + 1] * H;
    float s = 0.0f;
    for (long d = 0; d < H; d++) s += hf(x[d]) * r[d];
    out[k] = s;
  }
}

/* The Gated DeltaNet mixer after the in-projection (src/d3-kernels.ts:23-149 gdnLayer, the default "ort" form), one
 * (sequence, head) at a time. Z rows (stride `stride`): q | k | v (H*128 each) | z (H*128, from `qkv`) | b (H) |
 * a (H). A sequence is span a then span b (spans[4s..]: a start, a length | write-a << 31, b start, b length);
 * sequence index v is token a0 + v below the a length, b0 + v - alen above it. Per token:
 *   x_c(v) = causal 4-tap conv of channel c within the sequence, y = f16(silu(x)) (q, k, v channels);
 *   k = y / sqrt(sum y^2 + 1e-6), q = y * (1 / sqrt(sum y^2 + 1e-6) / sqrt(128)) (f32, over the head's 128);
 *   decay = exp(-exp(A_log) softplus(a + dt_bias)) (softplus(x) = x above 20), beta = sigmoid(b);
 *   per value row i of the state S [128 x 128], on the old state: r = S_i.k, p = S_i.q, kq = k.q,
 *   delta = (v_i - decay r) beta, o_i = decay p + kq delta, S_i = decay S_i + delta k;
 *   Y[t, h*128 + d] = f16(o_d / sqrt(mean(o^2) + eps) * gw_d * silu(z_d)), the a span's tokens only when flagged.
 * Y is [T, H*128]; W the conv taps [3*H*128 channels, 4] f16; A_log, dt_bias [H] f16; gw [128] f16. */
static inline float silu_f(float x) { return x / (1.0f + expf(-x)); }

void or_gdn(const uint16_t *Z, long stride, long qkv, int H, const uint16_t *W, const uint16_t *Alog,
            const uint16_t *dtb, const uint16_t *gw, const unsigned *spans, int nseq, float eps, uint16_t *Y) {
  const long QK = (long)H * 128;
#pragma omp parallel for schedule(dynamic) collapse(2)
  for (int s = 0; s < nseq; s++)
    for (int h = 0; h < H; h++) {
      const unsigned a0 = spans[4 * s], alen = spans[4 * s + 1] & 0x7fffffffu, b0 = spans[4 * s + 2];
      const int writeA = (spans[4 * s + 1] >> 31) == 1u;
      const long end = (long)alen + spans[4 * s + 3];
      float *S = calloc(128 * 128, sizeof(float));
      float q[128], k[128], v[128], o[128];
      for (long vi = 0; vi < end; vi++) {
        const long t = vi < alen ? a0 + vi : b0 + vi - alen;
        /* conv + SiLU (f16) of the q, k and v channels */
        for (int part = 0; part < 3; part++) {
          float *dst = part == 0 ? q : part == 1 ? k : v;
          for (int c = 0; c < 128; c++) {
            const long ch = part * QK + h * 128 + c;
            float x[4];
            for (int back = 3; back >= 0; back--) {
              if (vi < back) { x[3 - back] = 0.0f; continue; }
              const long u = vi - back, tp = u < alen ? a0 + u : b0 + u - alen;
              x[3 - back] = hf(Z[tp * stride + ch]);
            }
            float y = hf(W[ch * 4]) * x[0] + hf(W[ch * 4 + 1]) * x[1] + hf(W[ch * 4 + 2]) * x[2] +
                      hf(W[ch * 4 + 3]) * x[3];
            dst[c] = r16(silu_f(y));
          }
        }
        float sq = 0.0f, sk = 0.0f;
        for (int c = 0; c < 128; c++) sq += q[c] * q[c], sk += k[c] * k[c];
        const float iq = 1.0f / sqrtf(sq + 1e-6f), ik = 1.0f / sqrtf(sk + 1e-6f);
        for (int c = 0; c < 128; c++) k[c] = k[c] * ik, q[c] = q[c] * (iq * (1.0f / sqrtf(128.0f)));
        const long zr = t * stride + qkv + QK;
        const float b = hf(Z[zr + h]), a = hf(Z[zr + H + h]) + hf(dtb[h]);
        const float sp = a > 20.0f ? a : logf(1.0f + expf(a));
        const float dec = expf(-expf(hf(Alog[h])) * sp), beta = 1.0f / (1.0f + expf(-b));
        float kq = 0.0f;
        for (int j = 0; j < 128; j++) kq += k[j] * q[j];
        for (int i = 0; i < 128; i++) {
          float *Si = S + i * 128;
          float r = 0.0f, p = 0.0f;
          for (int j = 0; j < 128; j++) r += Si[j] * k[j], p += Si[j] * q[j];
          const float delta = (v[i] - dec * r) * beta;
          o[i] = dec * p + kq * delta;
          for (int j = 0; j < 128; j++) Si[j] = Si[j] * dec + k[j] * delta;
        }
        if (vi < alen && !writeA) continue;
        float so = 0.0f;
        for (int d = 0; d < 128; d++) so += o[d] * o[d];
        const float inv = 1.0f / sqrtf(so / 128.0f + eps);
        for (int d = 0; d < 128; d++) {
          const float z = hf(Z[t * stride + qkv + h * 128 + d]);
          Y[t * QK + h * 128 + d] = fh(o[d] * inv * hf(gw[d]) * z / (1.0f + expf(-z)));
        }
      }
      free(S);
    }
}

/* ADD_ROWS (src/kernels.ts:189-201): Xo[t,k] = f16(Xi[t,k] + E[idx[t],k]). */
void or_add_rows(const uint16_t *Xi, const int *idx, const uint16_t *E, uint16_t *Xo, int T, int H) {
  for (long t = 0; t < T; t++)
    for (long k = 0; k < H; k++) Xo[t * H + k] = fh(hf(Xi[t * H + k]) + hf(E[(long)idx[t] * H + k]));
}

/* BIAS_ACT (src/kernels.ts:203-221): Y[t,n] = f16(act(Y[t,n] + b[n])), act 0 none, 1 ReLU, 2 GELU (erf). */
void or_bias_act(uint16_t *Y, const uint16_t *b, int T, int N, int act) {
  for (long i = 0; i < (long)T * N; i++) {
    float v = hf(Y[i]) + hf(b[i % N]);
    if (act == 1) v = v > 0.0f ? v : 0.0f;
    if (act == 2) v = 0.5f * v * (1.0f + erf_as(v * 0.70710678f));
    Y[i] = fh(v);
  }
}

/* ADD_LAYERNORM (src/kernels.ts:223-252): optionally X += Yr (stored f16; the sums over the unrounded f32 sum),
 * O = f16((X - mean) * rsqrt(max(E[x^2] - mean^2, 0) + eps) * W + B) over the stored X; B may be NULL (zeros). */
void or_add_layernorm(uint16_t *X, const uint16_t *Yr, const uint16_t *W, const uint16_t *B, uint16_t *O, int T, int H,
                      int add, float eps) {
  for (long t = 0; t < T; t++) {
    float a = 0.0f, q = 0.0f;
    for (long k = 0; k < H; k++) {
      float v = hf(X[t * H + k]);
      if (add) { v += hf(Yr[t * H + k]); X[t * H + k] = fh(v); }
      a += v;
      q += v * v;
    }
    const float mean = a / (float)H;
    const float var = q / (float)H - mean * mean;
    const float inv = 1.0f / sqrtf((var > 0.0f ? var : 0.0f) + eps);
    for (long k = 0; k < H; k++)
      O[t * H + k] = fh((hf(X[t * H + k]) - mean) * inv * hf(W[k]) + (B ? hf(B[k]) : 0.0f));
  }
}

/* GATHER_ROWS (src/kernels.ts:254-266): G[m,:] = X[rows[m],:]. */
void or_gather_rows(const uint16_t *X, const int *rows, uint16_t *G, int M, int H) {
  for (long m = 0; m < M; m++) memcpy(G + m * H, X + (long)rows[m] * H, sizeof(uint16_t) * H);
}

/* SCORE (src/kernels.ts:268-283): out[m] = Y[m,:] . w + b[0] in f32. */
void or_score(const uint16_t *Y, const uint16_t *w, const uint16_t *b, float *out, int M, int H) {
  for (long m = 0; m < M; m++) {
    float d = 0.0f;
    for (long k = 0; k < H; k++) d += hf(Y[m * H + k]) * hf(w[k]);
    out[m] = d + hf(b[0]);
  }
}

/* Q/K (norm +) RoPE over rows of `stride`: q heads then kv k heads of D each. With norm (d3-lite's
 * QK_NORM_ROPE_256, src/d3-kernels.ts:150-172) x = x * rsqrt(mean(x^2) + eps) * w (f32, not rounded); then the
 * first `rot` dims rotate in half-split pairs (d, d + rot/2) by pos * theta^(-2d / rot) (Laya's ROPE,
 * src/encoder-kernels.ts:5-24, is D = rot = 64 without the norm). */
void or_qk_rope(uint16_t *Z, const uint16_t *qn, const uint16_t *kn, const int *pos, int T, int heads, int kv, int D,
                long stride, int rot, int norm, float eps, float theta) {
  float *v = (float *)malloc(sizeof(float) * D);
  for (long t = 0; t < T; t++)
    for (int h = 0; h < heads + kv; h++) {
      uint16_t *base = Z + t * stride + (long)h * D;
      const uint16_t *w = h < heads ? qn : kn;
      for (int d = 0; d < D; d++) v[d] = hf(base[d]);
      if (norm) {
        float ss = 0.0f;
        for (int d = 0; d < D; d++) ss += v[d] * v[d];
        const float inv = 1.0f / sqrtf(ss / (float)D + eps);
        for (int d = 0; d < D; d++) v[d] = v[d] * inv * hf(w[d]);
      }
      for (int d = 0; d < rot / 2; d++) {
        const float ang = (float)pos[t] * powf(theta, -(float)(2 * d) / (float)rot);
        const float c = cosf(ang), s = sinf(ang), a = v[d], b = v[d + rot / 2];
        v[d] = a * c - b * s;
        v[d + rot / 2] = b * c + a * s;
      }
      for (int d = 0; d < D; d++) base[d] = fh(v[d]);
    }
  free(v);
}
