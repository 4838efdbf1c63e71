// The EmbeddingGemma 2 typed-decision head (src/eg2-head.ts, GemmaDecisionHead), on the GPU in f32. The reference
// runs it on the host after the encoder pass; here one launch scores every question of a batch:
//   S, Q = the projections of the state's and the question's normalised embeddings
//   f    = LayerNorm(field([S, Q, S*Q]) + type_emb[type])          field = Linear(3W, W), GELU, Linear(W, W)
//   per option i (embedding o_i, O_i its projection, On_i = LayerNorm(O_i)):
//   logit_i = prior * cos(o_i, s + q) + gate * (joint * cos(f, On_i) + res_i)
//   res_i   = residual_bias + R3 . gelu(R0 [f, On_i, f * On_i, |f - On_i|] + r0 bias)
// One CTA (8 warps) per question instance: every matrix-vector product is warp-cooperative (a warp
// per output row at a time, lanes striding the row: coalesced reads of the f32 weights from L2, a shuffle sum),
// every vector lives in shared memory, and every reduction has a fixed order, so a question's logits do not depend
// on the batch it is in. GELU is the reference's: 0.5 x (1 + erf(x / sqrt 2)) with the Abramowitz-Stegun 7.1.26
// erf (|error| < 1.5e-7), as src/eg2-head.ts writes it.
#include <cuda_runtime.h>
#include <math.h>

#include "dc_internal.h"

namespace {

constexpr int HEAD_THREADS = 256;
constexpr int HEAD_WARPS = HEAD_THREADS / 32;

__device__ __forceinline__ float gelu_as(float x) {
  // erf(z) for z = x / sqrt(2) by Abramowitz & Stegun 7.1.26 (the reference's host head)
  const float z = x * 0.70710678118654752f;
  const float t = 1.0f / (1.0f + 0.3275911f * fabsf(z));
  const float y = 1.0f - ((((1.061405429f * t - 1.453152027f) * t + 1.421413741f) * t - 0.284496736f) * t +
                          0.254829592f) * t * expf(-z * z);
  return 0.5f * x * (1.0f + (z >= 0.f ? y : -y));
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// y[r] = (bias ? bias[r] : 0) + sum_k M[r * ld + col0 + k] * x[k] for r < rows, k < n (x and y in shared memory).
__device__ void matvec(float *y, const float *M, int ld, int col0, const float *x, int n, int rows,
                       const float *bias) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int r = warp; r < rows; r += HEAD_WARPS) {
    const float *row = M + (size_t)r * ld + col0;
    float acc = 0.f;
    for (int k = lane; k < n; k += 32) acc = fmaf(row[k], x[k], acc);
    acc = warp_sum(acc);
    if (lane == 0) y[r] = acc + (bias ? bias[r] : 0.f);
  }
  __syncthreads();
}

// A sum over the CTA, in a fixed order (per-warp shuffle sums, then the warps' partials in order).
__device__ float block_sum(float v, float *red) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float s = 0.f;
#pragma unroll
  for (int w = 0; w < HEAD_WARPS; w++) s += red[w];
  return s;
}

__device__ float dot_block(const float *a, const float *b, int n, float *red) {
  float v = 0.f;
  for (int i = threadIdx.x; i < n; i += HEAD_THREADS) v = fmaf(a[i], b[i], v);
  return block_sum(v, red);
}

// y = (x - mean) / sqrt(var + eps) * w + b over n values, in place allowed
__device__ void layer_norm(float *y, const float *x, const float *w, const float *b, int n, float eps, float *red) {
  float s = 0.f;
  for (int i = threadIdx.x; i < n; i += HEAD_THREADS) s += x[i];
  const float m = block_sum(s, red) / (float)n;
  float v = 0.f;
  for (int i = threadIdx.x; i < n; i += HEAD_THREADS) v += (x[i] - m) * (x[i] - m);
  const float inv = 1.0f / sqrtf(block_sum(v, red) / (float)n + eps);
  __syncthreads();
  for (int i = threadIdx.x; i < n; i += HEAD_THREADS) y[i] = (x[i] - m) * inv * w[i] + b[i];
  __syncthreads();
}

}  // namespace


namespace {

// items[6 i ..]: state row, question row, question type, first option row, option count, first output index
__global__ void __launch_bounds__(HEAD_THREADS) eg2_head_kernel(Eg2HeadW p, const float *S, const float *Qe,
                                                                const float *O, const int *items, int n_items,
                                                                int nS, int nQ, int nO, float *logits,
                                                                uint32_t *err) {
  dc_pdl_begin();
  const int it = blockIdx.x;
  if (it >= n_items) return;
  const int W = p.W, E = p.E;
  extern __shared__ float sm[];
  float *s = sm, *q = s + E, *e = q + E, *anchor = e + E;                 // 4 E
  float *Sv = anchor + E, *Qv = Sv + W, *fin = Qv + W, *f1 = fin + 3 * W;  // S, Q, [S, Q, S*Q], field hidden
  float *f2 = f1 + W, *f = f2 + W, *rf = f + W;
  float *Ov = rf + W, *on = Ov + W, *pd = on + W, *r = pd + 2 * W, *rm = r + W, *ra = rm + W;  // pd: prod | diff
  float *red = ra + W;
  const int *itm = items + 6 * it;
  int si = itm[0], qi = itm[1], ty = itm[2];
  const int o0 = itm[3], no = itm[4], out0 = itm[5];
  if (si < 0 || si >= nS || qi < 0 || qi >= nQ || ty < 0 || ty >= p.ntypes || o0 < 0 || no < 0 || o0 + no > nO) {
    if (threadIdx.x == 0 && err) atomicOr(err, (uint32_t)DC_DEVERR_TOKEN_ID);
    return;
  }
  for (int i = threadIdx.x; i < E; i += HEAD_THREADS) {
    s[i] = S[(size_t)si * E + i];
    q[i] = Qe[(size_t)qi * E + i];
    anchor[i] = s[i] + q[i];
  }
  __syncthreads();
  matvec(Sv, p.state_w, E, 0, s, E, W, p.state_b);
  matvec(Qv, p.question_w, E, 0, q, E, W, p.question_b);
  for (int i = threadIdx.x; i < W; i += HEAD_THREADS) {
    fin[i] = Sv[i];
    fin[W + i] = Qv[i];
    fin[2 * W + i] = Sv[i] * Qv[i];
  }
  __syncthreads();
  matvec(f1, p.field0_w, 3 * W, 0, fin, 3 * W, W, p.field0_b);
  for (int i = threadIdx.x; i < W; i += HEAD_THREADS) f1[i] = gelu_as(f1[i]);
  __syncthreads();
  matvec(f2, p.field3_w, W, 0, f1, W, W, p.field3_b);
  for (int i = threadIdx.x; i < W; i += HEAD_THREADS) f2[i] += p.type_emb[(size_t)ty * W + i];
  __syncthreads();
  layer_norm(f, f2, p.field_norm_w, p.field_norm_b, W, p.ln_eps, red);
  const float fnorm = sqrtf(dot_block(f, f, W, red));
  // the residual's first layer splits over its four input blocks: W_f f once per question
  matvec(rf, p.res0_w, 4 * W, 0, f, W, W, p.res0_b);
  const float an = fmaxf(sqrtf(dot_block(anchor, anchor, E, red)), 1e-12f);
  for (int j = 0; j < no; j++) {
    for (int i = threadIdx.x; i < E; i += HEAD_THREADS) e[i] = O[(size_t)(o0 + j) * E + i];
    __syncthreads();
    matvec(Ov, p.option_w, E, 0, e, E, W, p.option_b);
    layer_norm(on, Ov, p.option_norm_w, p.option_norm_b, W, p.ln_eps, red);
    const float onorm = sqrtf(dot_block(on, on, W, red));
    for (int i = threadIdx.x; i < W; i += HEAD_THREADS) {
      pd[i] = f[i] * on[i];
      pd[W + i] = fabsf(f[i] - on[i]);
    }
    __syncthreads();
    matvec(r, p.res0_w, 4 * W, W, on, W, W, nullptr);
    matvec(rm, p.res0_w, 4 * W, 2 * W, pd, W, W, nullptr);
    matvec(ra, p.res0_w, 4 * W, 3 * W, pd + W, W, W, nullptr);
    float part = 0.f;
    for (int i = threadIdx.x; i < W; i += HEAD_THREADS) part += p.res3_w[i] * gelu_as(rf[i] + r[i] + rm[i] + ra[i]);
    const float res = p.residual_bias + block_sum(part, red);
    const float fo = dot_block(f, on, W, red);
    const float joint = p.joint_scale * fo / fmaxf(fnorm * onorm, 1e-8f);
    const float enorm = fmaxf(sqrtf(dot_block(e, e, E, red)), 1e-12f);
    const float prior = p.prior_scale * (dot_block(e, anchor, E, red) / enorm) / an;
    if (threadIdx.x == 0) logits[out0 + j] = prior + p.gate * (joint + res);
    __syncthreads();
  }
}

}  // namespace

size_t eg2_head_smem(int W, int E) { return (size_t)(4 * E + 16 * W + HEAD_WARPS) * sizeof(float); }

int ops_eg2_head(dc_ctx *ctx, const Eg2HeadW &p, const float *S, const float *Q, const float *O, const int *items,
                 int n_items, int nS, int nQ, int nO, float *logits) {
  const size_t smem = eg2_head_smem(p.W, p.E);
  if (smem > 200 * 1024)
    return dc_fail(DC_EINVAL, "decision.js: eg2 head: width %d and embedding %d exceed shared memory", p.W, p.E);
  if (smem > 48 * 1024)
    DC_CUDA(cudaFuncSetAttribute(eg2_head_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  DC_CUDA(dc_launch_pdl(ctx->stream, eg2_head_kernel, dim3(n_items), dim3(HEAD_THREADS), smem, p, S, Q, O, items,
                        n_items, nS, nQ, nO, logits, ctx->d_err));
  return dc_launch_check("eg2 head");
}
