// Kernels of the reference's other layer kinds and heads, memory-bound like the norms around the matmul:
//   - SHORT_CONV (src/kernels.ts:65-84): LFM2's gated short convolution in d1-3B's conv layers,
//     y[t,c] = C[t,c] * sum_j w[c,j] * B[tap_j(t),c] * U[tap_j(t),c] over the in-projection row z = B | C | U;
//   - the causal taps of a packed forest (src/d1-3b-engine.ts:53-62), derived here from the key ranges the
//     attention layers already use, so a decoder pass needs no extra input;
//   - PLE_MIX (src/eg2-kernels.ts:181-200): EmbeddingGemma 2's per-layer-embedding gate,
//     out = gelu_tanh(gate) * rmsnorm(e) * w;
//   - READOUT (src/d3-kernels.ts:243-260): d3-lite's code readout, out[k] = X[row_k] . R[code_k] in f32.
// One warp per row (or per 8-channel group of a row), 16-byte loads and stores, f32 arithmetic in the reference's
// order with explicit roundings (no contraction into fused multiply-adds), f16 where the reference stores f16.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <math.h>

#include "dc_internal.h"

namespace {

__device__ __forceinline__ void unpack8(const uint4 &u, float (&f)[8]) {
  const __half2 *h = reinterpret_cast<const __half2 *>(&u);
#pragma unroll
  for (int j = 0; j < 4; j++) {
    const float2 v = __half22float2(h[j]);
    f[2 * j] = v.x, f[2 * j + 1] = v.y;
  }
}

__device__ __forceinline__ uint4 pack8(const float (&f)[8]) {
  uint4 u;
  __half2 *h = reinterpret_cast<__half2 *>(&u);
#pragma unroll
  for (int j = 0; j < 4; j++) h[j] = __floats2half2_rn(f[2 * j], f[2 * j + 1]);
  return u;
}

__device__ __forceinline__ uint4 ld16(const __half *p) { return *reinterpret_cast<const uint4 *>(p); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// ------------------------------------------------------------------ SHORT_CONV
// Thread = 8 channels of one token. The three tap rows are usually the two tokens before t (L1/L2 hits: the
// neighbouring threads of the same block read them too); a tap of -1 contributes 0, as bu() does in the reference.
__global__ void short_conv_kernel(const __half *Z, const __half *Wc, const int4 *taps, __half *Y, int T, int H) {
  dc_pdl_begin();
  const long i8 = (long)blockIdx.x * blockDim.x + threadIdx.x;
  const long per = H >> 3;
  if (i8 >= (long)T * per) return;
  const long t = i8 / per, c = (i8 % per) * 8;
  const int4 tp = taps[t];
  const int tap[3] = {tp.x, tp.y, tp.z};
  // the 3 taps of channels c .. c + 7: 24 halves, 48 bytes at c * 6 (16-byte aligned for c % 8 == 0)
  float w[24];
  {
    const uint4 a = ld16(Wc + c * 3), b = ld16(Wc + c * 3 + 8), d = ld16(Wc + c * 3 + 16);
    float f[8];
    unpack8(a, f);
#pragma unroll
    for (int e = 0; e < 8; e++) w[e] = f[e];
    unpack8(b, f);
#pragma unroll
    for (int e = 0; e < 8; e++) w[8 + e] = f[e];
    unpack8(d, f);
#pragma unroll
    for (int e = 0; e < 8; e++) w[16 + e] = f[e];
  }
  uint4 bq[3], uq[3];
#pragma unroll
  for (int j = 0; j < 3; j++) {
    const int r = tap[j];
    if (r >= 0 && r < T) {
      const __half *row = Z + (size_t)r * 3 * H;
      bq[j] = ld16(row + c);
      uq[j] = ld16(row + 2 * H + c);
    } else {
      bq[j] = uq[j] = make_uint4(0, 0, 0, 0);
    }
  }
  float cg[8];
  unpack8(ld16(Z + (size_t)t * 3 * H + H + c), cg);
  float conv[8];
#pragma unroll
  for (int e = 0; e < 8; e++) conv[e] = 0.f;
#pragma unroll
  for (int j = 0; j < 3; j++) {
    float b[8], u[8];
    unpack8(bq[j], b);
    unpack8(uq[j], u);
#pragma unroll
    for (int e = 0; e < 8; e++) {
      const float term = __fmul_rn(w[(e * 3) + j], __fmul_rn(b[e], u[e]));
      conv[e] = j == 0 ? term : __fadd_rn(conv[e], term);
    }
  }
  float y[8];
#pragma unroll
  for (int e = 0; e < 8; e++) y[e] = __fmul_rn(cg[e], conv[e]);
  *reinterpret_cast<uint4 *>(Y + (size_t)t * H + c) = pack8(y);
}

// Causal taps (t - 2, t - 1, t) of a packed forest from its key ranges: a token's sequence is the part of
// [x, y) then of [z, w) at or before it (a trunk token: its trunk prefix; a branch token: the whole trunk, then
// its branch up to itself), and tap j reads the token j places before it in that sequence, or nothing (-1)
// before the sequence's start. This is D13BEngine.run's `taps` (src/d1-3b-engine.ts:53-62).
__global__ void conv_taps_kernel(const int4 *rng, int4 *taps, int T) {
  dc_pdl_begin();
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= T) return;
  int4 r = rng[t];
  r.x = min(max(r.x, 0), T), r.y = min(max(r.y, r.x), T);
  r.z = min(max(r.z, 0), T), r.w = min(max(r.w, r.z), T);
  // the two parts clipped to tokens at or before t
  const int a0 = r.x, a1 = min(r.y, t + 1), b0 = r.z, b1 = min(r.w, t + 1);
  const int na = max(a1 - a0, 0), nb = max(b1 - b0, 0);
  auto back = [&](int j) -> int {
    if (j < nb) return b1 - 1 - j;
    const int k = j - nb;
    return k < na ? a1 - 1 - k : -1;
  };
  taps[t] = make_int4(back(2), back(1), t, 0);
}

// ------------------------------------------------------------------ PLE_MIX
__device__ __forceinline__ float gelu_tanh(float x) {
  // gelu_pytorch_tanh as the reference writes it (src/eg2-kernels.ts:9-13): tanh(u) = (e^2u - 1) / (e^2u + 1)
  float u = 0.7978845608f * (x + 0.044715f * x * x * x);
  u = fminf(fmaxf(u, -15.0f), 15.0f);
  const float e = expf(2.0f * u);
  return 0.5f * x * (1.0f + (e - 1.0f) / (e + 1.0f));
}

// One warp per row of P values (P a multiple of 8, at most 256 * CPL).
template <int CPL>
__global__ void ple_mix_kernel(const __half *G, const __half *E, const __half *W, __half *O, int T, int P,
                               float eps) {
  dc_pdl_begin();
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= T) return;
  const int nch = P >> 3;
  uint4 eq[CPL], gq[CPL];
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < CPL; j++) {
    const int c = lane + 32 * j;
    if (c < nch) {
      eq[j] = ld16(E + (size_t)row * P + 8 * c);
      gq[j] = ld16(G + (size_t)row * P + 8 * c);
    }
  }
#pragma unroll
  for (int j = 0; j < CPL; j++) {
    const int c = lane + 32 * j;
    if (c < nch) {
      float e[8];
      unpack8(eq[j], e);
#pragma unroll
      for (int k = 0; k < 8; k++) ss += e[k] * e[k];
    }
  }
  const float inv = rsqrtf(warp_sum(ss) / (float)P + eps);
#pragma unroll
  for (int j = 0; j < CPL; j++) {
    const int c = lane + 32 * j;
    if (c < nch) {
      float e[8], g[8], w[8], o[8];
      unpack8(eq[j], e);
      unpack8(gq[j], g);
      unpack8(ld16(W + 8 * c), w);
#pragma unroll
      for (int k = 0; k < 8; k++) o[k] = __fmul_rn(__fmul_rn(__fmul_rn(gelu_tanh(g[k]), e[k]), inv), w[k]);
      *reinterpret_cast<uint4 *>(O + (size_t)row * P + 8 * c) = pack8(o);
    }
  }
}

// ------------------------------------------------------------------ READOUT
// One warp per (row, code) pair; X f16 [*, H], R f32 [codes, H]. Rows or codes out of range read row / code 0 and
// flag the device error word.
__global__ void readout_kernel(const __half *X, const float *R, const int2 *pairs, float *out, int P, int H, int T,
                               int codes, uint32_t *err) {
  dc_pdl_begin();
  const int k = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (k >= P) return;
  int2 pr = pairs[k];
  if (pr.x < 0 || pr.x >= T || pr.y < 0 || pr.y >= codes) {
    if (lane == 0 && err) atomicOr(err, (uint32_t)DC_DEVERR_TOKEN_ID);
    pr.x = (pr.x < 0 || pr.x >= T) ? 0 : pr.x;
    pr.y = (pr.y < 0 || pr.y >= codes) ? 0 : pr.y;
  }
  const __half *x = X + (size_t)pr.x * H;
  const float *r = R + (size_t)pr.y * H;
  float s = 0.f;
  for (int d = 8 * lane; d < H; d += 256) {
    float xv[8];
    unpack8(ld16(x + d), xv);
    const float4 r0 = *reinterpret_cast<const float4 *>(r + d), r1 = *reinterpret_cast<const float4 *>(r + d + 4);
    s += xv[0] * r0.x + xv[1] * r0.y + xv[2] * r0.z + xv[3] * r0.w;
    s += xv[4] * r1.x + xv[5] * r1.y + xv[6] * r1.z + xv[7] * r1.w;
  }
  s = warp_sum(s);
  if (lane == 0) out[k] = s;
}

}  // namespace

int ops_short_conv(dc_ctx *ctx, const void *Z, const void *Wc, const int *taps, void *Y, int T, int H) {
  const long n = (long)T * (H / 8);
  DC_CUDA(dc_launch_pdl(ctx->stream, short_conv_kernel, dim3((unsigned)((n + 255) / 256)), dim3(256), 0,
                        (const __half *)Z, (const __half *)Wc, (const int4 *)taps, (__half *)Y, T, H));
  return dc_launch_check("short_conv");
}

int ops_conv_taps(dc_ctx *ctx, const int *rng, int *taps, int T) {
  DC_CUDA(dc_launch_pdl(ctx->stream, conv_taps_kernel, dim3((unsigned)((T + 255) / 256)), dim3(256), 0,
                        (const int4 *)rng, (int4 *)taps, T));
  return dc_launch_check("conv_taps");
}

int ops_ple_mix(dc_ctx *ctx, const void *G, const void *E, const void *W, void *O, int T, int P, float eps) {
  const int cpl = (P / 8 + 31) / 32;
  const dim3 grid((T + 7) / 8), block(256);
  auto g = (const __half *)G;
  auto e = (const __half *)E;
  auto w = (const __half *)W;
  auto o = (__half *)O;
  if (cpl <= 1) DC_CUDA(dc_launch_pdl(ctx->stream, ple_mix_kernel<1>, grid, block, 0, g, e, w, o, T, P, eps));
  else if (cpl <= 2) DC_CUDA(dc_launch_pdl(ctx->stream, ple_mix_kernel<2>, grid, block, 0, g, e, w, o, T, P, eps));
  else if (cpl <= 4) DC_CUDA(dc_launch_pdl(ctx->stream, ple_mix_kernel<4>, grid, block, 0, g, e, w, o, T, P, eps));
  else return dc_fail(DC_EINVAL, "decision.js: ple_mix supports widths up to 1024 (got %d)", P);
  return dc_launch_check("ple_mix");
}

int ops_readout(dc_ctx *ctx, const void *X, const float *R, const int *pairs, float *out, int P, int H, int T,
                int codes) {
  DC_CUDA(dc_launch_pdl(ctx->stream, readout_kernel, dim3((unsigned)((P + 7) / 8)), dim3(256), 0, (const __half *)X, R,
                        (const int2 *)pairs, out, P, H, T, codes, ctx->d_err));
  return dc_launch_check("readout");
}
