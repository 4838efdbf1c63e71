// The memory-bound kernels around the matmul: RMSNorm (+ residual), Gemma's sandwich norm, per-head q/k(/v)
// norm + RoPE, the gated activations, the embedding gather, mean pooling, the readout logits and a plain
// dequantisation. One warp per row (or per head group), 16-byte loads and stores, shuffle reductions; each
// kernel reads and writes its row once. Arithmetic follows the reference WGSL at every f16 store.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <math.h>

#include <algorithm>

#include "dc_internal.h"

namespace {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ void load8(const __half *p, float (&f)[8]) {
  uint4 u = *reinterpret_cast<const uint4 *>(p);
  const __half2 *h = reinterpret_cast<const __half2 *>(&u);
#pragma unroll
  for (int j = 0; j < 4; j++) {
    float2 v = __half22float2(h[j]);
    f[2 * j] = v.x, f[2 * j + 1] = v.y;
  }
}

__device__ __forceinline__ void store8(__half *p, const float (&f)[8]) {
  uint4 u;
  __half2 *h = reinterpret_cast<__half2 *>(&u);
#pragma unroll
  for (int j = 0; j < 4; j++) h[j] = __floats2half2_rn(f[2 * j], f[2 * j + 1]);
  *reinterpret_cast<uint4 *>(p) = u;
}

__device__ __forceinline__ float r16(float v) { return __half2float(__float2half_rn(v)); }

__device__ __forceinline__ void unpack8(const uint4 &u, float (&f)[8]) {
  const __half2 *h = reinterpret_cast<const __half2 *>(&u);
#pragma unroll
  for (int j = 0; j < 4; j++) {
    float2 v = __half22float2(h[j]);
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
__device__ __forceinline__ void st16(__half *p, const uint4 &u) { *reinterpret_cast<uint4 *>(p) = u; }

// The row kernels below take one warp per row with CPL 16-byte chunks per lane (H <= 256 * CPL). Each phase
// issues all of its loads before its first store, and the row stays in registers as packed f16 (the values the
// reference stores), so a row costs one memory round trip per phase whatever H is; a store cannot hold back a
// later load of the same row, and X may be the same buffer as O.

// ------------------------------------------------------------------ ADD_RMSNORM (src/kernels.ts:24-46)
template <int CPL>
__global__ void add_rmsnorm_kernel(__half *X, const __half *Yr, const __half *W, __half *O, int T, int H, int add,
                                   float eps) {
  dc_pdl_begin();
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= T) return;
  __half *x = X + (size_t)row * H;
  const int nch = H >> 3;
  uint4 xr[CPL], yr[CPL];
#pragma unroll
  for (int j = 0; j < CPL; j++) {
    const int c = lane + 32 * j;
    if (c < nch) {
      xr[j] = ld16(x + 8 * c);
      if (add) yr[j] = ld16(Yr + (size_t)row * H + 8 * c);
    }
  }
  // the reference sums the squares of the f32 sums and normalises the stored (f16) values
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < CPL; j++) {
    const int c = lane + 32 * j;
    if (c < nch) {
      float v[8];
      unpack8(xr[j], v);
      if (add) {
        float y[8];
        unpack8(yr[j], y);
#pragma unroll
        for (int e = 0; e < 8; e++) v[e] += y[e];
        xr[j] = pack8(v);
        st16(x + 8 * c, xr[j]);
      }
#pragma unroll
      for (int e = 0; e < 8; e++) ss += v[e] * v[e];
    }
  }
  ss = warp_sum(ss);
  const float inv = rsqrtf(ss / (float)H + eps);
  uint4 wr[CPL];
#pragma unroll
  for (int j = 0; j < CPL; j++) {
    const int c = lane + 32 * j;
    if (c < nch) wr[j] = ld16(W + 8 * c);
  }
#pragma unroll
  for (int j = 0; j < CPL; j++) {
    const int c = lane + 32 * j;
    if (c < nch) {
      float v[8], w[8], o[8];
      unpack8(xr[j], v);
      unpack8(wr[j], w);
#pragma unroll
      for (int e = 0; e < 8; e++) o[e] = v[e] * inv * w[e];
      st16(O + (size_t)row * H + 8 * c, pack8(o));
    }
  }
}

// ------------------------------------------------------------------ SANDWICH (src/eg2-kernels.ts:18-48)
template <int CPL>
__global__ void sandwich_kernel(__half *X, const __half *Y, const __half *W1, const __half *W2, __half *O, int T,
                                int H, float eps, float scale) {
  dc_pdl_begin();
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= T) return;
  const int nch = H >> 3;
  __half *x = X + (size_t)row * H;
  uint4 yr[CPL], xr[CPL], wr[CPL];
#pragma unroll
  for (int j = 0; j < CPL; j++) {
    const int c = lane + 32 * j;
    if (c < nch) {
      yr[j] = ld16(Y + (size_t)row * H + 8 * c);
      xr[j] = ld16(x + 8 * c);
      if (CPL <= 4) wr[j] = ld16(W1 + 8 * c);  // wide rows load W1 after the first reduction (registers)
    }
  }
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < CPL; j++) {
    const int c = lane + 32 * j;
    if (c < nch) {
      float y[8];
      unpack8(yr[j], y);
#pragma unroll
      for (int e = 0; e < 8; e++) ss += y[e] * y[e];
    }
  }
  ss = warp_sum(ss);
  const float iy = rsqrtf(ss / (float)H + eps);
  if (CPL > 4) {
#pragma unroll
    for (int j = 0; j < CPL; j++) {
      const int c = lane + 32 * j;
      if (c < nch) wr[j] = ld16(W1 + 8 * c);
    }
  }
  float s2 = 0.f;
#pragma unroll
  for (int j = 0; j < CPL; j++) {
    const int c = lane + 32 * j;
    if (c < nch) {
      float y[8], xv[8], w[8];
      unpack8(yr[j], y);
      unpack8(xr[j], xv);
      unpack8(wr[j], w);
#pragma unroll
      for (int e = 0; e < 8; e++) {
        y[e] = r16((xv[e] + y[e] * iy * w[e]) * scale);  // the stored residual
        s2 += y[e] * y[e];
      }
      xr[j] = pack8(y);
      st16(x + 8 * c, xr[j]);
    }
  }
  if (!W2) return;
  s2 = warp_sum(s2);
  const float ix = rsqrtf(s2 / (float)H + eps);
#pragma unroll
  for (int j = 0; j < CPL; j++) {
    const int c = lane + 32 * j;
    if (c < nch) wr[j] = ld16(W2 + 8 * c);
  }
#pragma unroll
  for (int j = 0; j < CPL; j++) {
    const int c = lane + 32 * j;
    if (c < nch) {
      float v[8], w[8], o[8];
      unpack8(xr[j], v);
      unpack8(wr[j], w);
#pragma unroll
      for (int e = 0; e < 8; e++) o[e] = v[e] * ix * w[e];
      st16(O + (size_t)row * H + 8 * c, pack8(o));
    }
  }
}

// ------------------------------------------------------------------ QKV_NORM_ROPE / QK_NORM_ROPE
// (src/eg2-kernels.ts:53-96, src/kernels.ts:87-112). A head of D values is LPH = D/16 lanes of two 16-byte chunks
// each, d = 8 li .. 8 li + 7 and the same d + D/2 (as the reference keeps d and d + D/2 in one thread), so RoPE's
// pairs sit in one lane and need no shuffle; a warp pass covers HPP = 32 / LPH heads. One warp per token
// (qkv_norm_rope_token_kernel).
template <int D>
struct QkvLanes {
  static constexpr int LPH = D / 16, CPL = 2, HPP = 32 / LPH;
  static_assert(D >= 64 && D <= 512 && (D & (D - 1)) == 0, "head dim");
};
// Norm (+ weights) and RoPE of one head chunk set held by this lane; `v` in, result in place. wq / wk: this lane's
// chunks of the q and k norm weights (the same for every head).
template <int D, int LPH, int CPL>
__device__ __forceinline__ void norm_rope_head(float (&v)[CPL][8], bool isQ, bool isK, const uint4 (&wq)[CPL],
                                               const uint4 (&wk)[CPL], int li, float eps, const float (&sn)[8],
                                               const float (&cs)[8]) {
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < CPL; j++)
#pragma unroll
    for (int e = 0; e < 8; e++) ss += v[j][e] * v[j][e];
#pragma unroll
  for (int o = LPH / 2; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const float inv = rsqrtf(ss / (float)D + eps);
#pragma unroll
  for (int j = 0; j < CPL; j++) {
    float w[8];
    unpack8(isQ ? wq[j] : wk[j], w);
#pragma unroll
    for (int e = 0; e < 8; e++) {
      v[j][e] *= inv;
      if (isQ || isK) v[j][e] *= w[e];
    }
  }
  static_assert(CPL == 2, "d and d + D/2 in one lane");
  if (isQ || isK) {
    // chunk 0 holds d = 8li + e (first half), chunk 1 holds d + D/2
#pragma unroll
    for (int e = 0; e < 8; e++) {
      const float a = v[0][e], b = v[1][e];
      v[0][e] = a * cs[e] - b * sn[e];
      v[1][e] = b * cs[e] + a * sn[e];
    }
  }
}

template <int D>
__device__ __forceinline__ void rope_angles(float ps, int li, const float *invf, float (&sn)[8], float (&cs)[8]) {
  const int d0 = 8 * li;
#pragma unroll
  for (int e = 0; e < 8; e++) __sincosf(ps * invf[d0 + e], &sn[e], &cs[e]);
}

// inverse frequencies 1 / theta^(2d/D), d < D/2, computed once per block; the angles' sine and cosine come from
// the hardware approximation, whose phase error (|angle| x 2^-24 or so, under 1e-4 at position 1024) is far
// below the f16 rounding of the result
template <int D>
__device__ __forceinline__ void fill_invf(float *invf, float theta) {
  for (int d = threadIdx.x; d < D / 2; d += blockDim.x) invf[d] = 1.0f / powf(theta, (float)(2 * d) / (float)D);
  __syncthreads();
}

// One warp per token: the heads it changes (q and k, and v when v is normed; an un-normed v is neither read nor
// written) in passes of HPP heads, NP passes at a time with all their loads in flight; the position's sines and
// cosines are computed once per lane for all of the token's heads.
template <int D, int NP>
__global__ void __launch_bounds__(256, 3) qkv_norm_rope_token_kernel(__half *Z, const __half *qn, const __half *kn, const int *pos, int T,
                                           int heads, int kv, float eps, float theta, int vnorm) {
  dc_pdl_begin();
  constexpr int LPH = QkvLanes<D>::LPH, CPL = QkvLanes<D>::CPL, HPP = QkvLanes<D>::HPP;
  __shared__ float invf[D / 2];
  fill_invf<D>(invf, theta);
  const int per = heads + 2 * kv;
  const int nproc = vnorm ? per : heads + kv;
  const int npass = (nproc + HPP - 1) / HPP;
  const int lane = threadIdx.x & 31, li = lane % LPH, sub = lane / LPH;
  const long t = (long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (t >= T) return;
  __half *zt = Z + (size_t)t * per * D;
  uint4 wq[CPL], wk[CPL];
#pragma unroll
  for (int j = 0; j < CPL; j++) wq[j] = ld16(qn + 8 * (li + LPH * j)), wk[j] = ld16(kn + 8 * (li + LPH * j));
  float sn[8], cs[8];
  for (int p0 = 0; p0 < npass; p0 += NP) {
    uint4 raw[NP][CPL];
#pragma unroll
    for (int p = 0; p < NP; p++) {
      const int h = (p0 + p) * HPP + sub;
#pragma unroll
      for (int j = 0; j < CPL; j++)
        raw[p][j] = h < nproc ? ld16(zt + (size_t)h * D + 8 * (li + LPH * j)) : make_uint4(0, 0, 0, 0);
    }
    if (p0 == 0) rope_angles<D>((float)pos[t], li, invf, sn, cs);
#pragma unroll
    for (int p = 0; p < NP; p++) {
      const int h = (p0 + p) * HPP + sub;
      const bool isQ = h < heads, isK = !isQ && h < heads + kv;
      float v[CPL][8];
#pragma unroll
      for (int j = 0; j < CPL; j++) unpack8(raw[p][j], v[j]);
      norm_rope_head<D, LPH, CPL>(v, isQ, isK, wq, wk, li, eps, sn, cs);  // every lane: it shuffles
      if (h < nproc) {
#pragma unroll
        for (int j = 0; j < CPL; j++) store8(zt + (size_t)h * D + 8 * (li + LPH * j), v[j]);
      }
    }
  }
}

// The same for tokens whose changed heads fit one group of NP passes (the encoders: q, k and v of 5 heads at
// D = 256): each warp walks tokens with a grid stride and loads the next token's heads (and position) before working
// on the current one, so its loads overlap its arithmetic.
template <int D, int NP>
__global__ void __launch_bounds__(256, 2) qkv_norm_rope_pipe_kernel(__half *Z, const __half *qn, const __half *kn,
                                                                     const int *pos, int T, int heads, int kv,
                                                                     float eps, float theta, int vnorm) {
  dc_pdl_begin();
  constexpr int LPH = QkvLanes<D>::LPH, CPL = QkvLanes<D>::CPL, HPP = QkvLanes<D>::HPP;
  __shared__ float invf[D / 2];
  __shared__ __align__(16) __half wqk[2][D];  // the q and k norm weights, read per head (registers go to the loads)
  for (int d = threadIdx.x; d < D; d += blockDim.x) wqk[0][d] = qn[d], wqk[1][d] = kn[d];
  fill_invf<D>(invf, theta);  // (its barrier also publishes wqk)
  const int per = heads + 2 * kv;
  const int nproc = vnorm ? per : heads + kv;
  const int lane = threadIdx.x & 31, li = lane % LPH, sub = lane / LPH;
  const long W = (long)gridDim.x * (blockDim.x >> 5);
  long t = (long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  auto load = [&](long tt, uint4 (&raw)[NP][CPL], int &ps) {
    const bool live = tt < T;
    const __half *zt = Z + (size_t)(live ? tt : 0) * per * D;
#pragma unroll
    for (int p = 0; p < NP; p++) {
      const int h = p * HPP + sub;
#pragma unroll
      for (int j = 0; j < CPL; j++)
        raw[p][j] = live && h < nproc ? ld16(zt + (size_t)h * D + 8 * (li + LPH * j)) : make_uint4(0, 0, 0, 0);
    }
    ps = live ? pos[tt] : 0;
  };
  uint4 cur[NP][CPL], nxt[NP][CPL];
  int pcur, pnxt;
  load(t, cur, pcur);
  for (; t < T; t += W) {
    load(t + W, nxt, pnxt);
    float sn[8], cs[8];
    rope_angles<D>((float)pcur, li, invf, sn, cs);
    __half *zt = Z + (size_t)t * per * D;
#pragma unroll
    for (int p = 0; p < NP; p++) {
      const int h = p * HPP + sub;
      const bool isQ = h < heads, isK = !isQ && h < heads + kv;
      float v[CPL][8];
#pragma unroll
      for (int j = 0; j < CPL; j++) unpack8(cur[p][j], v[j]);
      uint4 w[CPL];
#pragma unroll
      for (int j = 0; j < CPL; j++) w[j] = *reinterpret_cast<const uint4 *>(&wqk[isQ ? 0 : 1][8 * (li + LPH * j)]);
      norm_rope_head<D, LPH, CPL>(v, isQ, isK, w, w, li, eps, sn, cs);  // every lane: it shuffles
      if (h < nproc) {
#pragma unroll
        for (int j = 0; j < CPL; j++) store8(zt + (size_t)h * D + 8 * (li + LPH * j), v[j]);
      }
    }
#pragma unroll
    for (int p = 0; p < NP; p++)
#pragma unroll
      for (int j = 0; j < CPL; j++) cur[p][j] = nxt[p][j];
    pcur = pnxt;
  }
}

// ------------------------------------------------------------------ gated activations
// SILU_MUL (src/kernels.ts:49-60), GELU_MUL tanh (src/eg2-kernels.ts:166-177), GELU_MUL erf (Laya's,
// src/encoder-kernels.ts:26-44): 8 outputs per thread.
__device__ __forceinline__ float gelu_tanh(float x) {
  float u = 0.7978845608f * (x + 0.044715f * x * x * x);
  u = fminf(fmaxf(u, -15.0f), 15.0f);
  const float e = expf(2.0f * u);
  return 0.5f * x * (1.0f + (e - 1.0f) / (e + 1.0f));
}

// interleaved: A's columns alternate gate, up (the load-time layout of fused gate|up weights) instead of all
// gate columns then all up columns.
__global__ void glu_kernel(const __half *A, __half *Hh, int T, int I, int act, int interleaved) {
  dc_pdl_begin();
  const long i8 = (long)blockIdx.x * blockDim.x + threadIdx.x;
  const long per = I >> 3;
  if (i8 >= (long)T * per) return;
  const long t = i8 / per, c = (i8 % per) * 8;
  float a[8], b[8], o[8];
  if (interleaved) {
    float p0[8], p1[8];
    load8(A + t * 2 * I + 2 * c, p0);
    load8(A + t * 2 * I + 2 * c + 8, p1);
#pragma unroll
    for (int e = 0; e < 4; e++) {
      a[e] = p0[2 * e], b[e] = p0[2 * e + 1];
      a[4 + e] = p1[2 * e], b[4 + e] = p1[2 * e + 1];
    }
  } else {
    load8(A + t * 2 * I + c, a);
    load8(A + t * 2 * I + I + c, b);
  }
#pragma unroll
  for (int e = 0; e < 8; e++)
    o[e] = (act == 0 ? a[e] / (1.0f + expf(-a[e])) : act == 1 ? gelu_tanh(a[e]) : dc_gelu_erf_as(a[e])) * b[e];
  store8(Hh + t * I + c, o);
}

// ------------------------------------------------------------------ GATHER_Q8 / _Q4 (src/kernels.ts:7-21,293-296)
__global__ void gather_kernel(const int *ids, const uint8_t *Eq, const __half *Es, __half *X, int T, int H,
                              int bits, int V, uint32_t *err) {
  dc_pdl_begin();
  const long i8 = (long)blockIdx.x * blockDim.x + threadIdx.x;
  const long per = H >> 3;
  if (i8 >= (long)T * per) return;
  const long t = i8 / per, k = (i8 % per) * 8;
  long row = ids[t];
  if (row < 0 || row >= V) {  // never read outside the table: flag it, gather row 0
    if (err && k == 0) atomicOr(err, (uint32_t)DC_DEVERR_TOKEN_ID);
    row = 0;
  }
  const float s = __half2float(Es[row * (H / 32) + k / 32]);
  float o[8];
  if (bits == 8) {
    uint2 w = *reinterpret_cast<const uint2 *>(Eq + row * H + k);
    const uint8_t *b = reinterpret_cast<const uint8_t *>(&w);
#pragma unroll
    for (int e = 0; e < 8; e++) o[e] = (float)((int)b[e] - 128) * s;
  } else {
    const uint32_t w = *reinterpret_cast<const uint32_t *>(Eq + (row * H + k) / 2);
#pragma unroll
    for (int e = 0; e < 8; e++) o[e] = (float)((int)((w >> (4 * e)) & 15u) - 8) * s;
  }
  store8(X + t * H + k, o);  // one rounding of the exact product
}

// Per-token metadata of packed encoder sequences, built on the device from the sequences' [start, end):
// positions, whole-sequence key ranges and windowed key ranges (src/eg2-engine.ts:75-85). Bounds that are not
// increasing and inside [0, T) are flagged and clamped.
__global__ void encoder_meta_kernel(const int *bounds, int S, int T, int window, int *pos, int4 *full, int4 *slide,
                                    uint32_t *err) {
  dc_pdl_begin();
  const int s = blockIdx.x;
  int a = bounds[2 * s], b = bounds[2 * s + 1];
  const int prev = s > 0 ? bounds[2 * s - 1] : 0;
  if (a < prev || b <= a || b > T) {
    if (threadIdx.x == 0 && err) atomicOr(err, (uint32_t)DC_DEVERR_BOUNDS);
    a = min(max(a, 0), T);
    b = min(max(b, a), T);
  }
  for (int t = a + threadIdx.x; t < b; t += blockDim.x) {
    pos[t] = t - a;
    full[t] = make_int4(a, b, 0, 0);
    slide[t] = window > 0 ? make_int4(max(a, t - window), min(b, t + window + 1), 0, 0) : make_int4(a, b, 0, 0);
  }
}

// ------------------------------------------------------------------ dequantisation (src/kernels.ts:528-543)
__global__ void dequant_kernel(const uint8_t *Wq, const __half *S, __half *W16, int N, int K, int bits) {
  const long i8 = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i8 >= (long)N * K / 8) return;
  const long n = (i8 * 8) / K, k = (i8 * 8) % K;
  const float s = __half2float(S[n * (K / 32) + k / 32]);
  float o[8];
  if (bits == 8) {
    uint2 w = *reinterpret_cast<const uint2 *>(Wq + n * K + k);
    const uint8_t *b = reinterpret_cast<const uint8_t *>(&w);
#pragma unroll
    for (int e = 0; e < 8; e++) o[e] = (float)((int)b[e] - 128) * s;
  } else {
    const uint32_t w = *reinterpret_cast<const uint32_t *>(Wq + (n * K + k) / 2);
#pragma unroll
    for (int e = 0; e < 8; e++) o[e] = (float)((int)((w >> (4 * e)) & 15u) - 8) * s;
  }
  store8(W16 + n * K + k, o);
}

// ------------------------------------------------------------------ POOL_PROJECT (src/eg2-kernels.ts:204-228)
// One block per sequence: 8 warps split the rows, lanes own 16-byte column chunks; f32 sums, then the mean,
// then (optionally) the projection, one output column per thread.
__global__ void pool_kernel(const __half *X, const int *seqs, const __half *W, float *out, int S, int H, int N) {
  dc_pdl_begin();
  extern __shared__ float sm[];  // [8][H] partial sums, then [H] mean
  const int s = blockIdx.x;
  const int a = seqs[2 * s], b = seqs[2 * s + 1];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nch = H >> 3;
  for (int c = lane; c < nch; c += 32) {
    // warp w adds tokens a + w, a + w + 8, ... in order; eight of them are loaded at a time
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    int t = a + warp;
    for (; t + 56 < b; t += 64) {
      uint4 raw[8];
#pragma unroll
      for (int u = 0; u < 8; u++) raw[u] = ld16(X + (size_t)(t + 8 * u) * H + 8 * c);
#pragma unroll
      for (int u = 0; u < 8; u++) {
        float v[8];
        unpack8(raw[u], v);
#pragma unroll
        for (int e = 0; e < 8; e++) acc[e] += v[e];
      }
    }
    for (; t < b; t += 8) {
      float v[8];
      load8(X + (size_t)t * H + 8 * c, v);
#pragma unroll
      for (int e = 0; e < 8; e++) acc[e] += v[e];
    }
#pragma unroll
    for (int e = 0; e < 8; e++) sm[warp * H + 8 * c + e] = acc[e];
  }
  __syncthreads();
  float *mean = sm + 8 * H;
  const float inv_n = 1.0f / (float)(b - a);
  for (int k = threadIdx.x; k < H; k += blockDim.x) {
    float acc = 0.f;
#pragma unroll
    for (int w = 0; w < 8; w++) acc += sm[w * H + k];
    mean[k] = acc * inv_n;
  }
  __syncthreads();
  if (!W) {
    for (int k = threadIdx.x; k < H; k += blockDim.x) out[(size_t)s * H + k] = mean[k];
    return;
  }
  for (int o = threadIdx.x; o < N; o += blockDim.x) {
    float d = 0.f;
    for (int k = 0; k < H; k++) d += mean[k] * __half2float(W[(size_t)o * H + k]);
    out[(size_t)s * N + o] = d;
  }
}

// ------------------------------------------------------------------ LEAF_LOGITS (src/kernels.ts:150-185)
// One block per readout row: the final RMSNorm in f32 (not rounded) into shared memory, then one warp per id.
__global__ void leaf_logits_kernel(const __half *X, const int *leaves, const __half *W, const int *ids,
                                   const uint8_t *Eq, const __half *Es, float *out, int H, int nIds, int bits,
                                   float eps, int T, int V, uint32_t *err) {
  dc_pdl_begin();
  extern __shared__ float normed[];
  __shared__ float part[32];
  const int lf = blockIdx.x;
  int row = leaves[lf];
  if (row < 0 || row >= T) {  // never read outside the activations: flag it, read row 0
    if (threadIdx.x == 0 && err) atomicOr(err, (uint32_t)DC_DEVERR_TOKEN_ID);
    row = 0;
  }
  const __half *x = X + (size_t)row * H;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  float ss = 0.f;
  for (int k = threadIdx.x; k < H; k += blockDim.x) {
    const float v = __half2float(x[k]);
    ss += v * v;
  }
  ss = warp_sum(ss);
  if (lane == 0) part[warp] = ss;
  __syncthreads();
  if (warp == 0) {
    float v = lane < nw ? part[lane] : 0.f;
    v = warp_sum(v);
    if (lane == 0) part[0] = v;
  }
  __syncthreads();
  const float inv = rsqrtf(part[0] / (float)H + eps);
  for (int k = threadIdx.x; k < H; k += blockDim.x) normed[k] = __half2float(x[k]) * inv * __half2float(W[k]);
  __syncthreads();
  const int z = bits == 8 ? 128 : 8;
  for (int j = warp; j < nIds; j += nw) {
    long id = ids[(size_t)lf * nIds + j];
    if (id < 0 || id >= V) {
      if (lane == 0 && err) atomicOr(err, (uint32_t)DC_DEVERR_TOKEN_ID);
      id = 0;
    }
    float dot = 0.f;
    for (int k = lane; k < H; k += 32) {
      int code;
      if (bits == 8) code = Eq[id * H + k];
      else {
        const uint8_t byte = Eq[(id * H + k) >> 1];
        code = ((id * H + k) & 1) ? (byte >> 4) : (byte & 15);
      }
      dot += normed[k] * ((float)(code - z) * __half2float(Es[id * (H / 32) + k / 32]));
    }
    dot = warp_sum(dot);
    if (lane == 0) out[(size_t)lf * nIds + j] = dot;
  }
}

}  // namespace

// ------------------------------------------------------------------ host launchers

#define DC_ROWS_LAUNCH(KERNEL, CPLV, ...)                                                                  \
  DC_CUDA(dc_launch_pdl(ctx->stream, KERNEL<CPLV>, dim3((T + 7) / 8), dim3(256), 0, __VA_ARGS__))

int ops_add_rmsnorm(dc_ctx *ctx, void *X, const void *Yr, const void *W, void *O, int T, int H, int add,
                    float eps) {
  const int cpl = (H / 8 + 31) / 32;
  auto x = (__half *)X;
  auto y = (const __half *)Yr;
  auto w = (const __half *)W;
  auto o = (__half *)O;
  if (cpl <= 1) DC_ROWS_LAUNCH(add_rmsnorm_kernel, 1, x, y, w, o, T, H, add, eps);
  else if (cpl <= 2) DC_ROWS_LAUNCH(add_rmsnorm_kernel, 2, x, y, w, o, T, H, add, eps);
  else if (cpl <= 3) DC_ROWS_LAUNCH(add_rmsnorm_kernel, 3, x, y, w, o, T, H, add, eps);
  else if (cpl <= 4) DC_ROWS_LAUNCH(add_rmsnorm_kernel, 4, x, y, w, o, T, H, add, eps);
  else if (cpl <= 8) DC_ROWS_LAUNCH(add_rmsnorm_kernel, 8, x, y, w, o, T, H, add, eps);
  else if (cpl <= 12) DC_ROWS_LAUNCH(add_rmsnorm_kernel, 12, x, y, w, o, T, H, add, eps);
  else if (cpl <= 16) DC_ROWS_LAUNCH(add_rmsnorm_kernel, 16, x, y, w, o, T, H, add, eps);
  else return dc_fail(DC_EINVAL, "decision.js: rmsnorm supports H <= 4096 (got %d)", H);
  return dc_launch_check("add_rmsnorm");
}

int ops_sandwich(dc_ctx *ctx, void *X, const void *Y, const void *W1, const void *W2, void *O, int T, int H,
                 float eps, float scale) {
  const int cpl = (H / 8 + 31) / 32;
  auto x = (__half *)X;
  auto y = (const __half *)Y;
  auto w1 = (const __half *)W1;
  auto w2 = (const __half *)W2;
  auto o = (__half *)O;
  if (cpl <= 1) DC_ROWS_LAUNCH(sandwich_kernel, 1, x, y, w1, w2, o, T, H, eps, scale);
  else if (cpl <= 2) DC_ROWS_LAUNCH(sandwich_kernel, 2, x, y, w1, w2, o, T, H, eps, scale);
  else if (cpl <= 3) DC_ROWS_LAUNCH(sandwich_kernel, 3, x, y, w1, w2, o, T, H, eps, scale);
  else if (cpl <= 4) DC_ROWS_LAUNCH(sandwich_kernel, 4, x, y, w1, w2, o, T, H, eps, scale);
  else if (cpl <= 8) DC_ROWS_LAUNCH(sandwich_kernel, 8, x, y, w1, w2, o, T, H, eps, scale);
  else if (cpl <= 12) DC_ROWS_LAUNCH(sandwich_kernel, 12, x, y, w1, w2, o, T, H, eps, scale);
  else if (cpl <= 16) DC_ROWS_LAUNCH(sandwich_kernel, 16, x, y, w1, w2, o, T, H, eps, scale);
  else return dc_fail(DC_EINVAL, "decision.js: sandwich norm supports H <= 4096 (got %d)", H);
  return dc_launch_check("sandwich");
}

namespace {
template <int D, int NP>
int qkv_launch1(dc_ctx *ctx, __half *z, const __half *q, const __half *k, const int *pos, int T, int heads, int kv,
                float eps, float theta, int vnorm, bool one_group) {
  if (one_group) {
    // the pipelined form: two blocks of 8 warps per SM, each warp several tokens
    const int sms = ctx->sms > 0 ? ctx->sms : 148;
    const unsigned blocks = (unsigned)std::min<long>((T + 7) / 8, 2L * sms);
    DC_CUDA(dc_launch_pdl(ctx->stream, qkv_norm_rope_pipe_kernel<D, NP>, dim3(blocks), dim3(256), 0, z, q, k, pos, T,
                          heads, kv, eps, theta, vnorm));
    return DC_OK;
  }
  DC_CUDA(dc_launch_pdl(ctx->stream, qkv_norm_rope_token_kernel<D, NP>, dim3((unsigned)((T + 7) / 8)), dim3(256), 0, z,
                        q, k, pos, T, heads, kv, eps, theta, vnorm));
  return DC_OK;
}

// NP = the passes a token needs, up to 3 (a pass is 1 KB per warp in flight; three blocks of 8 warps per SM fit
// the registers of 3 passes); more passes loop in groups of about equal size
template <int D>
int qkv_launch(dc_ctx *ctx, __half *z, const __half *q, const __half *k, const int *pos, int T, int heads, int kv,
               float eps, float theta, int vnorm) {
  constexpr int HPP = QkvLanes<D>::HPP;
  const int nproc = vnorm ? heads + 2 * kv : heads + kv;
  const int np = (nproc + HPP - 1) / HPP;
  const int groups = (np + 2) / 3, g = (np + groups - 1) / groups;
  const bool one = groups == 1;
  if (g <= 1) return qkv_launch1<D, 1>(ctx, z, q, k, pos, T, heads, kv, eps, theta, vnorm, one);
  if (g <= 2) return qkv_launch1<D, 2>(ctx, z, q, k, pos, T, heads, kv, eps, theta, vnorm, one);
  return qkv_launch1<D, 3>(ctx, z, q, k, pos, T, heads, kv, eps, theta, vnorm, one);
}
}  // namespace

int ops_qkv_norm_rope(dc_ctx *ctx, void *Z, const void *qn, const void *kn, const int *pos, int T, int heads,
                      int kv, int D, float eps, float theta, int vnorm) {
  auto z = (__half *)Z;
  auto q = (const __half *)qn;
  auto k = (const __half *)kn;
  int rc;
  if (D == 64) rc = qkv_launch<64>(ctx, z, q, k, pos, T, heads, kv, eps, theta, vnorm);
  else if (D == 128) rc = qkv_launch<128>(ctx, z, q, k, pos, T, heads, kv, eps, theta, vnorm);
  else if (D == 256) rc = qkv_launch<256>(ctx, z, q, k, pos, T, heads, kv, eps, theta, vnorm);
  else if (D == 512) rc = qkv_launch<512>(ctx, z, q, k, pos, T, heads, kv, eps, theta, vnorm);
  else return dc_fail(DC_EINVAL, "decision.js: head dim %d unsupported (64, 128, 256, 512)", D);
  if (rc) return rc;
  return dc_launch_check("qkv_norm_rope");
}

int ops_glu(dc_ctx *ctx, const void *A, void *Hh, int T, int I, int act, int interleaved) {
  const long n = (long)T * (I / 8);
  DC_CUDA(dc_launch_pdl(ctx->stream, glu_kernel, dim3((unsigned)((n + 255) / 256)), dim3(256), 0, (const __half *)A,
                        (__half *)Hh, T, I, act, interleaved));
  return dc_launch_check("glu");
}

int ops_gather(dc_ctx *ctx, const int *ids, const void *Eq, const void *Es, void *X, int T, int H, int bits,
               int V) {
  const long n = (long)T * (H / 8);
  DC_CUDA(dc_launch_pdl(ctx->stream, gather_kernel, dim3((unsigned)((n + 255) / 256)), dim3(256), 0, ids,
                        (const uint8_t *)Eq, (const __half *)Es, (__half *)X, T, H, bits, V, ctx->d_err));
  return dc_launch_check("gather");
}

int ops_encoder_meta(dc_ctx *ctx, const int *bounds, int S, int T, int window, int *pos, int *full, int *slide) {
  DC_CUDA(dc_launch_pdl(ctx->stream, encoder_meta_kernel, dim3(S), dim3(256), 0, bounds, S, T, window, pos,
                        (int4 *)full, (int4 *)slide, ctx->d_err));
  return dc_launch_check("encoder_meta");
}

int ops_dequant(dc_ctx *ctx, const void *Wq, const void *S, void *W16, int N, int K, int bits) {
  const long n = (long)N * K / 8;
  dequant_kernel<<<(unsigned)((n + 255) / 256), 256, 0, ctx->stream>>>((const uint8_t *)Wq, (const __half *)S,
                                                                       (__half *)W16, N, K, bits);
  return dc_launch_check("dequant");
}

int ops_pool(dc_ctx *ctx, const void *X, const int *seqs, const void *W, float *out, int S, int H, int N) {
  // eight warps' partial sums and the mean, 9 H floats, within a CTA's 227 KB of shared memory
  if (H > 6400) return dc_fail(DC_EINVAL, "decision.js: pool supports H <= 6400 (got %d)", H);
  const size_t smem = (size_t)9 * H * sizeof(float);
  if (smem > 48 * 1024) DC_CUDA(cudaFuncSetAttribute(pool_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  DC_CUDA(dc_launch_pdl(ctx->stream, pool_kernel, dim3(S), dim3(256), smem, (const __half *)X, seqs, (const __half *)W,
                        out, S, H, N));
  return dc_launch_check("pool");
}

int ops_leaf_logits(dc_ctx *ctx, const void *X, const int *leaves, const void *W, const int *ids, const void *Eq,
                    const void *Es, float *out, int L, int H, int nIds, int bits, float eps, int T, int V) {
  const size_t smem = (size_t)H * sizeof(float);
  if (smem > 48 * 1024)
    DC_CUDA(cudaFuncSetAttribute(leaf_logits_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  DC_CUDA(dc_launch_pdl(ctx->stream, leaf_logits_kernel, dim3(L), dim3(256), smem, (const __half *)X, leaves,
                        (const __half *)W, ids, (const uint8_t *)Eq, (const __half *)Es, out, H, nIds, bits, eps, T, V,
                        ctx->d_err));
  return dc_launch_check("leaf_logits");
}

// Load-time re-layout of a fused gate|up weight [2I rows]: output row 2i takes gate row i and row 2i + 1 up row
// I + i, so the gate and up rows of every output sit side by side (a lane pair of the gated GEMM epilogue).
__global__ void interleave_rows_kernel(const uint8_t *src, uint8_t *dst, long rows, long row_bytes, long I) {
  const long r = blockIdx.x;
  const long from = (r & 1) ? I + (r >> 1) : (r >> 1);
  for (long b = threadIdx.x; b < row_bytes; b += blockDim.x) dst[r * row_bytes + b] = src[from * row_bytes + b];
}

int ops_interleave_rows(dc_ctx *ctx, const void *src, void *dst, long rows, long row_bytes) {
  interleave_rows_kernel<<<(unsigned)rows, 128, 0, ctx->stream>>>((const uint8_t *)src, (uint8_t *)dst, rows,
                                                                   row_bytes, rows / 2);
  return dc_launch_check("interleave_rows");
}
