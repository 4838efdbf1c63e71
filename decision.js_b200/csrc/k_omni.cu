// The kernels of the d1-omni and Laya decision heads and of the backbones around them that the other kernels do not
// cover (src/kernels.ts:187-283, src/encoder-kernels.ts:5-24, src/d3-kernels.ts:150-172):
//   - ADD_ROWS:      Xo[t] = Xi[t] + E[idx[t]] (the question-type embedding);
//   - BIAS_ACT:      Y[t, n] = act(Y[t, n] + b[n]) in place, act none / ReLU / GELU (erf);
//   - ADD_LAYERNORM: optionally x += y (stored f16), then O = (x - mean) / sqrt(var + eps) * w + b (b optional);
//   - GATHER_ROWS:   G[m] = X[rows[m]] (the hidden states at the option markers);
//   - SCORE:         out[m] = Y[m] . w + b (the scorer's last Linear(H, 1)), f32;
//   - QK (norm +) RoPE over q and k heads of D in rows of any stride: an optional RMSNorm over each head with its
//     weight, then the half-split rotation of the first `rot` dims (pairs d, d + rot/2) at the token's position:
//     Laya's ROPE (D = rot = 64, no norm) and d3-lite's QK_NORM_ROPE_256 (D = 256, rot = 64, normed).
// Rows are a warp's work (or 8 values a thread's) with 16-byte accesses; f32 arithmetic in the reference's order per
// element (explicit roundings, no contraction into fused multiply-adds); the sums over a row run in a fixed order of
// their own (per-lane partials, then a shuffle tree).
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <math.h>

#include "dc_internal.h"

namespace {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

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

// ADD_ROWS (src/kernels.ts:189-201): 8 values per thread
__global__ void add_rows_kernel(const __half *Xi, const int *idx, const __half *E, __half *Xo, int T, int H, int nE,
                                uint32_t *err) {
  dc_pdl_begin();
  const long i8 = (long)blockIdx.x * blockDim.x + threadIdx.x, per = H / 8;
  if (i8 >= (long)T * per) return;
  const long t = i8 / per, c = (i8 % per) * 8;
  int r = idx[t];
  if (r < 0 || r >= nE) {
    if (c == 0) atomicOr(err, (uint32_t)DC_DEVERR_TOKEN_ID);
    r = 0;
  }
  float a[8], e[8], o[8];
  unpack8(*reinterpret_cast<const uint4 *>(Xi + t * H + c), a);
  unpack8(*reinterpret_cast<const uint4 *>(E + (long)r * H + c), e);
#pragma unroll
  for (int k = 0; k < 8; k++) o[k] = __fadd_rn(a[k], e[k]);
  *reinterpret_cast<uint4 *>(Xo + t * H + c) = pack8(o);
}

// BIAS_ACT (src/kernels.ts:203-221): 8 values per thread, in place
__global__ void bias_act_kernel(__half *Y, const __half *b, int T, int N, int act) {
  dc_pdl_begin();
  const long i8 = (long)blockIdx.x * blockDim.x + threadIdx.x, per = N / 8;
  if (i8 >= (long)T * per) return;
  const long t = i8 / per, c = (i8 % per) * 8;
  float y[8], bb[8];
  unpack8(*reinterpret_cast<const uint4 *>(Y + t * N + c), y);
  unpack8(*reinterpret_cast<const uint4 *>(b + c), bb);
#pragma unroll
  for (int k = 0; k < 8; k++) {
    float v = __fadd_rn(y[k], bb[k]);
    if (act == 1) v = fmaxf(v, 0.0f);
    if (act == 2) v = dc_gelu_erf_as(v);
    y[k] = v;
  }
  *reinterpret_cast<uint4 *>(Y + t * N + c) = pack8(y);
}

// ADD_LAYERNORM (src/kernels.ts:223-252): a warp per row, H a multiple of 8 up to 8 x 32 x 8 = 2048. The sums use
// the unrounded x (as the reference's registers hold it); the normalisation reads the stored f16 x back.
constexpr int LN_MAXC = 8;  // 16-byte chunks per lane
__global__ void add_layernorm_kernel(__half *X, const __half *Yr, const __half *W, const __half *B, __half *O, int T,
                                     int H, int add, float eps) {
  dc_pdl_begin();
  const long t = (long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (t >= T) return;
  const int nch = H / 8;
  float s1 = 0.f, s2 = 0.f;
  uint4 xs[LN_MAXC];
#pragma unroll
  for (int j = 0; j < LN_MAXC; j++) {
    const int c = lane + 32 * j;
    if (c < nch) {
      float v[8];
      unpack8(*reinterpret_cast<const uint4 *>(X + t * H + 8 * c), v);
      if (add) {
        float y[8];
        unpack8(*reinterpret_cast<const uint4 *>(Yr + t * H + 8 * c), y);
#pragma unroll
        for (int e = 0; e < 8; e++) v[e] = __fadd_rn(v[e], y[e]);
      }
#pragma unroll
      for (int e = 0; e < 8; e++) s1 = __fadd_rn(s1, v[e]), s2 = __fadd_rn(s2, __fmul_rn(v[e], v[e]));
      xs[j] = pack8(v);
      if (add) *reinterpret_cast<uint4 *>(X + t * H + 8 * c) = xs[j];
    }
  }
  s1 = warp_sum(s1);
  s2 = warp_sum(s2);
  const float mean = s1 / (float)H;
  const float inv = 1.0f / sqrtf(__fadd_rn(fmaxf(__fsub_rn(s2 / (float)H, __fmul_rn(mean, mean)), 0.0f), eps));
#pragma unroll
  for (int j = 0; j < LN_MAXC; j++) {
    const int c = lane + 32 * j;
    if (c < nch) {
      float v[8], w[8], bb[8], o[8];
      unpack8(xs[j], v);
      unpack8(*reinterpret_cast<const uint4 *>(W + 8 * c), w);
      if (B) unpack8(*reinterpret_cast<const uint4 *>(B + 8 * c), bb);
#pragma unroll
      for (int e = 0; e < 8; e++)
        o[e] = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(v[e], mean), inv), w[e]), B ? bb[e] : 0.0f);
      *reinterpret_cast<uint4 *>(O + t * H + 8 * c) = pack8(o);
    }
  }
}

// GATHER_ROWS (src/kernels.ts:254-266): 8 values per thread, bit-exact copies
__global__ void gather_rows_kernel(const __half *X, const int *rows, __half *G, int M, int H, int T, uint32_t *err) {
  dc_pdl_begin();
  const long i8 = (long)blockIdx.x * blockDim.x + threadIdx.x, per = H / 8;
  if (i8 >= (long)M * per) return;
  const long m = i8 / per, c = (i8 % per) * 8;
  int r = rows[m];
  if (r < 0 || r >= T) {
    if (c == 0) atomicOr(err, (uint32_t)DC_DEVERR_BOUNDS);
    r = 0;
  }
  *reinterpret_cast<uint4 *>(G + m * H + c) = *reinterpret_cast<const uint4 *>(X + (long)r * H + c);
}

// SCORE (src/kernels.ts:268-283): a warp per marker
__global__ void score_kernel(const __half *Y, const __half *w, const __half *b, float *out, int M, int H) {
  dc_pdl_begin();
  const long m = (long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (m >= M) return;
  float d = 0.f;
  for (int c = lane; c < H / 8; c += 32) {
    float y[8], ww[8];
    unpack8(*reinterpret_cast<const uint4 *>(Y + m * H + 8 * c), y);
    unpack8(*reinterpret_cast<const uint4 *>(w + 8 * c), ww);
#pragma unroll
    for (int e = 0; e < 8; e++) d = __fadd_rn(d, __fmul_rn(y[e], ww[e]));
  }
  d = warp_sum(d);
  if (lane == 0) out[m] = __fadd_rn(d, __half2float(b[0]));
}

// QK (norm +) RoPE: a warp per (token, head) of q or k; lane l holds dims 8 c .. 8 c + 7 of chunks c = l, l + 32, ...
// (D / 8 chunks). The rotation pairs d < rot/2 with d + rot/2: chunk c pairs with chunk c + rot/16, both among the
// first rot/8 chunks, held by lanes rot/16 apart (a power of two: one xor shuffle). Angles pos * theta^(-2d / rot),
// sine and cosine to full f32 accuracy.
template <int D>
__global__ void qk_rope_kernel(__half *Z, const __half *qn, const __half *kn, const int *pos, int T, int heads, int kv,
                               long stride, int rot, int norm, float eps, float theta) {
  dc_pdl_begin();
  constexpr int NC = D / 8;                   // 16-byte chunks per head
  constexpr int CPL = NC > 32 ? NC / 32 : 1;  // chunks per lane
  const long wid = (long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  const int per = heads + kv;
  if (wid >= (long)T * per) return;
  const long t = wid / per;
  const int h = (int)(wid % per);
  const bool isQ = h < heads;
  __half *base = Z + t * stride + (long)h * D;
  float v[CPL][8];
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < CPL; j++) {
    const int c = lane + 32 * j;
#pragma unroll
    for (int e = 0; e < 8; e++) v[j][e] = 0.f;
    if (c < NC) {
      unpack8(*reinterpret_cast<const uint4 *>(base + 8 * c), v[j]);
#pragma unroll
      for (int e = 0; e < 8; e++) ss = __fadd_rn(ss, __fmul_rn(v[j][e], v[j][e]));
    }
  }
  if (norm) {
    ss = warp_sum(ss);
    const float inv = 1.0f / sqrtf(ss / (float)D + eps);
    const __half *wn = isQ ? qn : kn;
#pragma unroll
    for (int j = 0; j < CPL; j++) {
      const int c = lane + 32 * j;
      if (c < NC) {
        float w[8];
        unpack8(*reinterpret_cast<const uint4 *>(wn + 8 * c), w);
#pragma unroll
        for (int e = 0; e < 8; e++) v[j][e] = __fmul_rn(__fmul_rn(v[j][e], inv), w[e]);
      }
    }
  }
  const int rc = rot / 8, half = rot / 16;
  const float ps = (float)pos[t];
#pragma unroll
  for (int e = 0; e < 8; e++) {
    const float partner = __shfl_xor_sync(0xffffffffu, v[0][e], half);
    if (lane < rc) {
      const bool lo = lane < half;
      const int d = 8 * (lo ? lane : lane - half) + e;
      const float ang = ps * powf(theta, -(float)(2 * d) / (float)rot);
      float sn, cs;
      sincosf(ang, &sn, &cs);
      // lo: a = v, b = partner, a c - b s; hi: b = v, a = partner, b c + a s
      v[0][e] = lo ? __fsub_rn(__fmul_rn(v[0][e], cs), __fmul_rn(partner, sn))
                   : __fadd_rn(__fmul_rn(v[0][e], cs), __fmul_rn(partner, sn));
    }
  }
#pragma unroll
  for (int j = 0; j < CPL; j++) {
    const int c = lane + 32 * j;
    if (c < NC) *reinterpret_cast<uint4 *>(base + 8 * c) = pack8(v[j]);
  }
}

}  // namespace

int ops_add_rows(dc_ctx *ctx, const void *Xi, const int *idx, const void *E, void *Xo, int T, int H, int nE) {
  const long n = (long)T * (H / 8);
  DC_CUDA(dc_launch_pdl(ctx->stream, add_rows_kernel, dim3((unsigned)((n + 255) / 256)), dim3(256), 0,
                        (const __half *)Xi, idx, (const __half *)E, (__half *)Xo, T, H, nE, ctx->d_err));
  return dc_launch_check("add_rows");
}

int ops_bias_act(dc_ctx *ctx, void *Y, const void *b, int T, int N, int act) {
  const long n = (long)T * (N / 8);
  DC_CUDA(dc_launch_pdl(ctx->stream, bias_act_kernel, dim3((unsigned)((n + 255) / 256)), dim3(256), 0, (__half *)Y,
                        (const __half *)b, T, N, act));
  return dc_launch_check("bias_act");
}

int ops_add_layernorm(dc_ctx *ctx, void *X, const void *Yr, const void *W, const void *B, void *O, int T, int H,
                      int add, float eps) {
  DC_CUDA(dc_launch_pdl(ctx->stream, add_layernorm_kernel, dim3((unsigned)((T + 7) / 8)), dim3(256), 0, (__half *)X,
                        (const __half *)Yr, (const __half *)W, (const __half *)B, (__half *)O, T, H, add, eps));
  return dc_launch_check("add_layernorm");
}

int ops_gather_rows(dc_ctx *ctx, const void *X, const int *rows, void *G, int M, int H, int T) {
  const long n = (long)M * (H / 8);
  DC_CUDA(dc_launch_pdl(ctx->stream, gather_rows_kernel, dim3((unsigned)((n + 255) / 256)), dim3(256), 0,
                        (const __half *)X, rows, (__half *)G, M, H, T, ctx->d_err));
  return dc_launch_check("gather_rows");
}

int ops_score(dc_ctx *ctx, const void *Y, const void *w, const void *b, float *out, int M, int H) {
  DC_CUDA(dc_launch_pdl(ctx->stream, score_kernel, dim3((unsigned)((M + 7) / 8)), dim3(256), 0, (const __half *)Y,
                        (const __half *)w, (const __half *)b, out, M, H));
  return dc_launch_check("score");
}

int ops_qk_rope(dc_ctx *ctx, void *Z, const void *qn, const void *kn, const int *pos, int T, int heads, int kv, int D,
                long stride, int rot, int norm, float eps, float theta) {
  const long warps = (long)T * (heads + kv);
  const dim3 grid((unsigned)((warps + 7) / 8));
#define QKR(DD)                                                                                                  \
  if (D == DD)                                                                                                   \
    DC_CUDA(dc_launch_pdl(ctx->stream, qk_rope_kernel<DD>, grid, dim3(256), 0, (__half *)Z, (const __half *)qn,  \
                          (const __half *)kn, pos, T, heads, kv, stride, rot, norm, eps, theta));
  QKR(64) QKR(128) QKR(256) QKR(512)
#undef QKR
  return dc_launch_check("qk_rope");
}
