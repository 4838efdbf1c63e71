// The Gated DeltaNet mixer of d3-lite's linear-attention layers (src/d3-kernels.ts:23-149 gdnLayer, its default
// "ort" form), after the in-projection: one CTA per (sequence, head), 256 threads, the head's 128 x 128 f32 state in
// registers (thread = value row i and half p of the key dimension: 64 floats, key index j = 2 jj + p so the two
// halves of a warp read adjacent shared words). Per chunk of 16 tokens of the sequence:
//   1. in parallel: the causal 4-tap conv + SiLU of the chunk's q, k and v channels (within the sequence, rounded
//      to f16 as the reference's stored activation is), q and k L2-normalised (q also by 128^-1/2), the gates
//      decay = exp(-exp(A_log) softplus(a + dt_bias)) and beta = sigmoid(b), and k.q, all into shared memory;
//   2. the recurrence, token by token on the old state: r = S_i.k, p = S_i.q, delta = beta (v_i - decay r),
//      o_i = decay p + (k.q) delta, S_i = decay S_i + delta k (each row's two halves meet by one shuffle);
//   3. the gated RMSNorm, Y = f16(rmsnorm(o) * w * silu(z)), a warp per token.
// A sequence is span a then span b (a shared trunk scanned again by each of its branches, written only by the
// branch flagged to, then the branch; or the whole sequence and nothing). Arithmetic is f32 in the reference's
// order per term; its sums over the 128 channels run in a fixed order of their own (per-lane partials, then a
// shuffle tree), so results match the reference to f32 rounding, and repeat bit for bit.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <math.h>

#include "dc_internal.h"

namespace {

constexpr int GDN_THREADS = 256;
constexpr int GDN_CHUNK = 16;
constexpr int GDN_D = 128;  // key and value width of a head

struct GdnArgs {
  const __half *Z;     // in-projection rows: q | k | v (H*128 each) | z (H*128) | b (H) | a (H)
  const __half *W;     // conv taps [3*H*128 channels][4]
  const __half *Alog;  // [H]
  const __half *dtb;   // [H]
  const __half *gw;    // gated norm weight [128]
  const uint4 *spans;  // per sequence: a start, a length | write-a << 31, b start, b length
  __half *Y;           // [T, H*128]
  uint32_t *err;
  long stride, qkv;
  int H, T;
  float eps;
};

__device__ __forceinline__ float silu_rn16(float y) { return __half2float(__float2half_rn(y / (1.0f + expf(-y)))); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__global__ void __launch_bounds__(GDN_THREADS, 1) gdn_kernel(GdnArgs a) {
  dc_pdl_begin();
  __shared__ float qs[GDN_CHUNK][GDN_D], ks[GDN_CHUNK][GDN_D], vs[GDN_CHUNK][GDN_D];  // vs: v, then o
  __shared__ float gdec[GDN_CHUNK], gbeta[GDN_CHUNK], gkq[GDN_CHUNK];
  const int sq = blockIdx.x / a.H, h = blockIdx.x % a.H;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint4 sp = a.spans[sq];
  const long a0 = sp.x, alen = sp.y & 0x7fffffffu, b0 = sp.z;
  const bool writeA = (sp.y >> 31) == 1u;
  const long end = alen + sp.w;
  if (a0 + alen > a.T || (sp.w > 0 && b0 + sp.w > a.T)) {
    if (threadIdx.x == 0) atomicOr(a.err, (uint32_t)DC_DEVERR_BOUNDS);
    return;
  }
  auto phys = [&](long v) { return v < alen ? a0 + v : b0 + v - alen; };
  const long QK = (long)a.H * GDN_D;
  // recurrence layout: thread = value row i, key half p (key j = 2 jj + p)
  const int row = threadIdx.x >> 1, p = threadIdx.x & 1;
  float S[GDN_D / 2];
#pragma unroll
  for (int jj = 0; jj < GDN_D / 2; jj++) S[jj] = 0.f;
  const float dscale = -expf(__half2float(a.Alog[h]));
  const float dtb = __half2float(a.dtb[h]);
  const float inv_sqrt_d = 1.0f / sqrtf((float)GDN_D);

  for (long t0 = 0; t0 < end; t0 += GDN_CHUNK) {
    const int n = (int)min((long)GDN_CHUNK, end - t0);
    // 1a. q and k: warp w takes (token, q|k) pairs w, w + 8, ...; lane = 4 channels
    for (int pr = warp; pr < 2 * GDN_CHUNK; pr += GDN_THREADS / 32) {
      const int c = pr >> 1;
      const bool isK = pr & 1;
      if (c >= n) continue;
      const long v = t0 + c;
      const long ch0 = (isK ? QK : 0) + (long)h * GDN_D + 4 * lane;
      float y[4], ss = 0.f;
#pragma unroll
      for (int e = 0; e < 4; e++) {
        const long ch = ch0 + e;
        float x[4];
#pragma unroll
        for (int back = 3; back >= 0; back--)
          x[3 - back] = v < back ? 0.f : __half2float(a.Z[phys(v - back) * a.stride + ch]);
        const float s = __fadd_rn(__fadd_rn(__fadd_rn(__fmul_rn(__half2float(a.W[ch * 4]), x[0]),
                                                      __fmul_rn(__half2float(a.W[ch * 4 + 1]), x[1])),
                                            __fmul_rn(__half2float(a.W[ch * 4 + 2]), x[2])),
                                  __fmul_rn(__half2float(a.W[ch * 4 + 3]), x[3]));
        y[e] = silu_rn16(s);
        ss = fmaf(y[e], y[e], ss);
      }
      ss = warp_sum(ss);
      const float inv = 1.0f / sqrtf(ss + 1e-6f);
#pragma unroll
      for (int e = 0; e < 4; e++) {
        if (isK) ks[c][4 * lane + e] = y[e] * inv;
        else qs[c][4 * lane + e] = y[e] * (inv * inv_sqrt_d);
      }
    }
    // 1b. v: thread = (token, channel) pairs; the gates: threads 0 .. n-1
    for (int i = threadIdx.x; i < n * GDN_D; i += GDN_THREADS) {
      const int c = i / GDN_D, d = i % GDN_D;
      const long v = t0 + c, ch = 2 * QK + (long)h * GDN_D + d;
      float x[4];
#pragma unroll
      for (int back = 3; back >= 0; back--)
        x[3 - back] = v < back ? 0.f : __half2float(a.Z[phys(v - back) * a.stride + ch]);
      const float s = __fadd_rn(__fadd_rn(__fadd_rn(__fmul_rn(__half2float(a.W[ch * 4]), x[0]),
                                                    __fmul_rn(__half2float(a.W[ch * 4 + 1]), x[1])),
                                          __fmul_rn(__half2float(a.W[ch * 4 + 2]), x[2])),
                                __fmul_rn(__half2float(a.W[ch * 4 + 3]), x[3]));
      vs[c][d] = silu_rn16(s);
    }
    if (threadIdx.x < n) {
      const long zr = phys(t0 + threadIdx.x) * a.stride + a.qkv + QK;
      const float b = __half2float(a.Z[zr + h]), av = __half2float(a.Z[zr + a.H + h]) + dtb;
      const float spl = av > 20.0f ? av : logf(1.0f + expf(av));
      gdec[threadIdx.x] = expf(dscale * spl);
      gbeta[threadIdx.x] = 1.0f / (1.0f + expf(-b));
    }
    __syncthreads();
    // 1c. k.q per token (a warp per token)
    for (int c = warp; c < n; c += GDN_THREADS / 32) {
      float kq = 0.f;
#pragma unroll
      for (int e = 0; e < 4; e++) kq = fmaf(ks[c][4 * lane + e], qs[c][4 * lane + e], kq);
      kq = warp_sum(kq);
      if (lane == 0) gkq[c] = kq;
    }
    __syncthreads();
    // 2. the recurrence
    for (int c = 0; c < n; c++) {
      const float dec = gdec[c], beta = gbeta[c], kq = gkq[c];
      float r = 0.f, pq = 0.f;
#pragma unroll
      for (int jj = 0; jj < GDN_D / 2; jj++) {
        r = fmaf(S[jj], ks[c][2 * jj + p], r);
        pq = fmaf(S[jj], qs[c][2 * jj + p], pq);
      }
      r += __shfl_xor_sync(0xffffffffu, r, 1);
      pq += __shfl_xor_sync(0xffffffffu, pq, 1);
      const float delta = (vs[c][row] - dec * r) * beta;
      const float o = dec * pq + kq * delta;
#pragma unroll
      for (int jj = 0; jj < GDN_D / 2; jj++) S[jj] = fmaf(S[jj], dec, ks[c][2 * jj + p] * delta);
      __syncwarp();
      if (p == 0) vs[c][row] = o;  // (both halves read v_i above; the pair is in one warp)
    }
    __syncthreads();
    // 3. gated RMSNorm, a warp per token
    for (int c = warp; c < n; c += GDN_THREADS / 32) {
      const long v = t0 + c;
      if (v < alen && !writeA) continue;  // a shared trunk is written by one of its branches only
      const long t = phys(v);
      float x[4], ss = 0.f;
#pragma unroll
      for (int e = 0; e < 4; e++) x[e] = vs[c][4 * lane + e], ss = fmaf(x[e], x[e], ss);
      ss = warp_sum(ss);
      const float inv = 1.0f / sqrtf(ss / (float)GDN_D + a.eps);
#pragma unroll
      for (int e = 0; e < 4; e++) {
        const int d = 4 * lane + e;
        const float z = __half2float(a.Z[t * a.stride + a.qkv + (long)h * GDN_D + d]);
        const float g = __fmul_rn(__fmul_rn(__fmul_rn(x[e], inv), __half2float(a.gw[d])), z);
        a.Y[t * QK + (long)h * GDN_D + d] = __float2half_rn(g / (1.0f + expf(-z)));
      }
    }
    __syncthreads();
  }
}

}  // namespace

int ops_gdn(dc_ctx *ctx, const void *Z, long stride, long qkv, int H, const void *W, const void *Alog, const void *dtb,
            const void *gw, const uint32_t *spans, int nseq, float eps, void *Y, int T) {
  if (nseq == 0) return DC_OK;
  GdnArgs a;
  a.Z = static_cast<const __half *>(Z);
  a.W = static_cast<const __half *>(W);
  a.Alog = static_cast<const __half *>(Alog);
  a.dtb = static_cast<const __half *>(dtb);
  a.gw = static_cast<const __half *>(gw);
  a.spans = reinterpret_cast<const uint4 *>(spans);
  a.Y = static_cast<__half *>(Y);
  a.err = ctx->d_err;
  a.stride = stride, a.qkv = qkv, a.H = H, a.T = T, a.eps = eps;
  DC_CUDA(dc_launch_pdl(ctx->stream, gdn_kernel, dim3((unsigned)(nseq * H)), dim3(GDN_THREADS), 0, a));
  return dc_launch_check("gdn");
}
