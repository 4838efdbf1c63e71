// Attention over packed sequences with per-token key sets (src/eg2-kernels.ts:104-163 `attention`,
// src/kernels.ts:117-147 `ATTENTION`): query token t reads the keys of [lo0, hi0) union [lo1, hi1) — its whole
// sequence (bidirectional), its causal prefix, a window, or a tree branch's trunk plus its own branch. GQA.
//
// A block takes 64 query tokens of one query head (4 warps x 16 rows); keys and values stream through shared
// memory 64 at a time over the union of the tile's key ranges; scores and P.V run on f16 tensor-core MMAs
// (m16n8k16, f32 accumulation) with an online softmax in f32 (exp2 of log2e-scaled scores). P is rounded to
// f16 for the P.V product. Head dims 64, 128, 256 and 512; at D = 512 (EmbeddingGemma 2's full-attention layers,
// src/eg2-kernels.ts:104) a block writes one 256-wide half of the output head (grid z), computing the full
// 512-wide scores, so its accumulators stay at 128 floats per thread.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <float.h>

#include "dc_internal.h"
#include "dc_ptx.cuh"

using dcx::ex2_approx;

namespace {

constexpr int QT = 64;  // queries per block
constexpr int KT = 64;  // keys per tile

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack_h2(float a, float b) {
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t *>(&h);
}

// Key ranges are clamped to [0, T): a malformed range reads no memory outside the packed tokens.
__device__ __forceinline__ int4 clamp_rng(int4 r, int T) {
  r.x = min(max(r.x, 0), T), r.y = min(max(r.y, 0), T);
  r.z = min(max(r.z, 0), T), r.w = min(max(r.w, 0), T);
  return r;
}

// DV: output columns per block (D, or 256 at D = 512); blockIdx.z picks which DV-wide part of the head.
template <int D, int DV>
__global__ void __launch_bounds__(128, 2)
    attention_kernel(const __half *Z, const int4 *rng, __half *Y, int T, int heads, int kv, float scale_log2,
                     long zstride, int gate) {
  constexpr int PITCH = D * 2 + 16;    // bytes per Q / K smem row (padding breaks ldmatrix bank conflicts)
  constexpr int VPITCH = DV * 2 + 16;  // bytes per V smem row
  constexpr int NT = DV / 8;           // output n-tiles per warp
  static_assert(D % DV == 0 && NT % 2 == 0, "head split");
  extern __shared__ __align__(16) uint8_t sm[];
  uint8_t *sQ = sm;
  uint8_t *sK = sQ + QT * PITCH;
  uint8_t *sV = sK + KT * PITCH;
  __shared__ int s_kmin, s_kmax;

  const int h = blockIdx.y, t0 = blockIdx.x * QT, dv0 = blockIdx.z * DV;
  const int kvh = h / (heads / kv);
  const size_t stride = (size_t)zstride;  // elements per token row of Z: q | k | v heads (| gate heads | padding)
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, tq = lane & 3;

  if (tid == 0) { s_kmin = 0x7fffffff; s_kmax = -1; }
  __syncthreads();
  if (tid < QT && t0 + tid < T) {
    const int4 r = clamp_rng(rng[t0 + tid], T);
    int lo = 0x7fffffff, hi = -1;
    if (r.y > r.x) lo = min(lo, r.x), hi = max(hi, r.y);
    if (r.w > r.z) lo = min(lo, r.z), hi = max(hi, r.w);
    if (hi >= 0) { atomicMin(&s_kmin, lo); atomicMax(&s_kmax, hi); }
  }
  // Q tile: 64 rows x D
  constexpr int CH = D / 8;  // 16-byte chunks per row
  for (int i = tid; i < QT * CH; i += 128) {
    const int r = i / CH, c = i % CH;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (t0 + r < T) v = *reinterpret_cast<const uint4 *>(Z + (size_t)(t0 + r) * stride + (size_t)h * D + 8 * c);
    *reinterpret_cast<uint4 *>(sQ + r * PITCH + 16 * c) = v;
  }
  __syncthreads();
  const int kmin = s_kmin, kmax = s_kmax;

  // this thread's two query rows: warp*16 + g and + 8
  int4 myr[2];
#pragma unroll
  for (int i = 0; i < 2; i++) {
    const int t = t0 + warp * 16 + g + 8 * i;
    myr[i] = t < T ? clamp_rng(rng[t], T) : make_int4(0, 0, 0, 0);
  }

  float o[NT][4];
#pragma unroll
  for (int j = 0; j < NT; j++) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
  float m_i[2] = {-FLT_MAX, -FLT_MAX}, l_i[2] = {0.f, 0.f};

  const uint32_t sQa = (uint32_t)__cvta_generic_to_shared(sQ);
  const uint32_t sKa = (uint32_t)__cvta_generic_to_shared(sK);
  const uint32_t sVa = (uint32_t)__cvta_generic_to_shared(sV);

  for (int kc = kmin; kc < kmax; kc += KT) {
    __syncthreads();  // previous tile fully consumed
    for (int i = tid; i < KT * CH; i += 128) {
      const int r = i / CH, c = i % CH;
      const int k = kc + r;
      uint4 kv4 = make_uint4(0, 0, 0, 0);
      if (k < kmax) kv4 = *reinterpret_cast<const uint4 *>(Z + (size_t)k * stride + (size_t)(heads + kvh) * D + 8 * c);
      *reinterpret_cast<uint4 *>(sK + r * PITCH + 16 * c) = kv4;
    }
    constexpr int VCH = DV / 8;
    for (int i = tid; i < KT * VCH; i += 128) {
      const int r = i / VCH, c = i % VCH;
      const int k = kc + r;
      uint4 vv4 = make_uint4(0, 0, 0, 0);
      if (k < kmax)
        vv4 = *reinterpret_cast<const uint4 *>(Z + (size_t)k * stride + (size_t)(heads + kv + kvh) * D + dv0 + 8 * c);
      *reinterpret_cast<uint4 *>(sV + r * VPITCH + 16 * c) = vv4;
    }
    __syncthreads();

    // S = Q K^T for this warp's 16 rows x 64 keys
    float s[KT / 8][4];
#pragma unroll
    for (int j = 0; j < KT / 8; j++) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
#pragma unroll 4
    for (int kd = 0; kd < D / 16; kd++) {
      uint32_t a0, a1, a2, a3;
      {
        const int row = warp * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
        const int col = kd * 16 + (lane >> 4) * 8;
        ldsm_x4(sQa + row * PITCH + col * 2, a0, a1, a2, a3);
      }
#pragma unroll
      for (int j = 0; j < KT / 8; j += 2) {
        uint32_t b0, b1, b2, b3;
        const int key = j * 8 + (lane & 7) + (lane >> 4) * 8;
        const int col = kd * 16 + ((lane >> 3) & 1) * 8;
        ldsm_x4(sKa + key * PITCH + col * 2, b0, b1, b2, b3);
        mma16816(s[j], a0, a1, a2, a3, b0, b1);
        mma16816(s[j + 1], a0, a1, a2, a3, b2, b3);
      }
    }
    // mask, scale (log2 domain), online softmax
    float mx[2] = {-FLT_MAX, -FLT_MAX};
#pragma unroll
    for (int j = 0; j < KT / 8; j++) {
#pragma unroll
      for (int e = 0; e < 4; e++) {
        const int i = e >> 1;
        const int k = kc + j * 8 + 2 * tq + (e & 1);
        const int4 r = myr[i];
        const bool vis = (k >= r.x && k < r.y) || (k >= r.z && k < r.w);
        const float v = vis ? s[j][e] * scale_log2 : -FLT_MAX;
        s[j][e] = v;
        mx[i] = fmaxf(mx[i], v);
      }
    }
    float corr[2];
#pragma unroll
    for (int i = 0; i < 2; i++) {
      mx[i] = fmaxf(mx[i], __shfl_xor_sync(0xffffffffu, mx[i], 1));
      mx[i] = fmaxf(mx[i], __shfl_xor_sync(0xffffffffu, mx[i], 2));
      const float mn = fmaxf(m_i[i], mx[i]);
      corr[i] = (m_i[i] == -FLT_MAX) ? 0.f : ex2_approx(m_i[i] - mn);
      m_i[i] = mn;
    }
    float rs[2] = {0.f, 0.f};
    uint32_t p[KT / 8][2];
#pragma unroll
    for (int j = 0; j < KT / 8; j++) {
      float e4[4];
#pragma unroll
      for (int e = 0; e < 4; e++) {
        const int i = e >> 1;
        e4[e] = (s[j][e] == -FLT_MAX) ? 0.f : ex2_approx(s[j][e] - m_i[i]);
        rs[i] += e4[e];
      }
      p[j][0] = pack_h2(e4[0], e4[1]);
      p[j][1] = pack_h2(e4[2], e4[3]);
    }
#pragma unroll
    for (int i = 0; i < 2; i++) {
      rs[i] += __shfl_xor_sync(0xffffffffu, rs[i], 1);
      rs[i] += __shfl_xor_sync(0xffffffffu, rs[i], 2);
      l_i[i] = l_i[i] * corr[i] + rs[i];
    }
#pragma unroll
    for (int j = 0; j < NT; j++) {
      o[j][0] *= corr[0], o[j][1] *= corr[0];
      o[j][2] *= corr[1], o[j][3] *= corr[1];
    }
    // O += P V
#pragma unroll
    for (int kk = 0; kk < KT / 16; kk++) {
      const uint32_t a0 = p[2 * kk][0], a1 = p[2 * kk][1], a2 = p[2 * kk + 1][0], a3 = p[2 * kk + 1][1];
#pragma unroll
      for (int j = 0; j < NT; j += 2) {
        uint32_t b0, b1, b2, b3;
        const int key = kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
        const int col = j * 8 + (lane >> 4) * 8;
        ldsm_x4_t(sVa + key * VPITCH + col * 2, b0, b1, b2, b3);
        mma16816(o[j], a0, a1, a2, a3, b0, b1);
        mma16816(o[j + 1], a0, a1, a2, a3, b2, b3);
      }
    }
  }

  // normalise and store f16
#pragma unroll
  for (int i = 0; i < 2; i++) {
    const int t = t0 + warp * 16 + g + 8 * i;
    if (t >= T) continue;
    const float inv = l_i[i] > 0.f ? 1.0f / l_i[i] : 0.f;
    __half *y = Y + (size_t)t * heads * D + (size_t)h * D + dv0;
    // the output gate (d3-lite's gated attention): the row's gate heads follow its v heads
    const __half *gr = Z + (size_t)t * stride + (size_t)(heads + 2 * kv) * D + (size_t)h * D + dv0;
#pragma unroll
    for (int j = 0; j < NT; j++) {
      float a = o[j][2 * i] * inv, b = o[j][2 * i + 1] * inv;
      if (gate) {
        const float2 gv = __half22float2(*reinterpret_cast<const __half2 *>(gr + j * 8 + 2 * tq));
        a = a / (1.0f + expf(-gv.x)), b = b / (1.0f + expf(-gv.y));
      }
      *reinterpret_cast<__half2 *>(y + j * 8 + 2 * tq) = __floats2half2_rn(a, b);
    }
  }
}

}  // namespace

int attn_tc_launch(dc_ctx *ctx, const void *Z, const int *rng, void *Y, int T, int heads, int kv, int D, float scale,
                   long zstride, int gate);
int attn_sync_launch(dc_ctx *ctx, const void *Z, const int *rng, void *Y, int T, int heads, int kv, int D, float scale,
                     long zstride, int gate);

// form 0: the mma.sync kernel below (D = 64, 128, 256 or 512); form 1: the tcgen05 kernel (k_attn_tc.cu, D = 64,
// 128 or 256); form < 0: the tcgen05 kernel when D allows it. Z rows hold `zstride` halves: q | k | v heads, then
// with `gate` the q heads' output gates (Y = attention * sigmoid(gate), src/d3-kernels.ts:174-240), then padding.
int attn_launch_ex(dc_ctx *ctx, const void *Z, const int *rng, void *Y, int T, int heads, int kv, int D, float scale,
                   int form, long zstride, int gate) {
  if (form != 0 && (D == 64 || D == 128 || D == 256))
    return attn_tc_launch(ctx, Z, rng, Y, T, heads, kv, D, scale, zstride, gate);
  if (form == 1)
    return dc_fail(DC_EINVAL, "decision.js: tensor-core attention takes D = 64, 128 or 256 (got %d)", D);
  return attn_sync_launch(ctx, Z, rng, Y, T, heads, kv, D, scale, zstride, gate);
}

int attn_launch_form(dc_ctx *ctx, const void *Z, const int *rng, void *Y, int T, int heads, int kv, int D, float scale,
                     int form) {
  return attn_launch_ex(ctx, Z, rng, Y, T, heads, kv, D, scale, form, (long)(heads + 2 * kv) * D, 0);
}

int attn_launch(dc_ctx *ctx, const void *Z, const int *rng, void *Y, int T, int heads, int kv, int D, float scale) {
  return attn_launch_form(ctx, Z, rng, Y, T, heads, kv, D, scale, -1);
}

namespace {
template <int D, int DV>
int sync_launch(dc_ctx *ctx, const void *Z, const int *rng, void *Y, int T, int heads, int kv, float scale_log2,
                long zstride, int gate) {
  const int smem = (QT + KT) * (D * 2 + 16) + KT * (DV * 2 + 16);
  DC_CUDA(cudaFuncSetAttribute(attention_kernel<D, DV>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  dim3 grid((T + QT - 1) / QT, heads, D / DV);
  attention_kernel<D, DV><<<grid, 128, smem, ctx->stream>>>((const __half *)Z, (const int4 *)rng, (__half *)Y, T,
                                                            heads, kv, scale_log2, zstride, gate);
  return dc_launch_check("attention");
}
}  // namespace

int attn_sync_launch(dc_ctx *ctx, const void *Z, const int *rng, void *Y, int T, int heads, int kv, int D, float scale,
                     long zstride, int gate) {
  const float scale_log2 = scale * 1.4426950408889634f;
  if (D == 64) return sync_launch<64, 64>(ctx, Z, rng, Y, T, heads, kv, scale_log2, zstride, gate);
  if (D == 128) return sync_launch<128, 128>(ctx, Z, rng, Y, T, heads, kv, scale_log2, zstride, gate);
  if (D == 256) return sync_launch<256, 256>(ctx, Z, rng, Y, T, heads, kv, scale_log2, zstride, gate);
  if (D == 512) return sync_launch<512, 256>(ctx, Z, rng, Y, T, heads, kv, scale_log2, zstride, gate);
  return dc_fail(DC_EINVAL, "decision.js: attention head dim %d unsupported (64, 128, 256, 512)", D);
}
