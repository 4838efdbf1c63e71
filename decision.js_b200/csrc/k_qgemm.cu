// The quantized matmul Y[M,N] = X[M,K] . deq(W)[N,K]^T of decision.js (src/gpu.ts:202-226; semantics of
// MATMUL_PORTABLE_Q8/Q4, src/kernels.ts:445-520: f16 dequantisation rounded once, f32 accumulation, f16 out).
// Every form dequantises exactly f16((code - Z) * scale) on chip, accumulates in f32 in tensor memory
// (tcgen05.mma) and reads the tokens and codes with TMA into shared-memory rings guarded by mbarriers.
//
// Kernels (the dc_qmatmul_form numbers; qgemm_pick_form chooses among 3, 4, 5 and 6):
//  - qgemm_kernel<FORM 0>: prefill, one CTA per output tile, tokens on the MMA's M side (form 0);
//  - qgemm_kernel<FORM 1>: skinny, 128 weight rows on the M side, 16..128 tokens, split-K across CTAs (form 1);
//  - qgemm_persistent: prefill, one CTA per SM walking the tiles, double-buffered accumulators (form 2);
//  - qgemm_ts<BITS, BT, EPI, ASM>: persistent, weight rows on the M side. BT = 256 with the dequantised A in
//    shared memory is the prefill default (form 3) and carries the fused GeGLU/SwiGLU epilogues; BT = 16..64 and
//    192 keep A in tensor memory (TS MMA): form 4 (decode-to-mid M, with split-K) and form 6;
//  - qgemm_pair: the prefill tile on a CTA pair, tcgen05 cta_group::2, 256 weight rows x 256 tokens (form 7).
// The decode form (5, M <= 16) is k_gemv.cu.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <mutex>

#include "dc_internal.h"
#include "dc_ptx.cuh"

using namespace dcx;

namespace {

constexpr int BK = 64;          // K per stage (one 128-byte swizzle atom of f16)

// ------------------------------------------------------------------ forms 0 and 1 (qgemm_kernel)
// Per 64-wide K block: a TMA warp loads the token tile (f16, 128-byte swizzle) and the weight codes (u8) into a ring
// of shared-memory stages; four converter warps dequantise the codes to f16 straight into the swizzled K-major
// layout the MMA reads; one thread issues tcgen05.mma into an f32 TMEM accumulator; the converter warps then read
// TMEM back (tcgen05.ld) and store f16.
constexpr int NCONV = 128;      // converter / epilogue threads (warps 0-3)
constexpr int THREADS = 192;    // + warp 4 (TMA) + warp 5 (MMA, TMEM owner)

template <int BITS, int FORM, int BNT>
struct Cfg {
  static constexpr int ROWS_W = FORM == 0 ? BNT : 128;  // weight rows per tile
  static constexpr int ROWS_X = FORM == 0 ? 128 : BNT;  // token rows per tile
  static constexpr int MMA_N = FORM == 0 ? ROWS_W : ROWS_X;
  static constexpr int X_BYTES = ROWS_X * BK * 2;
  static constexpr int C_BYTES = ROWS_W * BK * BITS / 8;
  static constexpr int D_BYTES = ROWS_W * BK * 2;
  static constexpr int S = FORM == 0 ? (BITS == 8 && BNT == 256 ? 4 : 5) : (BNT >= 128 ? 5 : 8);  // X+codes
  static constexpr int SD = FORM == 0 ? 2 : 3;                                  // dequantised stages
  static constexpr int X_OFF = 0;
  static constexpr int D_OFF = X_OFF + S * X_BYTES;
  static constexpr int C_OFF = D_OFF + SD * D_BYTES;
  static constexpr int BAR_OFF = ((C_OFF + S * C_BYTES + 7) / 8) * 8;
  // full[S], empty[S], dfull[SD], dempty[SD], acc, then tmem address, abort flag, ticket
  static constexpr int NBARS = 2 * S + 2 * SD + 1;
  static constexpr int MISC_OFF = BAR_OFF + NBARS * 8;
  static constexpr int SMEM = MISC_OFF + 16 + 1024;  // + slack to align the base to 1024
  static constexpr int TCOLS = MMA_N < 32 ? 32 : MMA_N;
  static constexpr int ITEMS = ROWS_W * (BK / 16);  // 16-code items per stage
  static_assert(ITEMS % NCONV == 0, "items");
  static_assert(SMEM <= 227 * 1024, "shared memory");
};

struct GemmArgs {
  __half *Y;
  float *ws;            // split-K partials [splits, M, N] (FORM 1 only)
  uint32_t *counters;   // one per output tile (FORM 1 only)
  const __half *S;      // scales [N, K/32]
  uint32_t *err;
  int M, N, K, nkb, splits;
};

// Converts one 16-code item (row r, codes k0 .. k0+15 of the stage) into two swizzled 16-byte chunks.
template <int BITS>
__device__ __forceinline__ void convert_item(const uint8_t *cstage, uint8_t *dstage, int r, int c2, __half2 s2) {
  uint32_t w[4];
  if (BITS == 8) {
    uint4 v = *reinterpret_cast<const uint4 *>(cstage + r * 64 + c2 * 16);
    w[0] = v.x, w[1] = v.y, w[2] = v.z, w[3] = v.w;
  } else {
    uint2 v = *reinterpret_cast<const uint2 *>(cstage + r * 32 + c2 * 8);
    w[0] = v.x, w[1] = v.y;
  }
  __half2 h[8];
  if (BITS == 8) {
#pragma unroll
    for (int j = 0; j < 4; j++) deq_q8_word(w[j], s2, h[2 * j], h[2 * j + 1]);
  } else {
    __half2 a[4], b[4];
    deq_q4_word(w[0], s2, a);
    deq_q4_word(w[1], s2, b);
#pragma unroll
    for (int j = 0; j < 4; j++) h[j] = a[j], h[4 + j] = b[j];
  }
  const int x = r & 7;
  uint8_t *row = dstage + r * 128;
  *reinterpret_cast<uint4 *>(row + (((2 * c2) ^ x) << 4)) = *reinterpret_cast<uint4 *>(&h[0]);
  *reinterpret_cast<uint4 *>(row + (((2 * c2 + 1) ^ x) << 4)) = *reinterpret_cast<uint4 *>(&h[4]);
}

// Split K: the last CTA of an output tile adds weight row n's f32 partials for tokens [m0, m0 + mv) in split
// order (deterministic) and stores f16. Each round loads CH tokens of two splits (2 CH loads in flight), so a
// 64-token tile of two splits costs 64 / CH memory round trips instead of one per token and split.
template <int CH>
__device__ __forceinline__ void reduce_split_row(const float *ws, __half *Y, int M, int N, int n, int m0, int mv,
                                                 int splits) {
  for (int e0 = 0; e0 < mv; e0 += CH) {
    float acc[CH];
#pragma unroll
    for (int e = 0; e < CH; e++) acc[e] = 0.f;
    int q = 0;
    for (; q + 2 <= splits; q += 2) {
      const float *p0 = ws + ((size_t)q * M + m0 + e0) * N + n;
      const float *p1 = p0 + (size_t)M * N;
      float v0[CH], v1[CH];
#pragma unroll
      for (int e = 0; e < CH; e++) {
        const bool in = e0 + e < mv;
        v0[e] = in ? __ldcg(p0 + (size_t)e * N) : 0.f;
        v1[e] = in ? __ldcg(p1 + (size_t)e * N) : 0.f;
      }
#pragma unroll
      for (int e = 0; e < CH; e++) acc[e] = (acc[e] + v0[e]) + v1[e];
    }
    if (q < splits) {
      const float *p0 = ws + ((size_t)q * M + m0 + e0) * N + n;
      float v0[CH];
#pragma unroll
      for (int e = 0; e < CH; e++) v0[e] = e0 + e < mv ? __ldcg(p0 + (size_t)e * N) : 0.f;
#pragma unroll
      for (int e = 0; e < CH; e++) acc[e] += v0[e];
    }
#pragma unroll
    for (int e = 0; e < CH; e++)
      if (e0 + e < mv) Y[(size_t)(m0 + e0 + e) * N + n] = __float2half_rn(acc[e]);
  }
}

template <int BITS, int FORM, int BNT>
__global__ void __launch_bounds__(THREADS, 1)
    qgemm_kernel(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmW, GemmArgs a) {
  using C = Cfg<BITS, FORM, BNT>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bars = sbase + C::BAR_OFF;
  auto FULL = [&](int s) { return bars + 8u * s; };
  auto EMPTY = [&](int s) { return bars + 8u * (C::S + s); };
  auto DFULL = [&](int s) { return bars + 8u * (2 * C::S + s); };
  auto DEMPTY = [&](int s) { return bars + 8u * (2 * C::S + C::SD + s); };
  const uint32_t ACC = bars + 8u * (2 * C::S + 2 * C::SD);
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + C::MISC_OFF);
  volatile int *abort = reinterpret_cast<volatile int *>(smem + C::MISC_OFF + 4);
  volatile int *ticket = reinterpret_cast<volatile int *>(smem + C::MISC_OFF + 8);
  volatile int *verdict = reinterpret_cast<volatile int *>(smem + C::MISC_OFF + 12);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // tile coordinates: FORM 0 grid (n tiles, m tiles); FORM 1 grid (n tiles, splits, m tiles)
  const int n0 = blockIdx.x * C::ROWS_W;
  const int m0 = (FORM == 0 ? blockIdx.y : blockIdx.z) * C::ROWS_X;
  const int split = FORM == 0 ? 0 : blockIdx.y;
  const int kb_per = (a.nkb + a.splits - 1) / a.splits;
  const int kb0 = split * kb_per;
  const int kb1 = min(a.nkb, kb0 + kb_per);
  const int nk = max(0, kb1 - kb0);

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::S; s++) { mbar_init(FULL(s), 1); mbar_init(EMPTY(s), 1 + NCONV); }
    for (int s = 0; s < C::SD; s++) { mbar_init(DFULL(s), NCONV); mbar_init(DEMPTY(s), 1); }
    mbar_init(ACC, 1);
    *abort = 0;
    mbar_init_fence();
  }
  if (warp == 5) tmem_alloc(smem_u32(tmem_slot), C::TCOLS);
  if (warp == 4 && lane == 0) { tma_prefetch_desc(&tmX); tma_prefetch_desc(&tmW); }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 4) {
    // ---------------- TMA producer
    if (lane == 0) {
      for (int i = 0; i < nk; i++) {
        const int s = i % C::S;
        if (!mbar_wait(EMPTY(s), ((i / C::S) & 1) ^ 1, abort, a.err, DC_DEVERR_GEMM_WAIT)) break;
        mbar_expect_tx(FULL(s), C::X_BYTES + C::C_BYTES);
        const int kb = kb0 + i;
        tma_load_2d(sbase + C::X_OFF + s * C::X_BYTES, &tmX, kb * BK, m0, FULL(s));
        tma_load_2d(sbase + C::C_OFF + s * C::C_BYTES, &tmW, kb * BK * BITS / 8, n0, FULL(s));
      }
    }
  } else if (warp == 5) {
    // ---------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_f16_f32(128, C::MMA_N);
      for (int i = 0; i < nk; i++) {
        const int s = i % C::S, sd = i % C::SD;
        if (!mbar_wait(FULL(s), (i / C::S) & 1, abort, a.err, DC_DEVERR_GEMM_WAIT)) break;
        if (!mbar_wait(DFULL(sd), (i / C::SD) & 1, abort, a.err, DC_DEVERR_GEMM_WAIT)) break;
        tc_fence_after();
        const uint32_t xs = sbase + C::X_OFF + s * C::X_BYTES;
        const uint32_t ds = sbase + C::D_OFF + sd * C::D_BYTES;
        const uint64_t adesc = desc_sw128(FORM == 0 ? xs : ds);
        const uint64_t bdesc = desc_sw128(FORM == 0 ? ds : xs);
#pragma unroll
        for (int j = 0; j < BK / 16; j++)
          mma_f16(tmem, adesc + 2 * j, bdesc + 2 * j, idesc, (i > 0 || j > 0) ? 1u : 0u);
        mma_commit(EMPTY(s));
        mma_commit(DEMPTY(sd));
      }
      mma_commit(ACC);  // also after an abort, so the epilogue's wait ends with every MMA retired
    }
  } else {
    // ---------------- converters (warps 0-3), then the epilogue
    const int tid = threadIdx.x;
    const int kq = a.K / 32;
    for (int i = 0; i < nk; i++) {
      const int s = i % C::S, sd = i % C::SD;
      const int kb = kb0 + i;
      // scales of this thread's items: row n, 32-group (kb*64 + c2*16) / 32; rows past N and K past the
      // end read nothing (their codes are TMA zero fill and their products meet zero activations)
      __half2 sc[C::ITEMS / NCONV];
#pragma unroll
      for (int it = 0; it < C::ITEMS / NCONV; it++) {
        const int item = it * NCONV + tid, r = item >> 2, c2 = item & 3;
        const int n = n0 + r, g = kb * 2 + (c2 >> 1);
        __half v = __ushort_as_half(0);
        if (n < a.N && g < kq) v = __ldg(a.S + (size_t)n * kq + g);
        sc[it] = __halves2half2(v, v);
      }
      if (!mbar_wait(FULL(s), (i / C::S) & 1, abort, a.err, DC_DEVERR_GEMM_WAIT)) break;
      if (!mbar_wait(DEMPTY(sd), ((i / C::SD) & 1) ^ 1, abort, a.err, DC_DEVERR_GEMM_WAIT)) break;
      const uint8_t *cst = smem + C::C_OFF + s * C::C_BYTES;
      uint8_t *dst = smem + C::D_OFF + sd * C::D_BYTES;
#pragma unroll
      for (int it = 0; it < C::ITEMS / NCONV; it++) {
        const int item = it * NCONV + tid;
        convert_item<BITS>(cst, dst, item >> 2, item & 3, sc[it]);
      }
      fence_proxy_async_smem();
      mbar_arrive(DFULL(sd));
      mbar_arrive(EMPTY(s));
    }

    // ---------------- epilogue: TMEM lane = row of the MMA's M side
    const bool ok = mbar_wait(ACC, 0, abort, a.err, DC_DEVERR_GEMM_WAIT, 4000000000ull);
    if (!ok) *abort = 1;
    tc_fence_after();
    // one verdict for all 128 threads, so the named barriers below are reached by all or none
    asm volatile("bar.sync 1, 128;" ::: "memory");
    if (tid == 0) *verdict = *abort;
    asm volatile("bar.sync 1, 128;" ::: "memory");
    if (!*verdict) {
      const int row = warp * 32 + lane;
      const uint32_t trow = tmem + ((uint32_t)(warp * 32) << 16);
      if (FORM == 0) {
        const int m = m0 + row;
        const bool vec = (a.N % 8) == 0;
        for (int c = 0; c < C::MMA_N; c += 32) {
          uint32_t r[32];
          __syncwarp();  // tcgen05.ld is warp-collective: issue it converged
          tmem_ld32(trow + c, r);
          tmem_ld_wait(r);
          if (m < a.M) {
            __half *yr = a.Y + (size_t)m * a.N + n0 + c;
            const int nv = min(32, a.N - (n0 + c));
            if (nv == 32 && vec) {
#pragma unroll
              for (int q = 0; q < 4; q++) {
                __half2 h[4];
#pragma unroll
                for (int e = 0; e < 4; e++)
                  h[e] = __floats2half2_rn(__uint_as_float(r[8 * q + 2 * e]), __uint_as_float(r[8 * q + 2 * e + 1]));
                *reinterpret_cast<uint4 *>(yr + 8 * q) = *reinterpret_cast<uint4 *>(h);
              }
            } else {
#pragma unroll
              for (int e = 0; e < 32; e++)
                if (e < nv) yr[e] = __float2half_rn(__uint_as_float(r[e]));
            }
          }
        }
      } else {
        // skinny: the thread's row is weight row n; TMEM columns are tokens
        const int n = n0 + row;
        const bool partial = a.splits > 1;
        for (int c = 0; c < C::MMA_N; c += 16) {
          uint32_t r[16];
          __syncwarp();  // tcgen05.ld is warp-collective: issue it converged
          tmem_ld16(trow + c, r);
          tmem_ld_wait(r);
          if (n < a.N) {
#pragma unroll
            for (int e = 0; e < 16; e++) {
              const int m = m0 + c + e;
              if (m < a.M) {
                if (partial)
                  a.ws[((size_t)split * a.M + m) * a.N + n] = __uint_as_float(r[e]);
                else
                  a.Y[(size_t)m * a.N + n] = __float2half_rn(__uint_as_float(r[e]));
              }
            }
          }
        }
        if (partial) {
          // the last CTA of this output tile to finish adds the partials, in split order (deterministic)
          __threadfence();
          asm volatile("bar.sync 1, 128;" ::: "memory");
          const int tile = blockIdx.x + gridDim.x * blockIdx.z;
          if (tid == 0) *ticket = (int)atomicAdd(&a.counters[tile], 1u);
          asm volatile("bar.sync 1, 128;" ::: "memory");
          if (*ticket == a.splits - 1) {
            __threadfence();
            if (n < a.N) reduce_split_row<16>(a.ws, a.Y, a.M, a.N, n, m0, min(C::ROWS_X, a.M - m0), a.splits);
            if (tid == 0) a.counters[tile] = 0;
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TCOLS);
  }
}

// ------------------------------------------------------------------ persistent prefill form
// One CTA per SM walks output tiles (128 tokens x BN weight rows) in a static round-robin. Warps 0-3: epilogue
// (TMEM lanes 0-127); warps 4-11: converters; warp 12: TMA; warp 13: MMA and TMEM owner. Two TMEM accumulators
// (2 x BN columns) let the epilogue drain tile i while the MMA fills tile i+1; the stage rings run on one
// iteration counter across tiles. The epilogue stores f16 (EPI must be 0: the gated epilogues live in the TS form).

constexpr int P_CONV_WARPS = 8;
constexpr int P_NCONV = P_CONV_WARPS * 32;
constexpr int P_WARP_TMA = 4 + P_CONV_WARPS;
constexpr int P_WARP_MMA = P_WARP_TMA + 1;
constexpr int P_THREADS = (P_WARP_MMA + 1) * 32;

template <int BITS, int BN>
struct PCfg {
  static constexpr int X_BYTES = 128 * BK * 2;
  static constexpr int C_BYTES = BN * BK * BITS / 8;
  static constexpr int D_BYTES = BN * BK * 2;
  static constexpr int S = BN == 256 ? 4 : 6;
  static constexpr int SD = BN == 256 ? (BITS == 8 ? 2 : 3) : (BITS == 8 ? 3 : 4);
  static constexpr int X_OFF = 0;
  static constexpr int D_OFF = X_OFF + S * X_BYTES;
  static constexpr int C_OFF = D_OFF + SD * D_BYTES;
  static constexpr int BAR_OFF = ((C_OFF + S * C_BYTES + 7) / 8) * 8;
  static constexpr int NBARS = 2 * S + 2 * SD + 5;  // + accfull[2], accempty[2], done
  static constexpr int MISC_OFF = BAR_OFF + NBARS * 8;
  static constexpr int SMEM = MISC_OFF + 16 + 1024;
  static constexpr int TCOLS = 2 * BN;
  static constexpr int ITEMS = BN * (BK / 16);
  static_assert(ITEMS % P_NCONV == 0, "items");
  static_assert(SMEM <= 227 * 1024, "shared memory");
  static_assert(TCOLS <= 512, "tensor memory");
};

struct PArgs {
  __half *Y;
  const __half *S;
  uint32_t *err;
  int M, N, K, nkb, tn, tiles;
};

// The gating activations of the epilogue, in the reference's formulas (src/eg2-kernels.ts:9-13, src/kernels.ts:59)
// with the hardware exponential and divide intrinsics: their few-ulp f32 error vanishes in the f16 output.
// GELU, tanh approximation (src/eg2-kernels.ts:9-13): 0.5 x (1 + tanh u), u = 0.7978845608 (x + 0.044715 x^3),
// evaluated as x / (1 + e^(-2u)), the same function: one exponential and one reciprocal, no cancellation as tanh u
// nears -1, and the limits (0 and x) without the reference's clamp of u (an infinite e^(-2u) gives x / inf = 0).
// The epilogue spends a third less time on it than on the reference's (e - 1) / (e + 1) form.
__device__ __forceinline__ float gelu_tanh_f(float x) {
  const float u = 0.7978845608f * x * fmaf(0.044715f, x * x, 1.0f);
  return __fdividef(x, 1.0f + __expf(-2.0f * u));
}
__device__ __forceinline__ float silu_f(float x) { return __fdividef(x, 1.0f + __expf(-x)); }

template <int BITS, int BN, int EPI>
__global__ void __launch_bounds__(P_THREADS, 1)
    qgemm_persistent(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmW, PArgs a) {
  static_assert(EPI == 0, "the persistent SS form has no gated epilogue");
  using C = PCfg<BITS, BN>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bars = sbase + C::BAR_OFF;
  auto FULL = [&](int s) { return bars + 8u * s; };
  auto EMPTY = [&](int s) { return bars + 8u * (C::S + s); };
  auto DFULL = [&](int s) { return bars + 8u * (2 * C::S + s); };
  auto DEMPTY = [&](int s) { return bars + 8u * (2 * C::S + C::SD + s); };
  auto ACCF = [&](int b) { return bars + 8u * (2 * C::S + 2 * C::SD + b); };
  auto ACCE = [&](int b) { return bars + 8u * (2 * C::S + 2 * C::SD + 2 + b); };
  const uint32_t DONE = bars + 8u * (2 * C::S + 2 * C::SD + 4);
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + C::MISC_OFF);
  volatile int *abort = reinterpret_cast<volatile int *>(smem + C::MISC_OFF + 4);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    // converters and the epilogue arrive once per warp (after __syncwarp), not once per thread
    for (int s = 0; s < C::S; s++) { mbar_init(FULL(s), 1); mbar_init(EMPTY(s), 1 + P_CONV_WARPS); }
    for (int s = 0; s < C::SD; s++) { mbar_init(DFULL(s), P_CONV_WARPS); mbar_init(DEMPTY(s), 1); }
    for (int b = 0; b < 2; b++) { mbar_init(ACCF(b), 1); mbar_init(ACCE(b), 4); }
    mbar_init(DONE, 1);
    *abort = 0;
    mbar_init_fence();
  }
  if (warp == P_WARP_MMA) tmem_alloc(smem_u32(tmem_slot), C::TCOLS);
  if (warp == P_WARP_TMA && lane == 0) { tma_prefetch_desc(&tmX); tma_prefetch_desc(&tmW); }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == P_WARP_TMA) {
    if (lane == 0) {
      int it = 0;
      for (int tile = blockIdx.x; tile < a.tiles && !*abort; tile += gridDim.x) {
        const int n0 = (tile % a.tn) * BN, m0 = (tile / a.tn) * 128;
        for (int kb = 0; kb < a.nkb; kb++, it++) {
          const int s = it % C::S;
          if (!mbar_wait(EMPTY(s), ((it / C::S) & 1) ^ 1, abort, a.err, DC_DEVERR_GEMM_WAIT)) break;
          mbar_expect_tx(FULL(s), C::X_BYTES + C::C_BYTES);
          tma_load_2d(sbase + C::X_OFF + s * C::X_BYTES, &tmX, kb * BK, m0, FULL(s));
          tma_load_2d(sbase + C::C_OFF + s * C::C_BYTES, &tmW, kb * BK * BITS / 8, n0, FULL(s));
        }
      }
    }
  } else if (warp == P_WARP_MMA) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_f16_f32(128, BN);
      int it = 0, j = 0;
      for (int tile = blockIdx.x; tile < a.tiles && !*abort; tile += gridDim.x, j++) {
        const int b = j & 1;
        if (!mbar_wait(ACCE(b), ((j >> 1) & 1) ^ 1, abort, a.err, DC_DEVERR_GEMM_WAIT)) break;
        tc_fence_after();
        const uint32_t acc = tmem + (uint32_t)(b * BN);
        bool ok = true;
        for (int kb = 0; kb < a.nkb; kb++, it++) {
          const int s = it % C::S, sd = it % C::SD;
          if (!mbar_wait(FULL(s), (it / C::S) & 1, abort, a.err, DC_DEVERR_GEMM_WAIT) ||
              !mbar_wait(DFULL(sd), (it / C::SD) & 1, abort, a.err, DC_DEVERR_GEMM_WAIT)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t adesc = desc_sw128(sbase + C::X_OFF + s * C::X_BYTES);
          const uint64_t bdesc = desc_sw128(sbase + C::D_OFF + sd * C::D_BYTES);
#pragma unroll
          for (int k = 0; k < BK / 16; k++)
            mma_f16(acc, adesc + 2 * k, bdesc + 2 * k, idesc, (kb > 0 || k > 0) ? 1u : 0u);
          mma_commit(EMPTY(s));
          mma_commit(DEMPTY(sd));
        }
        if (!ok) break;
        mma_commit(ACCF(b));
      }
      mma_commit(DONE);  // retires every MMA issued, also after an abort
    }
  } else if (warp >= 4) {
    const int ctid = threadIdx.x - 128;
    const int kq = a.K / 32;
    constexpr int NQ = C::ITEMS / P_NCONV;
    // A thread always converts the same rows (ctid/4 + 64q) and the same 16-code column (ctid % 4) of a stage, so
    // its scales for iteration it are NQ values at group 2*kb + (ctid%4)/2; they are loaded two iterations ahead.
    const int nit = ((a.tiles - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x) * a.nkb;
    auto load_scales = [&](int it, __half2 (&sc)[NQ]) {
      const int tile = blockIdx.x + (it / a.nkb) * gridDim.x, kb = it % a.nkb;
      const int n0 = (tile % a.tn) * BN, g = kb * 2 + ((ctid & 3) >> 1);
#pragma unroll
      for (int q = 0; q < NQ; q++) {
        const int n = n0 + q * (P_NCONV / 4) + (ctid >> 2);
        __half v = __ushort_as_half(0);
        if (it < nit && n < a.N && g < kq) v = __ldg(a.S + (size_t)n * kq + g);
        sc[q] = __halves2half2(v, v);
      }
    };
    __half2 sc0[NQ], sc1[NQ], sc2[NQ];
    load_scales(0, sc0);
    load_scales(1, sc1);
    for (int it = 0; it < nit; it++) {
      load_scales(it + 2, sc2);
      const int s = it % C::S, sd = it % C::SD;
      if (!mbar_wait(FULL(s), (it / C::S) & 1, abort, a.err, DC_DEVERR_GEMM_WAIT) ||
          !mbar_wait(DEMPTY(sd), ((it / C::SD) & 1) ^ 1, abort, a.err, DC_DEVERR_GEMM_WAIT))
        break;
      const uint8_t *cst = smem + C::C_OFF + s * C::C_BYTES;
      uint8_t *dst = smem + C::D_OFF + sd * C::D_BYTES;
#pragma unroll
      for (int q = 0; q < NQ; q++) {
        const int item = q * P_NCONV + ctid;
        convert_item<BITS>(cst, dst, item >> 2, item & 3, sc0[q]);
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(DFULL(sd));
        mbar_arrive(EMPTY(s));
      }
#pragma unroll
      for (int q = 0; q < NQ; q++) sc0[q] = sc1[q], sc1[q] = sc2[q];
    }
  } else {
    // epilogue: warp w reads TMEM lanes 32w..32w+31, i.e. output rows m0 + 32w + lane
    const int row = warp * 32 + lane;
    const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
    int j = 0;
    for (int tile = blockIdx.x; tile < a.tiles && !*abort; tile += gridDim.x, j++) {
      const int b = j & 1;
      const int n0 = (tile % a.tn) * BN, m0 = (tile / a.tn) * 128;
      // tcgen05.ld is warp-collective: the warp decides together whether to go on
      if (!__all_sync(0xffffffffu, mbar_wait(ACCF(b), (j >> 1) & 1, abort, a.err, DC_DEVERR_GEMM_WAIT))) break;
      tc_fence_after();
      const uint32_t trow = tmem + lane_base + (uint32_t)(b * BN);
      const int m = m0 + row;
      {
        const bool vec = (a.N % 8) == 0;
        for (int c = 0; c < BN; c += 32) {
          uint32_t r[32];
          __syncwarp();  // tcgen05.ld is warp-collective: issue it converged
          tmem_ld32(trow + c, r);
          tmem_ld_wait(r);
          if (m < a.M) {
            __half *yr = a.Y + (size_t)m * a.N + n0 + c;
            const int nv = min(32, a.N - (n0 + c));
            if (nv == 32 && vec) {
#pragma unroll
              for (int q = 0; q < 4; q++) {
                __half2 h[4];
#pragma unroll
                for (int e = 0; e < 4; e++)
                  h[e] = __floats2half2_rn(__uint_as_float(r[8 * q + 2 * e]), __uint_as_float(r[8 * q + 2 * e + 1]));
                *reinterpret_cast<uint4 *>(yr + 8 * q) = *reinterpret_cast<uint4 *>(h);
              }
            } else {
#pragma unroll
              for (int e = 0; e < 32; e++)
                if (e < nv) yr[e] = __float2half_rn(__uint_as_float(r[e]));
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(ACCE(b));
    }
  }

  __syncthreads();
  if (warp == P_WARP_MMA) {
    mbar_wait(DONE, 0, abort, a.err, DC_DEVERR_GEMM_WAIT, 4000000000ull);
    tc_fence_after();
    tmem_dealloc(tmem, C::TCOLS);
  }
}

// ------------------------------------------------------------------ weight-side GEMM (prefill and skinny)
// The weights go on the MMA's M side (128 rows per tile) and the tokens on its N side (BT per tile). Per 64-wide K
// block the converter warps dequantize 128 weight rows exactly, either into shared memory in the 128-byte-swizzled
// K-major layout (ASM; the prefill default, BT = 256: both TMEM accumulators can then be 256 columns wide, and an
// N = 256 MMA does more per instruction than N = 192) or straight into tensor memory as the A operand (tcgen05.mma
// with A from TMEM; token tiles up to 192, and the small ones of the skinny form). The tokens (B operand) stream in
// by TMA with 128-byte swizzling, the codes by TMA with a 64- or 32-byte swizzle (conflict-free 16-byte row reads),
// each on its own ring: the token ring is freed by the MMA, the code ring by the converters, so the codes run ahead
// of the MMA. TMEM columns: two BT-wide f32 accumulators (then, without ASM, SA stages of 32 columns of
// dequantized A). The accumulator row is a weight row, so the epilogue writes each token's outputs as 64-byte runs
// across a warp.
// Work items are (output tile, K split): with few tokens (decode shapes) the K range is split over CTAs so the
// weight stream covers every SM; each CTA writes its f32 partial and the last CTA of a tile adds the partials in
// split order (deterministic) and stores f16.
// With K % 64 == 0 the code producer also stages each K block's scales beside its codes (cp.async on the same
// barrier), so no converter waits on a global load.
// Warps 0-3: epilogue; 4-11: converters (the two warps of a TMEM lane quadrant take alternate K blocks); 12: token
// TMA; 13: code TMA; 14: MMA and TMEM owner. EPI 1 / 2 gate over fused weights whose rows alternate gate, up
// (row 2i the gate of output i, row 2i + 1 its up): a lane pair of the epilogue holds both (no split).

constexpr int T_CONV_WARPS = 8;
constexpr int T_CW = T_CONV_WARPS / 4;  // converter warps per TMEM lane quadrant
constexpr int T_WARP_TMAX = 4 + T_CONV_WARPS;  // token tiles
constexpr int T_WARP_TMAC = T_WARP_TMAX + 1;   // weight codes
constexpr int T_WARP_MMA = T_WARP_TMAC + 1;
constexpr int T_THREADS = (T_WARP_MMA + 1) * 32;

// ASM: the dequantized weights (A) go to shared memory in the 128-byte-swizzled K-major layout instead of tensor
// memory, so both TMEM accumulators can be 256 tokens wide (an N = 256 MMA does more per instruction than
// N = 192: the prefill form); without it (token tiles up to 192) A stays in TMEM.
template <int BITS, int BT, int EPI, bool ASM = false>
struct TCfg {
  static constexpr int X_BYTES = BT * BK * 2;
  static constexpr int C_BYTES = 128 * BK * BITS / 8;
  static constexpr int A_BYTES = ASM ? 128 * BK * 2 : 0;
  // code stages (freed by the converters): deeper when few tokens leave the weight stream as the whole job
  static constexpr int SC = BT <= 64 ? 12 : (BITS == 8 ? 4 : 6);
  static constexpr int SA = ASM ? 3 : 4;
  // token stages (freed by the MMA): as many as fit, at most 8
  static constexpr int SCL_BYTES = 128 * 4;  // the two scales of each row of a code stage
  static constexpr int SX_FIT = (224 * 1024 - SC * (C_BYTES + SCL_BYTES) - SA * A_BYTES) / X_BYTES;
  static constexpr int SX = SX_FIT > 8 ? 8 : SX_FIT;
  static constexpr int X_OFF = 0;
  static constexpr int A_OFF = ((X_OFF + SX * X_BYTES + 1023) / 1024) * 1024;
  static constexpr int C_OFF = A_OFF + SA * A_BYTES;
  static constexpr int SCL_OFF = C_OFF + SC * C_BYTES;
  static constexpr int BAR_OFF = ((SCL_OFF + SC * SCL_BYTES + 7) / 8) * 8;
  // fullx, emptyx, fullc, emptyc, afull, aempty, accfull[2], accempty[2], done, ebar
  static constexpr int NBARS = 2 * SX + 2 * SC + 2 * SA + 4 + 2;
  static constexpr int MISC_OFF = BAR_OFF + NBARS * 8;
  static constexpr int SMEM = MISC_OFF + 16 + 1024;
  static constexpr int TCOLS = 512;
  static constexpr int A_COL = 2 * BT;
  static_assert(2 * BT + (ASM ? 0 : SA * 32) <= TCOLS, "tensor memory");
  static_assert(SMEM <= 227 * 1024, "shared memory");
  static_assert(C_BYTES % 1024 == 0, "stage alignment");
  static_assert(SX >= 2, "token stages");
  static_assert(BT % 16 == 0 && BT >= 16 && BT <= (ASM ? 256 : 192), "token tile");
};

struct TArgs {
  __half *Y;
  const __half *S;
  uint32_t *err;
  float *ws;           // split partials [splits, M, N] (splits > 1)
  uint32_t *counters;  // one per output tile, zero between launches (splits > 1)
  int M, N, K, nkb, tnt, tiles, splits, kb_per;
  int sc_smem;  // 1: the code producer stages each K block's scales next to its codes (K % 64 == 0)
  int w_early;  // 1: static weights; the warps that only read weights start before the previous kernel completes
};

// Work item w of a CTA: output tile (token tiles fastest) and K split, with its K-block range.
struct TItem {
  int tile, n0, m0, kb0, kb1;
};
__device__ __forceinline__ TItem titem(const TArgs &a, int w, int BT) {
  TItem t;
  t.tile = w / a.splits;
  const int split = w % a.splits;
  t.n0 = (t.tile / a.tnt) * 128;
  t.m0 = (t.tile % a.tnt) * BT;
  t.kb0 = split * a.kb_per;
  t.kb1 = min(a.nkb, t.kb0 + a.kb_per);
  return t;
}

template <int BITS, int BT, int EPI, bool ASM>
__global__ void __launch_bounds__(T_THREADS, 1)
    qgemm_ts(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmW, TArgs a) {
  dc_pdl_launch_dependents();
  using C = TCfg<BITS, BT, EPI, ASM>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bars = sbase + C::BAR_OFF;
  auto FULLX = [&](int s) { return bars + 8u * s; };
  auto EMPTYX = [&](int s) { return bars + 8u * (C::SX + s); };
  auto FULLC = [&](int s) { return bars + 8u * (2 * C::SX + s); };
  auto EMPTYC = [&](int s) { return bars + 8u * (2 * C::SX + C::SC + s); };
  auto AFULL = [&](int s) { return bars + 8u * (2 * C::SX + 2 * C::SC + s); };
  auto AEMPTY = [&](int s) { return bars + 8u * (2 * C::SX + 2 * C::SC + C::SA + s); };
  const uint32_t ACC0 = bars + 8u * (2 * C::SX + 2 * C::SC + 2 * C::SA);
  auto ACCF = [&](int b) { return ACC0 + 8u * b; };
  auto ACCE = [&](int b) { return ACC0 + 8u * (2 + b); };
  const uint32_t DONE = ACC0 + 32u;
  const uint32_t EBAR = DONE + 8u;  // split epilogue: the four warps meet twice per item
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + C::MISC_OFF);
  volatile int *abort = reinterpret_cast<volatile int *>(smem + C::MISC_OFF + 4);
  volatile int *ticket = reinterpret_cast<volatile int *>(smem + C::MISC_OFF + 8);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int items = a.tiles * a.splits;
  if (threadIdx.x == 0) {
    for (int s = 0; s < C::SX; s++) { mbar_init(FULLX(s), 1); mbar_init(EMPTYX(s), 1); }
    // a code stage is full when its TMA bytes landed and, with staged scales, the 32 producer lanes' copies
    for (int s = 0; s < C::SC; s++) { mbar_init(FULLC(s), a.sc_smem ? 33 : 1); mbar_init(EMPTYC(s), 4); }
    for (int s = 0; s < C::SA; s++) { mbar_init(AFULL(s), 4); mbar_init(AEMPTY(s), 1); }
    for (int b = 0; b < 2; b++) { mbar_init(ACCF(b), 1); mbar_init(ACCE(b), 4); }
    mbar_init(DONE, 1);
    mbar_init(EBAR, 4);
    *abort = 0;
    mbar_init_fence();
  }
  if (warp == T_WARP_MMA) tmem_alloc(smem_u32(tmem_slot), C::TCOLS);
  if (warp == T_WARP_TMAX && lane == 0) { tma_prefetch_desc(&tmX); tma_prefetch_desc(&tmW); }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // programmatic dependent launch: the setup above overlapped the previous kernel's drain; the token producer and
  // the epilogue (activations, outputs, split partials) wait for it to complete, and so do the weight-only warps
  // (codes, scales, dequantization, MMA) unless the weights are static
  if (warp < 4 || warp == T_WARP_TMAX || !a.w_early) dc_pdl_wait();

  if (warp == T_WARP_TMAX) {
    // token producer: the ring refills as the MMA frees it
    if (lane == 0) {
      int it = 0;
      bool ok = true;
      for (int w = blockIdx.x; ok && w < items && !*abort; w += gridDim.x) {
        const TItem t = titem(a, w, BT);
        for (int kb = t.kb0; kb < t.kb1; kb++, it++) {
          const int s = it % C::SX;
          if (!mbar_wait(EMPTYX(s), ((it / C::SX) & 1) ^ 1, abort, a.err, DC_DEVERR_GEMM_WAIT)) { ok = false; break; }
          mbar_expect_tx(FULLX(s), C::X_BYTES);
          tma_load_2d(sbase + C::X_OFF + s * C::X_BYTES, &tmX, kb * BK, t.m0, FULLX(s));
        }
      }
    }
  } else if (warp == T_WARP_TMAC) {
    // code producer (whole warp): the ring refills as the converters free it. Lane 0 issues the codes' TMA; with
    // staged scales every lane also copies the two scales of 4 rows (cp.async, tracked by the same barrier), so
    // the converters never wait on a global load.
    const int kq = a.K / 32;
    int it = 0;
    bool ok = true;
    for (int w = blockIdx.x; ok && w < items; w += gridDim.x) {
      const TItem t = titem(a, w, BT);
      for (int kb = t.kb0; kb < t.kb1; kb++, it++) {
        const int s = it % C::SC;
        const bool got = mbar_wait(EMPTYC(s), ((it / C::SC) & 1) ^ 1, abort, a.err, DC_DEVERR_GEMM_WAIT);
        if (!__all_sync(0xffffffffu, got)) { ok = false; break; }
        if (lane == 0) {
          mbar_expect_tx(FULLC(s), C::C_BYTES);
          tma_load_2d(sbase + C::C_OFF + s * C::C_BYTES, &tmW, kb * BK * BITS / 8, t.n0, FULLC(s));
        }
        if (a.sc_smem) {
#pragma unroll
          for (int q = 0; q < 4; q++) {
            const int row = q * 32 + lane, n = t.n0 + row;
            const bool in = n < a.N;
            cp_async_4(sbase + C::SCL_OFF + s * C::SCL_BYTES + row * 4, a.S + (size_t)(in ? n : 0) * kq + 2 * kb,
                       in ? 4u : 0u);
          }
          cp_async_mbar_arrive(FULLC(s));
        }
      }
    }
    asm volatile("cp.async.wait_all;" ::: "memory");  // none of this warp's copies outlives the CTA
  } else if (warp == T_WARP_MMA) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_f16_f32(128, BT);
      int it = 0, j = 0;
      bool ok = true;
      for (int w = blockIdx.x; ok && w < items && !*abort; w += gridDim.x, j++) {
        const TItem t = titem(a, w, BT);
        const int b = j & 1;
        if (!mbar_wait(ACCE(b), ((j >> 1) & 1) ^ 1, abort, a.err, DC_DEVERR_GEMM_WAIT)) break;
        tc_fence_after();
        const uint32_t acc = tmem + (uint32_t)(b * BT);
        for (int kb = t.kb0; kb < t.kb1; kb++, it++) {
          const int s = it % C::SX, sa = it % C::SA;
          if (!mbar_wait(FULLX(s), (it / C::SX) & 1, abort, a.err, DC_DEVERR_GEMM_WAIT) ||
              !mbar_wait(AFULL(sa), (it / C::SA) & 1, abort, a.err, DC_DEVERR_GEMM_WAIT)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t bdesc = desc_sw128(sbase + C::X_OFF + s * C::X_BYTES);
          const uint32_t acol = tmem + (uint32_t)(C::A_COL + sa * 32);
#pragma unroll
          for (int k = 0; k < BK / 16; k++) {
            if (ASM)
              mma_f16(acc, desc_sw128(sbase + C::A_OFF + sa * C::A_BYTES) + 2 * k, bdesc + 2 * k, idesc,
                      (kb > t.kb0 || k > 0) ? 1u : 0u);
            else
              mma_f16_ts(acc, acol + 8 * k, bdesc + 2 * k, idesc, (kb > t.kb0 || k > 0) ? 1u : 0u);
          }
          mma_commit(EMPTYX(s));
          mma_commit(AEMPTY(sa));
        }
        if (!ok) break;
        mma_commit(ACCF(b));
      }
      mma_commit(DONE);  // retires every MMA issued, also after an abort
    }
  } else if (warp >= 4) {
    // converters: weight row r (TMEM lane); the two warps of a lane quadrant take alternate K blocks, each a whole
    // row of 64 codes (two scales), so one warp's dequantize-store-signal chain overlaps the other's
    const int quad = warp & 3, par = (warp - 4) >> 2;  // par: this warp's turn among the quadrant's T_CW
    const int r = quad * 32 + lane;
    const int kq = a.K / 32;
    const uint32_t trow = tmem + ((uint32_t)(quad * 32) << 16) + (uint32_t)C::A_COL;
    int it = 0;
    bool ok = true;
    for (int w = blockIdx.x; ok && w < items && !*abort; w += gridDim.x) {
      const TItem t = titem(a, w, BT);
      const int n = t.n0 + r;
      for (int kb = t.kb0; kb < t.kb1; kb++, it++) {
        if (it % T_CW != par) continue;
        __half v0 = __ushort_as_half(0), v1 = __ushort_as_half(0);
        if (!a.sc_smem && n < a.N) {
          if (2 * kb < kq) v0 = __ldg(a.S + (size_t)n * kq + 2 * kb);
          if (2 * kb + 1 < kq) v1 = __ldg(a.S + (size_t)n * kq + 2 * kb + 1);
        }
        const int s = it % C::SC, sa = it % C::SA;
        // tcgen05.st is warp-collective: the warp decides together whether to go on
        const bool got = mbar_wait(FULLC(s), (it / C::SC) & 1, abort, a.err, DC_DEVERR_GEMM_WAIT) &&
                         mbar_wait(AEMPTY(sa), ((it / C::SA) & 1) ^ 1, abort, a.err, DC_DEVERR_GEMM_WAIT);
        if (!__all_sync(0xffffffffu, got)) { ok = false; break; }
        tc_fence_after();
        if (a.sc_smem) {
          const uint32_t sv = *reinterpret_cast<const uint32_t *>(smem + C::SCL_OFF + s * C::SCL_BYTES + r * 4);
          v0 = __ushort_as_half((unsigned short)(sv & 0xFFFF));
          v1 = __ushort_as_half((unsigned short)(sv >> 16));
        }
        const __half2 a0 = __halves2half2(v0, v0), a1 = __halves2half2(v1, v1);
        const uint8_t *cst = smem + C::C_OFF + s * C::C_BYTES;
        uint32_t hv[32];
        if (BITS == 8) {
          // row r holds 64 codes in four 16-byte chunks, chunk c stored at c ^ ((r / 2) % 4) (64-byte swizzle)
          const int x = (r >> 1) & 3;
#pragma unroll
          for (int c = 0; c < 4; c++) {
            const uint4 v = *reinterpret_cast<const uint4 *>(cst + r * 64 + ((c ^ x) << 4));
            const uint32_t wd[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int q = 0; q < 4; q++) {
              __half2 lo, hi;
              deq_q8_word(wd[q], c < 2 ? a0 : a1, lo, hi);
              hv[8 * c + 2 * q] = *reinterpret_cast<uint32_t *>(&lo);
              hv[8 * c + 2 * q + 1] = *reinterpret_cast<uint32_t *>(&hi);
            }
          }
        } else {
          // row r holds 64 codes in two 16-byte chunks, chunk c stored at c ^ ((r / 4) % 2) (32-byte swizzle)
          const int x = (r >> 2) & 1;
#pragma unroll
          for (int c = 0; c < 2; c++) {
            const uint4 v = *reinterpret_cast<const uint4 *>(cst + r * 32 + ((c ^ x) << 4));
            const uint32_t wd[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int q = 0; q < 4; q++) {
              __half2 o[4];
              deq_q4_word(wd[q], c == 0 ? a0 : a1, o);
#pragma unroll
              for (int e = 0; e < 4; e++) hv[16 * c + 4 * q + e] = *reinterpret_cast<uint32_t *>(&o[e]);
            }
          }
        }
        // the codes are in registers: free the stage before the TMEM stores
        __syncwarp();
        if (lane == 0) mbar_arrive(EMPTYC(s));
        if (ASM) {
          // row r of the A stage: 16-byte chunk j at j ^ (r % 8) (the 128-byte swizzle the MMA descriptor reads)
          uint8_t *arow = smem + C::A_OFF + sa * C::A_BYTES + r * 128;
#pragma unroll
          for (int j = 0; j < 8; j++)
            *reinterpret_cast<uint4 *>(arow + ((j ^ (r & 7)) << 4)) = *reinterpret_cast<const uint4 *>(&hv[4 * j]);
          fence_proxy_async_smem();  // visible to the tensor core's (async proxy) reads
        } else {
          __syncwarp();
          tmem_st16(trow + (uint32_t)(sa * 32), *reinterpret_cast<uint32_t (*)[16]>(&hv[0]));
          tmem_st16(trow + (uint32_t)(sa * 32 + 16), *reinterpret_cast<uint32_t (*)[16]>(&hv[16]));
          tmem_st_wait();
          tc_fence_before();
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(AFULL(sa));
      }
    }
  } else {
    // epilogue: thread = weight row n0 + 32 * warp + lane; TMEM columns = tokens
    const int row = warp * 32 + lane;
    const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
    int j = 0, ek = 0;
    for (int w = blockIdx.x; w < items && !*abort; w += gridDim.x, j++) {
      const TItem t = titem(a, w, BT);
      const int b = j & 1;
      // tcgen05.ld is warp-collective: the warp decides together whether to go on
      if (!__all_sync(0xffffffffu, mbar_wait(ACCF(b), (j >> 1) & 1, abort, a.err, DC_DEVERR_GEMM_WAIT))) break;
      tc_fence_after();
      const uint32_t trow = tmem + lane_base + (uint32_t)(b * BT);
      const int n = t.n0 + row;
      bool ok = true;
      for (int c = 0; c < BT && ok; c += 16) {
        uint32_t v[16];
        __syncwarp();  // tcgen05.ld is warp-collective: issue it converged
        tmem_ld16(trow + c, v);
        tmem_ld_wait(v);
        if (EPI == 0) {
          const int mv = min(16, a.M - (t.m0 + c));  // tokens of this chunk inside M
          if (n < a.N && mv > 0) {
            if (BT > 128 || a.splits == 1) {
              __half *p = a.Y + (size_t)(t.m0 + c) * a.N + n;
#pragma unroll
              for (int e = 0; e < 16; e++) {
                if (e < mv) *p = __float2half_rn(__uint_as_float(v[e]));
                p += a.N;
              }
            } else {
              float *p = a.ws + ((size_t)(w % a.splits) * a.M + t.m0 + c) * a.N + n;
#pragma unroll
              for (int e = 0; e < 16; e++) {
                if (e < mv) *p = __uint_as_float(v[e]);
                p += a.N;
              }
            }
          }
        } else {
          // gated: weight rows 2i and 2i + 1 of the tile are the gate and up rows of output n0/2 + i, so a lane
          // pair holds both halves of 64 outputs for these 16 tokens. Both are rounded to f16 (the matmul's output
          // type), one shuffle per token pair trades the missing halves, then the even lane gates the even tokens
          // and the odd lane the odd ones; per store the warp writes 16 consecutive outputs of two tokens.
          const int I = a.N / 2, o = t.n0 / 2 + warp * 16 + (lane >> 1);
          const bool odd = lane & 1;
#pragma unroll
          for (int q = 0; q < 8; q++) {
            const __half mine0 = __float2half_rn(__uint_as_float(v[2 * q]));
            const __half mine1 = __float2half_rn(__uint_as_float(v[2 * q + 1]));
            // even lane (gate row) sends the gate of token 2q+1, odd lane (up row) the up of token 2q
            const unsigned short send = __half_as_ushort(odd ? mine0 : mine1);
            const unsigned short recv = (unsigned short)__shfl_xor_sync(0xffffffffu, (unsigned)send, 1);
            const float gt = __half2float(odd ? __ushort_as_half(recv) : mine0);
            const float up = __half2float(odd ? mine1 : __ushort_as_half(recv));
            const float h = (EPI == 1 ? gelu_tanh_f(gt) : silu_f(gt)) * up;
            const int m = t.m0 + c + 2 * q + (odd ? 1 : 0);
            if (m < a.M) a.Y[(size_t)m * I + o] = __float2half_rn(h);
          }
        }
      }
      if (!ok) break;
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(ACCE(b));
      if (EPI == 0 && BT <= 128 && a.splits > 1) {
        // the last CTA of this output tile to finish adds the partials, in split order (deterministic)
        __threadfence();
        __syncwarp();
        if (lane == 0) mbar_arrive(EBAR);
        if (!__all_sync(0xffffffffu, mbar_wait(EBAR, ek & 1, abort, a.err, DC_DEVERR_GEMM_WAIT))) break;
        ek++;
        if (threadIdx.x == 0) *ticket = (int)atomicAdd(&a.counters[t.tile], 1u);
        __syncwarp();
        if (lane == 0) mbar_arrive(EBAR);
        if (!__all_sync(0xffffffffu, mbar_wait(EBAR, ek & 1, abort, a.err, DC_DEVERR_GEMM_WAIT))) break;
        ek++;
        if (*ticket == a.splits - 1) {
          __threadfence();
          if (n < a.N) reduce_split_row<8>(a.ws, a.Y, a.M, a.N, n, t.m0, min(BT, a.M - t.m0), a.splits);
          if (threadIdx.x == 0) a.counters[t.tile] = 0;
        }
      }
    }
  }

  __syncthreads();
  if (warp == T_WARP_MMA) {
    mbar_wait(DONE, 0, abort, a.err, DC_DEVERR_GEMM_WAIT, 4000000000ull);
    tc_fence_after();
    tmem_dealloc(tmem, C::TCOLS);
  }
}

// ------------------------------------------------------------------ host side

typedef CUresult (*EncodeTiled)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiled encode_fn() {
  static EncodeTiled fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiled>(p);
  });
  return fn;
}

int make_map(CUtensorMap *m, CUtensorMapDataType dt, const void *base, uint64_t inner, uint64_t rows,
             uint64_t row_bytes, uint32_t box_inner, uint32_t box_rows, CUtensorMapSwizzle sw) {
  EncodeTiled enc = encode_fn();
  DC_CHECK(enc, DC_ECUDA, "decision.js: cuTensorMapEncodeTiled is unavailable");
  cuuint64_t dims[2] = {inner, rows};
  cuuint64_t strides[1] = {row_bytes};
  cuuint32_t box[2] = {box_inner, box_rows};
  cuuint32_t es[2] = {1, 1};
  CUresult r = enc(m, dt, 2, const_cast<void *>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  DC_CHECK(r == CUDA_SUCCESS, DC_ECUDA, "decision.js: tensor map encode failed (%d)", (int)r);
  return DC_OK;
}

template <int BITS, int FORM, int BNT>
int launch_cfg(dc_ctx *ctx, const void *X, const void *Wq, const void *S, void *Y, int M, int N, int K, int splits) {
  using C = Cfg<BITS, FORM, BNT>;
  CUtensorMap tmX, tmW;
  int rc = make_map(&tmX, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, X, (uint64_t)K, (uint64_t)M, (uint64_t)K * 2, BK,
                    C::ROWS_X, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  const uint64_t wrow = (uint64_t)K * BITS / 8;
  rc = make_map(&tmW, CU_TENSOR_MAP_DATA_TYPE_UINT8, Wq, wrow, (uint64_t)N, wrow, BK * BITS / 8, C::ROWS_W,
                CU_TENSOR_MAP_SWIZZLE_NONE);
  if (rc) return rc;
  static uint64_t attr_done = 0;  // per device
  if (!(attr_done & (1ull << ctx->device))) {
    DC_CUDA(cudaFuncSetAttribute(qgemm_kernel<BITS, FORM, BNT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 C::SMEM));
    attr_done |= 1ull << ctx->device;
  }
  GemmArgs a;
  a.Y = static_cast<__half *>(Y);
  a.S = static_cast<const __half *>(S);
  a.err = ctx->d_err;
  a.M = M, a.N = N, a.K = K;
  a.nkb = (K + BK - 1) / BK;
  a.splits = FORM == 0 ? 1 : splits;
  a.ws = nullptr;
  a.counters = nullptr;
  const int tn = (N + C::ROWS_W - 1) / C::ROWS_W, tm = (M + C::ROWS_X - 1) / C::ROWS_X;
  dim3 grid = FORM == 0 ? dim3(tn, tm, 1) : dim3(tn, a.splits, tm);
  if (FORM == 1 && a.splits > 1) {
    void *ws;
    uint32_t *cnt;
    rc = dc_scratch(ctx, (size_t)a.splits * M * N * sizeof(float), (size_t)tn * tm, &ws, &cnt);
    if (rc) return rc;
    a.ws = static_cast<float *>(ws);
    a.counters = cnt;
  }
  qgemm_kernel<BITS, FORM, BNT><<<grid, THREADS, C::SMEM, ctx->stream>>>(tmX, tmW, a);
  return dc_launch_check("qgemm");
}

template <int BITS, int BN, int EPI>
int launch_persistent(dc_ctx *ctx, const void *X, const void *Wq, const void *S, void *Y, int M, int N, int K) {
  using C = PCfg<BITS, BN>;
  CUtensorMap tmX, tmW;
  int rc = make_map(&tmX, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, X, (uint64_t)K, (uint64_t)M, (uint64_t)K * 2, BK, 128,
                    CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  const uint64_t wrow = (uint64_t)K * BITS / 8;
  rc = make_map(&tmW, CU_TENSOR_MAP_DATA_TYPE_UINT8, Wq, wrow, (uint64_t)N, wrow, BK * BITS / 8, BN,
                CU_TENSOR_MAP_SWIZZLE_NONE);
  if (rc) return rc;
  static uint64_t attr_done = 0;  // per device
  if (!(attr_done & (1ull << ctx->device))) {
    DC_CUDA(cudaFuncSetAttribute(qgemm_persistent<BITS, BN, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 C::SMEM));
    attr_done |= 1ull << ctx->device;
  }
  PArgs a;
  a.Y = static_cast<__half *>(Y);
  a.S = static_cast<const __half *>(S);
  a.err = ctx->d_err;
  a.M = M, a.N = N, a.K = K;
  a.nkb = (K + BK - 1) / BK;
  a.tn = (N + BN - 1) / BN;
  a.tiles = a.tn * ((M + 127) / 128);
  const int sms = ctx->sms > 0 ? ctx->sms : 148;
  const int grid = a.tiles < sms ? a.tiles : sms;
  qgemm_persistent<BITS, BN, EPI><<<grid, P_THREADS, C::SMEM, ctx->stream>>>(tmX, tmW, a);
  return dc_launch_check("qgemm (persistent)");
}

template <int BITS, int BT, int EPI, bool ASM = false>
int launch_ts(dc_ctx *ctx, const void *X, const void *Wq, const void *S, void *Y, int M, int N, int K, int splits);

// ------------------------------------------------------------------ CTA-pair prefill form
// The prefill GEMM on a CTA pair (a cluster of 2, tcgen05 cta_group::2): one MMA of M = 256 weight rows x N = 256
// tokens per K step, issued by one thread of the even CTA. Each CTA dequantizes its 128 weight rows into its own
// shared memory (A half) and loads 128 of the 256 tokens (B half), so a CTA moves 24 KB (q8) per 64-wide K block
// from L2 for the same MMA work that costs a single CTA 40 KB (the token tile is the larger operand, and the pair
// loads it once between them). Each CTA's tensor memory holds its 128 rows x 256 tokens of the accumulator
// (two buffers). Barriers that the MMA waits on live in the even CTA: both CTAs' token TMAs complete on its
// full-barriers, both CTAs' converters and epilogue warps arrive on its A-full and accumulator-empty barriers;
// the MMA thread's commits release the stages and accumulators of both CTAs. Roles per CTA as in qgemm_ts:
// warps 0-3 epilogue, 4-11 converters, 12 token TMA, 13 code TMA (+ scales), 14 MMA (even CTA) / TMEM owner.

template <int BITS>
struct PairCfg {
  static constexpr int BT = 256;                   // tokens per pair tile (128 per CTA)
  static constexpr int X_BYTES = 128 * BK * 2;     // this CTA's token half per K block
  static constexpr int C_BYTES = 128 * 2 * BK * BITS / 8;  // a code stage holds two K blocks (one TMA row = 128 or 64 B)
  static constexpr int A_BYTES = 128 * BK * 2;
  static constexpr int SCL_BYTES = 128 * 8;                // the four scales of each row of a code stage
  static constexpr int SX = 5, SA = 4, SC = BITS == 8 ? 4 : 6;
  static constexpr int X_OFF = 0;
  static constexpr int A_OFF = X_OFF + SX * X_BYTES;
  static constexpr int C_OFF = A_OFF + SA * A_BYTES;
  static constexpr int SCL_OFF = C_OFF + SC * C_BYTES;
  static constexpr int BAR_OFF = ((SCL_OFF + SC * SCL_BYTES + 7) / 8) * 8;
  // fullx, emptyx, fullc, emptyc, afull, aempty, accfull[2], accempty[2], done
  static constexpr int NBARS = 2 * SX + 2 * SC + 2 * SA + 4 + 1;
  static constexpr int MISC_OFF = BAR_OFF + NBARS * 8;
  static constexpr int SMEM = MISC_OFF + 16 + 1024;
  static constexpr int TCOLS = 512;
  static_assert(SMEM <= 227 * 1024, "shared memory");
  static_assert(X_BYTES % 1024 == 0 && A_BYTES % 1024 == 0 && C_BYTES % 1024 == 0, "stage alignment");
};

template <int BITS, int EPI>
__global__ void __launch_bounds__(T_THREADS, 1)
    qgemm_pair(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmW, TArgs a) {
  dc_pdl_launch_dependents();
  using C = PairCfg<BITS>;
  constexpr int BT = C::BT;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bars = sbase + C::BAR_OFF;
  auto FULLX = [&](int s) { return bars + 8u * s; };
  auto EMPTYX = [&](int s) { return bars + 8u * (C::SX + s); };
  auto FULLC = [&](int s) { return bars + 8u * (2 * C::SX + s); };
  auto EMPTYC = [&](int s) { return bars + 8u * (2 * C::SX + C::SC + s); };
  auto AFULL = [&](int s) { return bars + 8u * (2 * C::SX + 2 * C::SC + s); };
  auto AEMPTY = [&](int s) { return bars + 8u * (2 * C::SX + 2 * C::SC + C::SA + s); };
  const uint32_t ACC0 = bars + 8u * (2 * C::SX + 2 * C::SC + 2 * C::SA);
  auto ACCF = [&](int b) { return ACC0 + 8u * b; };
  auto ACCE = [&](int b) { return ACC0 + 8u * (2 + b); };
  const uint32_t DONE = ACC0 + 32u;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + C::MISC_OFF);
  volatile int *abort = reinterpret_cast<volatile int *>(smem + C::MISC_OFF + 4);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool lead = rank == 0;
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  const int items = a.tiles;
  auto lead_bar = [&](uint32_t bar) { return mapa_shared(bar, 0); };
  auto peer_bar = [&](uint32_t bar) { return mapa_shared(bar, 1); };
  // pair tile w: 256 weight rows from n0 (this CTA's 128 from n0 + 128 rank), 256 tokens from m0 (this CTA loads
  // the 128 from m0 + 128 rank); token tiles fastest
  auto tile_n0 = [&](int w) { return (w / a.tnt) * 256; };
  auto tile_m0 = [&](int w) { return (w % a.tnt) * BT; };

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::SX; s++) { mbar_init(FULLX(s), 1); mbar_init(EMPTYX(s), 1); }
    // a code stage (two K blocks) is emptied by the converter warp of each quadrant for each of its two K blocks
    for (int s = 0; s < C::SC; s++) { mbar_init(FULLC(s), a.sc_smem ? 33 : 1); mbar_init(EMPTYC(s), 8); }
    for (int s = 0; s < C::SA; s++) { mbar_init(AFULL(s), 8); mbar_init(AEMPTY(s), 1); }
    for (int b = 0; b < 2; b++) { mbar_init(ACCF(b), 1); mbar_init(ACCE(b), 8); }
    mbar_init(DONE, 1);
    *abort = 0;
    mbar_init_fence();
  }
  if (warp == T_WARP_MMA) tmem_alloc_pair(smem_u32(tmem_slot), C::TCOLS);
  if (warp == T_WARP_TMAX && lane == 0) { tma_prefetch_desc(&tmX); tma_prefetch_desc(&tmW); }
  tc_fence_before();
  cluster_sync_all();  // both CTAs' barriers initialised and tensor memory allocated before any cross-CTA traffic
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // programmatic dependent launch, as in qgemm_ts: the setup above overlapped the previous kernel's drain; the token
  // producer and the epilogue wait for it to complete, the weight-only warps too unless the weights are static
  if (warp < 4 || warp == T_WARP_TMAX || !a.w_early) dc_pdl_wait();

  if (warp == T_WARP_TMAX) {
    // token producer: this CTA's half of each K block, counted on the even CTA's full-barrier
    if (lane == 0) {
      int it = 0;
      bool ok = true;
      for (int w = pair; ok && w < items && !*abort; w += npairs) {
        const int m0 = tile_m0(w) + 128 * (int)rank;
        for (int kb = 0; kb < a.nkb; kb++, it++) {
          const int s = it % C::SX;
          if (!mbar_wait(EMPTYX(s), ((it / C::SX) & 1) ^ 1, abort, a.err, DC_DEVERR_GEMM_WAIT)) {
            ok = false;
            break;
          }
          if (lead) mbar_expect_tx(FULLX(s), 2 * C::X_BYTES);
          tma_load_2d_pair(sbase + C::X_OFF + s * C::X_BYTES, &tmX, kb * BK, m0, lead_bar(FULLX(s)));
        }
      }
    }
  } else if (warp == T_WARP_TMAC) {
    // code producer (whole warp), local to this CTA: two K blocks of codes per TMA (128-byte rows for q8), the
    // four scales of each row by cp.async (K % 128 == 0, so each row's four scales are 8-byte aligned)
    const int kq = a.K / 32;
    int it2 = 0;
    bool ok = true;
    for (int w = pair; ok && w < items; w += npairs) {
      const int n0 = tile_n0(w) + 128 * (int)rank;
      for (int kb2 = 0; kb2 < a.nkb / 2; kb2++, it2++) {
        const int s = it2 % C::SC;
        const bool got = mbar_wait(EMPTYC(s), ((it2 / C::SC) & 1) ^ 1, abort, a.err, DC_DEVERR_GEMM_WAIT);
        if (!__all_sync(0xffffffffu, got)) { ok = false; break; }
        if (lane == 0) {
          mbar_expect_tx(FULLC(s), C::C_BYTES);
          tma_load_2d(sbase + C::C_OFF + s * C::C_BYTES, &tmW, kb2 * 2 * BK * BITS / 8, n0, FULLC(s));
        }
        if (a.sc_smem) {
#pragma unroll
          for (int q = 0; q < 4; q++) {
            const int row = q * 32 + lane, n = n0 + row;
            const bool in = n < a.N;
            cp_async_8(sbase + C::SCL_OFF + s * C::SCL_BYTES + row * 8, a.S + (size_t)(in ? n : 0) * kq + 4 * kb2,
                       in ? 8u : 0u);
          }
          cp_async_mbar_arrive(FULLC(s));
        }
      }
    }
    asm volatile("cp.async.wait_all;" ::: "memory");  // none of this warp's copies outlives the CTA
  } else if (warp == T_WARP_MMA) {
    if (lead && lane == 0) {
      constexpr uint32_t idesc = idesc_f16_f32(256, BT);
      int it = 0, j = 0;
      bool ok = true;
      for (int w = pair; ok && w < items && !*abort; w += npairs, j++) {
        const int b = j & 1;
        if (!mbar_wait(ACCE(b), ((j >> 1) & 1) ^ 1, abort, a.err, DC_DEVERR_GEMM_WAIT)) break;
        tc_fence_after();
        const uint32_t acc = tmem + (uint32_t)(b * BT);
        for (int kb = 0; kb < a.nkb; kb++, it++) {
          const int s = it % C::SX, sa = it % C::SA;
          if (!mbar_wait(FULLX(s), (it / C::SX) & 1, abort, a.err, DC_DEVERR_GEMM_WAIT) ||
              !mbar_wait(AFULL(sa), (it / C::SA) & 1, abort, a.err, DC_DEVERR_GEMM_WAIT)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t adesc = desc_sw128(sbase + C::A_OFF + sa * C::A_BYTES);
          const uint64_t bdesc = desc_sw128(sbase + C::X_OFF + s * C::X_BYTES);
#pragma unroll
          for (int k = 0; k < BK / 16; k++) mma_f16_pair(acc, adesc + 2 * k, bdesc + 2 * k, idesc, (kb > 0 || k > 0) ? 1u : 0u);
          mma_commit_pair(EMPTYX(s));
          mma_commit_pair(peer_bar(EMPTYX(s)));
          mma_commit_pair(AEMPTY(sa));
          mma_commit_pair(peer_bar(AEMPTY(sa)));
        }
        if (!ok) break;
        mma_commit_pair(ACCF(b));
        mma_commit_pair(peer_bar(ACCF(b)));
      }
      mma_commit_pair(DONE);  // retires every MMA issued, also after an abort
      mma_commit_pair(peer_bar(DONE));
    }
  } else if (warp >= 4) {
    // converters: weight row r (of this CTA's 128) into this CTA's A stage; the two warps of a quadrant take
    // alternate K blocks; the even CTA's A-full barrier counts all eight quadrant arrivals of the pair
    const int quad = warp & 3, par = (warp - 4) >> 2;
    const int r = quad * 32 + lane;
    const int kq = a.K / 32;
    int it = 0;
    bool ok = true;
    for (int w = pair; ok && w < items && !*abort; w += npairs) {
      const int n = tile_n0(w) + 128 * (int)rank + r;
      for (int kb = 0; kb < a.nkb; kb++, it++) {
        if (it % T_CW != par) continue;
        __half v0 = __ushort_as_half(0), v1 = __ushort_as_half(0);
        if (!a.sc_smem && n < a.N) {
          if (2 * kb < kq) v0 = __ldg(a.S + (size_t)n * kq + 2 * kb);
          if (2 * kb + 1 < kq) v1 = __ldg(a.S + (size_t)n * kq + 2 * kb + 1);
        }
        // code stage it / 2 holds this K block as its half h = it % 2 (K blocks per item even, so it and kb agree)
        const int h = it & 1, s = (it >> 1) % C::SC, sa = it % C::SA;
        const bool got = mbar_wait(FULLC(s), ((it >> 1) / C::SC) & 1, abort, a.err, DC_DEVERR_GEMM_WAIT) &&
                         mbar_wait(AEMPTY(sa), ((it / C::SA) & 1) ^ 1, abort, a.err, DC_DEVERR_GEMM_WAIT);
        if (!__all_sync(0xffffffffu, got)) { ok = false; break; }
        if (a.sc_smem) {
          const uint32_t sv = *reinterpret_cast<const uint32_t *>(smem + C::SCL_OFF + s * C::SCL_BYTES + r * 8 + 4 * h);
          v0 = __ushort_as_half((unsigned short)(sv & 0xFFFF));
          v1 = __ushort_as_half((unsigned short)(sv >> 16));
        }
        const __half2 a0 = __halves2half2(v0, v0), a1 = __halves2half2(v1, v1);
        const uint8_t *cst = smem + C::C_OFF + s * C::C_BYTES;
        uint32_t hv[32];
        if (BITS == 8) {
          // row r: 128 bytes (two K blocks), 16-byte chunk c at c ^ (r % 8) (128-byte swizzle); this K block is
          // chunks 4h .. 4h + 3
#pragma unroll
          for (int c = 0; c < 4; c++) {
            const uint4 v = *reinterpret_cast<const uint4 *>(cst + r * 128 + (((4 * h + c) ^ (r & 7)) << 4));
            const uint32_t wd[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int q = 0; q < 4; q++) {
              __half2 lo, hi;
              deq_q8_word(wd[q], c < 2 ? a0 : a1, lo, hi);
              hv[8 * c + 2 * q] = *reinterpret_cast<uint32_t *>(&lo);
              hv[8 * c + 2 * q + 1] = *reinterpret_cast<uint32_t *>(&hi);
            }
          }
        } else {
          // row r: 64 bytes (two K blocks), chunk c at c ^ ((r / 2) % 4) (64-byte swizzle); this K block is
          // chunks 2h, 2h + 1
          const int x = (r >> 1) & 3;
#pragma unroll
          for (int c = 0; c < 2; c++) {
            const uint4 v = *reinterpret_cast<const uint4 *>(cst + r * 64 + (((2 * h + c) ^ x) << 4));
            const uint32_t wd[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int q = 0; q < 4; q++) {
              __half2 o[4];
              deq_q4_word(wd[q], c == 0 ? a0 : a1, o);
#pragma unroll
              for (int e = 0; e < 4; e++) hv[16 * c + 4 * q + e] = *reinterpret_cast<uint32_t *>(&o[e]);
            }
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(EMPTYC(s));
        uint8_t *arow = smem + C::A_OFF + sa * C::A_BYTES + r * 128;
#pragma unroll
        for (int jj = 0; jj < 8; jj++)
          *reinterpret_cast<uint4 *>(arow + ((jj ^ (r & 7)) << 4)) = *reinterpret_cast<const uint4 *>(&hv[4 * jj]);
        fence_proxy_async_smem();  // this CTA's tensor core reads its own A half
        __syncwarp();
        if (lane == 0) {
          if (lead) mbar_arrive(AFULL(sa));
          else mbar_arrive_remote(lead_bar(AFULL(sa)));
        }
      }
    }
  } else {
    // epilogue: thread = weight row n0 + 128 rank + 32 warp + lane; TMEM columns = the pair tile's 256 tokens
    const int row = warp * 32 + lane;
    const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
    int j = 0;
    for (int w = pair; w < items && !*abort; w += npairs, j++) {
      const int b = j & 1;
      const int nb = tile_n0(w) + 128 * (int)rank, m0 = tile_m0(w);
      if (!__all_sync(0xffffffffu, mbar_wait(ACCF(b), (j >> 1) & 1, abort, a.err, DC_DEVERR_GEMM_WAIT))) break;
      tc_fence_after();
      const uint32_t trow = tmem + lane_base + (uint32_t)(b * BT);
      const int n = nb + row;
      for (int c = 0; c < BT; c += 16) {
        uint32_t v[16];
        __syncwarp();  // tcgen05.ld is warp-collective: issue it converged
        tmem_ld16(trow + c, v);
        tmem_ld_wait(v);
        if (EPI == 0) {
          const int mv = min(16, a.M - (m0 + c));
          if (n < a.N && mv > 0) {
            __half *p = a.Y + (size_t)(m0 + c) * a.N + n;
#pragma unroll
            for (int e = 0; e < 16; e++) {
              if (e < mv) *p = __float2half_rn(__uint_as_float(v[e]));
              p += a.N;
            }
          }
        } else {
          // gated, as in qgemm_ts: weight rows 2i and 2i + 1 of this CTA's 128 are the gate and up rows of output
          // nb/2 + i, so a lane pair holds both halves; f16 rounding of both, one shuffle per token pair, the even
          // lane gates the even tokens and the odd lane the odd ones
          const int I = a.N / 2, o = nb / 2 + warp * 16 + (lane >> 1);
          const bool odd = lane & 1;
#pragma unroll
          for (int q = 0; q < 8; q++) {
            const __half mine0 = __float2half_rn(__uint_as_float(v[2 * q]));
            const __half mine1 = __float2half_rn(__uint_as_float(v[2 * q + 1]));
            const unsigned short send = __half_as_ushort(odd ? mine0 : mine1);
            const unsigned short recv = (unsigned short)__shfl_xor_sync(0xffffffffu, (unsigned)send, 1);
            const float gt = __half2float(odd ? __ushort_as_half(recv) : mine0);
            const float up = __half2float(odd ? mine1 : __ushort_as_half(recv));
            const float h = (EPI == 1 ? gelu_tanh_f(gt) : silu_f(gt)) * up;
            const int m = m0 + c + 2 * q + (odd ? 1 : 0);
            if (m < a.M && o < I) a.Y[(size_t)m * I + o] = __float2half_rn(h);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (lead) mbar_arrive(ACCE(b));
        else mbar_arrive_remote_relaxed(lead_bar(ACCE(b)));
      }
    }
  }

  __syncthreads();
  if (warp == T_WARP_MMA) {
    mbar_wait(DONE, 0, abort, a.err, DC_DEVERR_GEMM_WAIT, 4000000000ull);
    tc_fence_after();
  }
  tc_fence_before();
  cluster_sync_all();  // no CTA leaves while its peer may still signal its barriers or read its memory
  tc_fence_after();
  if (warp == T_WARP_MMA) tmem_dealloc_pair(tmem, C::TCOLS);
}

template <int BITS, int EPI>
int launch_pair(dc_ctx *ctx, const void *X, const void *Wq, const void *S, void *Y, int M, int N, int K) {
  using C = PairCfg<BITS>;
  // code stages pair K blocks: K a multiple of 128 and 8-byte aligned scales (four per row per stage, one 8-byte
  // cp.async); otherwise the single-CTA form
  if (K % 128 != 0 || (reinterpret_cast<uintptr_t>(S) & 7) != 0) return launch_ts<BITS, 256, EPI, true>(ctx, X, Wq, S, Y, M, N, K, 1);
  CUtensorMap tmX, tmW;
  int rc = make_map(&tmX, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, X, (uint64_t)K, (uint64_t)M, (uint64_t)K * 2, BK, 128,
                    CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  const uint64_t wrow = (uint64_t)K * BITS / 8;
  rc = make_map(&tmW, CU_TENSOR_MAP_DATA_TYPE_UINT8, Wq, wrow, (uint64_t)N, wrow, 2 * BK * BITS / 8, 128,
                BITS == 8 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B);
  if (rc) return rc;
  static uint64_t attr_done = 0;  // per device
  if (!(attr_done & (1ull << ctx->device))) {
    DC_CUDA(cudaFuncSetAttribute(qgemm_pair<BITS, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM));
    attr_done |= 1ull << ctx->device;
  }
  TArgs a;
  a.Y = static_cast<__half *>(Y);
  a.S = static_cast<const __half *>(S);
  a.err = ctx->d_err;
  a.M = M, a.N = N, a.K = K;
  a.nkb = (K + BK - 1) / BK;
  a.tnt = (M + C::BT - 1) / C::BT;
  a.tiles = a.tnt * ((N + 255) / 256);
  a.splits = 1, a.kb_per = a.nkb;
  a.sc_smem = (K % 64 == 0 && (reinterpret_cast<uintptr_t>(S) & 3) == 0) ? 1 : 0;
  a.w_early = ctx->static_weights ? 1 : 0;
  a.ws = nullptr;
  a.counters = nullptr;
  const int sms = ctx->sms > 0 ? ctx->sms : 148;
  const int pairs = a.tiles < sms / 2 ? a.tiles : sms / 2;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(2 * pairs), 1, 1);
  cfg.blockDim = dim3(T_THREADS, 1, 1);
  cfg.dynamicSmemBytes = C::SMEM;
  cfg.stream = ctx->stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;  // see dc_pdl_begin
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  DC_CUDA(cudaLaunchKernelEx(&cfg, qgemm_pair<BITS, EPI>, tmX, tmW, a));
  return dc_launch_check("qgemm (pair)");
}

// ------------------------------------------------------------------ direct form (pre-dequantized f16 weights)
// matmulDirect (src/kernels.ts:549-676): the weights were dequantized once, at load (tileWeights,
// src/kernels.ts:528-543; dc_dequant), so a K block of the A operand is a plain f16 tile that TMA drops into shared
// memory in the layout the converters of qgemm_pair write: no converter warps, no code ring. The pair tile is the
// same (cluster of 2, tcgen05 cta_group::2, 256 weight rows x 256 tokens, each CTA 128 of each); one thread per CTA
// loads its two 16 KB halves of a K block into one stage of a 6-deep ring, both CTAs' bytes completing on the even
// CTA's full-barrier; the even CTA's MMA thread commits each stage free in both CTAs. Roles: warps 0-3 epilogue
// (plain or gated, as qgemm_pair's; gated also 6-9), 4 producer, 5 MMA (even CTA) / TMEM owner. The arithmetic is the quantized forms':
// f16((code - Z) * scale) operands (identical values), f32 accumulation, f16 out. With the pipeline this short, the
// epilogue would set the pace for the gated epilogues (a tile's 256 tokens took one warp per lane quadrant longer than
// the tile's MMAs), so there two warps share each quadrant, a half of the token columns each.
struct DirectCfg {
  static constexpr int BT = 256;
  static constexpr int X_BYTES = 128 * BK * 2;  // this CTA's token half of a K block
  static constexpr int W_BYTES = 128 * BK * 2;  // this CTA's 128 weight rows of a K block
  static constexpr int STAGE = X_BYTES + W_BYTES;
  static constexpr int SS = 6;
  static constexpr int BAR_OFF = SS * STAGE;
  static constexpr int NBARS = 2 * SS + 4 + 1;  // full, empty, accfull[2], accempty[2], done
  static constexpr int MISC_OFF = BAR_OFF + NBARS * 8;
  static constexpr int SMEM = MISC_OFF + 16 + 1024;
  static constexpr int TCOLS = 512;
  // warps 0-3 epilogue (and 6-9 for the gated epilogues), 4 producer, 5 MMA
  static constexpr int threads(int epi) { return epi == 0 ? 192 : 320; }
  static_assert(SMEM <= 227 * 1024, "shared memory");
  static_assert(X_BYTES % 1024 == 0 && W_BYTES % 1024 == 0, "stage alignment");
};

template <int EPI>
__global__ void __launch_bounds__(DirectCfg::threads(EPI), 1)
    qgemm_direct(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmW, TArgs a) {
  dc_pdl_launch_dependents();
  using C = DirectCfg;
  constexpr int BT = C::BT;
  constexpr int WARP_PROD = 4, WARP_MMA = 5;
  // epilogue warps per TMEM lane quadrant, token columns per warp, columns per tensor-memory load
  constexpr int HALVES = EPI == 0 ? 1 : 2, CW = BT / HALVES, CH = EPI == 0 ? 16 : 32;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bars = sbase + C::BAR_OFF;
  auto FULL = [&](int s) { return bars + 8u * s; };
  auto EMPTY = [&](int s) { return bars + 8u * (C::SS + s); };
  const uint32_t ACC0 = bars + 8u * (2 * C::SS);
  auto ACCF = [&](int b) { return ACC0 + 8u * b; };
  auto ACCE = [&](int b) { return ACC0 + 8u * (2 + b); };
  const uint32_t DONE = ACC0 + 32u;
  auto XST = [&](int s) { return sbase + (uint32_t)(s * C::STAGE); };
  auto WST = [&](int s) { return sbase + (uint32_t)(s * C::STAGE + C::X_BYTES); };
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + C::MISC_OFF);
  volatile int *abort = reinterpret_cast<volatile int *>(smem + C::MISC_OFF + 4);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool lead = rank == 0;
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  const int items = a.tiles;
  auto lead_bar = [&](uint32_t bar) { return mapa_shared(bar, 0); };
  auto peer_bar = [&](uint32_t bar) { return mapa_shared(bar, 1); };
  auto tile_n0 = [&](int w) { return (w / a.tnt) * 256; };  // token tiles fastest
  auto tile_m0 = [&](int w) { return (w % a.tnt) * BT; };

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::SS; s++) { mbar_init(FULL(s), 1); mbar_init(EMPTY(s), 1); }
    for (int b = 0; b < 2; b++) { mbar_init(ACCF(b), 1); mbar_init(ACCE(b), 8 * HALVES); }
    mbar_init(DONE, 1);
    *abort = 0;
    mbar_init_fence();
  }
  if (warp == WARP_MMA) tmem_alloc_pair(smem_u32(tmem_slot), C::TCOLS);
  if (warp == WARP_PROD && lane == 0) { tma_prefetch_desc(&tmX); tma_prefetch_desc(&tmW); }
  tc_fence_before();
  cluster_sync_all();  // both CTAs' barriers initialised and tensor memory allocated before any cross-CTA traffic
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // programmatic dependent launch: the setup above overlapped the previous kernel's drain; the producer (tokens)
  // and the epilogue (Y) wait for it to complete
  if (warp != WARP_MMA) dc_pdl_wait();

  if (warp == WARP_PROD) {
    if (lane == 0) {
      int it = 0;
      bool ok = true;
      for (int w = pair; ok && w < items && !*abort; w += npairs) {
        const int m0 = tile_m0(w) + 128 * (int)rank, n0 = tile_n0(w) + 128 * (int)rank;
        for (int kb = 0; kb < a.nkb; kb++, it++) {
          const int s = it % C::SS;
          if (!mbar_wait(EMPTY(s), ((it / C::SS) & 1) ^ 1, abort, a.err, DC_DEVERR_GEMM_WAIT)) {
            ok = false;
            break;
          }
          if (lead) mbar_expect_tx(FULL(s), 2 * C::STAGE);
          tma_load_2d_pair(XST(s), &tmX, kb * BK, m0, lead_bar(FULL(s)));
          tma_load_2d_pair(WST(s), &tmW, kb * BK, n0, lead_bar(FULL(s)));
        }
      }
    }
  } else if (warp == WARP_MMA) {
    if (lead && lane == 0) {
      constexpr uint32_t idesc = idesc_f16_f32(256, BT);
      int it = 0, j = 0;
      bool ok = true;
      for (int w = pair; ok && w < items && !*abort; w += npairs, j++) {
        const int b = j & 1;
        if (!mbar_wait(ACCE(b), ((j >> 1) & 1) ^ 1, abort, a.err, DC_DEVERR_GEMM_WAIT)) break;
        tc_fence_after();
        const uint32_t acc = tmem + (uint32_t)(b * BT);
        for (int kb = 0; kb < a.nkb; kb++, it++) {
          const int s = it % C::SS;
          if (!mbar_wait(FULL(s), (it / C::SS) & 1, abort, a.err, DC_DEVERR_GEMM_WAIT)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t adesc = desc_sw128(WST(s));
          const uint64_t bdesc = desc_sw128(XST(s));
#pragma unroll
          for (int k = 0; k < BK / 16; k++) mma_f16_pair(acc, adesc + 2 * k, bdesc + 2 * k, idesc, (kb > 0 || k > 0) ? 1u : 0u);
          mma_commit_pair(EMPTY(s));
          mma_commit_pair(peer_bar(EMPTY(s)));
        }
        if (!ok) break;
        mma_commit_pair(ACCF(b));
        mma_commit_pair(peer_bar(ACCF(b)));
      }
      mma_commit_pair(DONE);  // retires every MMA issued, also after an abort
      mma_commit_pair(peer_bar(DONE));
    }
  } else {
    // epilogue: warp w reads TMEM lanes 32 (w % 4) .. + 31 (thread = weight row n0 + 128 rank + 32 (w % 4) + lane);
    // plain: warps 0-3, all 256 token columns, 16 per tensor-memory load; gated: two warps per lane quadrant, one
    // half of the columns each (warps 0-3 the first, 6-9 the second), 32 per load
    const int quad = warp & 3, half = warp >= 6 ? 1 : 0;
    const int row = quad * 32 + lane;
    const uint32_t lane_base = (uint32_t)(quad * 32) << 16;
    int j = 0;
    for (int w = pair; w < items && !*abort; w += npairs, j++) {
      const int b = j & 1;
      const int nb = tile_n0(w) + 128 * (int)rank, m0 = tile_m0(w) + CW * half;
      if (!__all_sync(0xffffffffu, mbar_wait(ACCF(b), (j >> 1) & 1, abort, a.err, DC_DEVERR_GEMM_WAIT))) break;
      tc_fence_after();
      const uint32_t trow = tmem + lane_base + (uint32_t)(b * BT + CW * half);
      const int n = nb + row;
      for (int c = 0; c < CW; c += CH) {
        uint32_t v[CH];
        __syncwarp();  // tcgen05.ld is warp-collective: issue it converged
        if constexpr (CH == 16) tmem_ld16(trow + c, v);
        else tmem_ld32(trow + c, v);
        tmem_ld_wait(v);
        if (EPI == 0) {
          const int mv = min(CH, a.M - (m0 + c));
          if (n < a.N && mv > 0) {
            __half *p = a.Y + (size_t)(m0 + c) * a.N + n;
#pragma unroll
            for (int e = 0; e < CH; e++) {
              if (e < mv) *p = __float2half_rn(__uint_as_float(v[e]));
              p += a.N;
            }
          }
        } else {
          // gated: weight rows 2i and 2i + 1 are the gate and up rows of output i (a lane pair holds both); f16
          // rounding of both, one shuffle per token pair, the even lane gates the even tokens, the odd lane the odd
          const int I = a.N / 2, o = nb / 2 + quad * 16 + (lane >> 1);
          const bool odd = lane & 1;
#pragma unroll
          for (int q = 0; q < CH / 2; q++) {
            const __half mine0 = __float2half_rn(__uint_as_float(v[2 * q]));
            const __half mine1 = __float2half_rn(__uint_as_float(v[2 * q + 1]));
            const unsigned short send = __half_as_ushort(odd ? mine0 : mine1);
            const unsigned short recv = (unsigned short)__shfl_xor_sync(0xffffffffu, (unsigned)send, 1);
            const float gt = __half2float(odd ? __ushort_as_half(recv) : mine0);
            const float up = __half2float(odd ? mine1 : __ushort_as_half(recv));
            const float h = (EPI == 1 ? gelu_tanh_f(gt) : silu_f(gt)) * up;
            const int m = m0 + c + 2 * q + (odd ? 1 : 0);
            if (m < a.M && o < I) a.Y[(size_t)m * I + o] = __float2half_rn(h);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (lead) mbar_arrive(ACCE(b));
        else mbar_arrive_remote_relaxed(lead_bar(ACCE(b)));
      }
    }
  }

  __syncthreads();
  if (warp == WARP_MMA) {
    mbar_wait(DONE, 0, abort, a.err, DC_DEVERR_GEMM_WAIT, 4000000000ull);
    tc_fence_after();
  }
  tc_fence_before();
  cluster_sync_all();  // no CTA leaves while its peer may still signal its barriers or read its memory
  tc_fence_after();
  if (warp == WARP_MMA) tmem_dealloc_pair(tmem, C::TCOLS);
}

template <int EPI>
int launch_direct(dc_ctx *ctx, const void *X, const void *W16, void *Y, int M, int N, int K) {
  using C = DirectCfg;
  CUtensorMap tmX, tmW;
  int rc = make_map(&tmX, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, X, (uint64_t)K, (uint64_t)M, (uint64_t)K * 2, BK, 128,
                    CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  rc = make_map(&tmW, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, W16, (uint64_t)K, (uint64_t)N, (uint64_t)K * 2, BK, 128,
                CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  static uint64_t attr_done = 0;  // per device
  if (!(attr_done & (1ull << ctx->device))) {
    DC_CUDA(cudaFuncSetAttribute(qgemm_direct<EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM));
    attr_done |= 1ull << ctx->device;
  }
  TArgs a;
  a.Y = static_cast<__half *>(Y);
  a.S = nullptr;
  a.err = ctx->d_err;
  a.M = M, a.N = N, a.K = K;
  a.nkb = (K + BK - 1) / BK;
  a.tnt = (M + C::BT - 1) / C::BT;
  a.tiles = a.tnt * ((N + 255) / 256);
  a.splits = 1, a.kb_per = a.nkb;
  a.sc_smem = 0;
  a.w_early = 0;
  a.ws = nullptr;
  a.counters = nullptr;
  const int sms = ctx->sms > 0 ? ctx->sms : 148;
  const int pairs = a.tiles < sms / 2 ? a.tiles : sms / 2;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(2 * pairs), 1, 1);
  cfg.blockDim = dim3(C::threads(EPI), 1, 1);
  cfg.dynamicSmemBytes = C::SMEM;
  cfg.stream = ctx->stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;  // see dc_pdl_begin
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  DC_CUDA(cudaLaunchKernelEx(&cfg, qgemm_direct<EPI>, tmX, tmW, a));
  return dc_launch_check("qgemm (direct)");
}

template <int BITS, int BT, int EPI, bool ASM>
int launch_ts(dc_ctx *ctx, const void *X, const void *Wq, const void *S, void *Y, int M, int N, int K, int splits) {
  using C = TCfg<BITS, BT, EPI, ASM>;
  CUtensorMap tmX, tmW;
  int rc = make_map(&tmX, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, X, (uint64_t)K, (uint64_t)M, (uint64_t)K * 2, BK, BT,
                    CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  const uint64_t wrow = (uint64_t)K * BITS / 8;
  rc = make_map(&tmW, CU_TENSOR_MAP_DATA_TYPE_UINT8, Wq, wrow, (uint64_t)N, wrow, BK * BITS / 8, 128,
                BITS == 8 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_32B);
  if (rc) return rc;
  static uint64_t attr_done = 0;  // per device
  if (!(attr_done & (1ull << ctx->device))) {
    DC_CUDA(cudaFuncSetAttribute(qgemm_ts<BITS, BT, EPI, ASM>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM));
    attr_done |= 1ull << ctx->device;
  }
  TArgs a;
  a.Y = static_cast<__half *>(Y);
  a.S = static_cast<const __half *>(S);
  a.err = ctx->d_err;
  a.M = M, a.N = N, a.K = K;
  a.nkb = (K + BK - 1) / BK;
  a.tnt = (M + BT - 1) / BT;
  a.tiles = a.tnt * ((N + 127) / 128);
  const int sms = ctx->sms > 0 ? ctx->sms : 148;
  if (EPI != 0 || BT > 128) splits = 1;  // the prefill tiles do not split K
  if (splits <= 0) {
    // split K only while the tiles leave most SMs idle, each split at least 24 K blocks long: the partials'
    // write, fence, tile ticket and ordered reduction add about 6 us to a launch, which shorter splits do not win
    // back (measured on B200: 100 x 1024 x 2048 takes 16 us whole, 19 us in 2 splits, 20 us in 4)
    splits = 1;
    while (a.tiles * splits * 2 <= sms / 2 && a.nkb / (splits * 2) >= 24) splits *= 2;
  }
  a.kb_per = (a.nkb + splits - 1) / splits;
  a.splits = (a.nkb + a.kb_per - 1) / a.kb_per;  // every split owns at least one K block
  a.sc_smem = (K % 64 == 0 && (reinterpret_cast<uintptr_t>(S) & 3) == 0) ? 1 : 0;
  a.w_early = ctx->static_weights ? 1 : 0;
  a.ws = nullptr;
  a.counters = nullptr;
  if (a.splits > 1) {
    void *ws;
    uint32_t *cnt;
    rc = dc_scratch(ctx, (size_t)a.splits * M * N * sizeof(float), (size_t)a.tiles, &ws, &cnt);
    if (rc) return rc;
    a.ws = static_cast<float *>(ws);
    a.counters = cnt;
  }
  const int items = a.tiles * a.splits;
  const int grid = items < sms ? items : sms;
  DC_CUDA(dc_launch_pdl(ctx->stream, qgemm_ts<BITS, BT, EPI, ASM>, dim3(grid), dim3(T_THREADS), C::SMEM, tmX, tmW, a));
  return dc_launch_check("qgemm (ts)");
}

// Split count for the skinny form: fewest waves x K blocks per CTA, one CTA per SM.
int pick_splits(dc_ctx *ctx, int tiles, int nkb, size_t MN) {
  const int sms = ctx->sms > 0 ? ctx->sms : 148;
  int best = 1;
  double best_cost = 1e30;
  for (int s = 1; s <= nkb; s++) {
    if ((size_t)s * MN * 4 > ((size_t)256 << 20)) break;  // partials stay under 256 MB
    const int per = (nkb + s - 1) / s;
    const int used = (nkb + per - 1) / per;  // splits that get work
    if (used != s) continue;
    const int waves = (tiles * s + sms - 1) / sms;
    const double cost = waves * (per + 1.5) + (s > 1 ? 0.5 : 0.0);
    if (cost < best_cost - 1e-9) best_cost = cost, best = s;
  }
  return best;
}

}  // namespace

// Which prefill form serves a shape: the CTA pair (form 7) halves each SM's token bytes per K block, which pays on
// long reductions over large weights (its K-block pairing needs K % 128 == 0); the single-CTA tile (form 3) keeps
// a finer wave granularity and a cheaper epilogue, which wins while K is short. Measured at 16384 tokens: the pair
// is 5-10% faster on q4 5120x3072, 3072x3072 and 3072x8192 and 1% on the gated 16384x3072, level on q8 1024x3072,
// and 1-9% slower (the gated GLU twice slower) on every shape with K <= 2048.
static bool use_pair(int M, int N, int K) {
  (void)M;
  return K % 128 == 0 && K >= 3072 && (long)N * K >= (8L << 20);
}

int qgemm_launch_glu(dc_ctx *ctx, const void *X, const void *Wq, const void *S, void *Y, int M, int N, int K,
                     int bits, int act) {
  if (use_pair(M, N, K)) {
    if (bits == 8)
      return act == 1 ? launch_pair<8, 1>(ctx, X, Wq, S, Y, M, N, K) : launch_pair<8, 2>(ctx, X, Wq, S, Y, M, N, K);
    return act == 1 ? launch_pair<4, 1>(ctx, X, Wq, S, Y, M, N, K) : launch_pair<4, 2>(ctx, X, Wq, S, Y, M, N, K);
  }
  if (bits == 8)
    return act == 1 ? launch_ts<8, 256, 1, true>(ctx, X, Wq, S, Y, M, N, K, 1)
                    : launch_ts<8, 256, 2, true>(ctx, X, Wq, S, Y, M, N, K, 1);
  return act == 1 ? launch_ts<4, 256, 1, true>(ctx, X, Wq, S, Y, M, N, K, 1)
                  : launch_ts<4, 256, 2, true>(ctx, X, Wq, S, Y, M, N, K, 1);
}

int qgemm_direct_launch(dc_ctx *ctx, const void *X, const void *W16, void *Y, int M, int N, int K, int epilogue) {
  if (epilogue == 1) return launch_direct<1>(ctx, X, W16, Y, M, N, K);
  if (epilogue == 2) return launch_direct<2>(ctx, X, W16, Y, M, N, K);
  return launch_direct<0>(ctx, X, W16, Y, M, N, K);
}

int qgemm_pick_form(int M, int N, int K, int bits, int sms) {
  // decode shapes: the register weight stream up to 32 tokens on any weight and up to 64 on weights of 4M codes or
  // fewer (measured against form 4 at 17-64 tokens, q8 and q4: 12-70% faster there; on 8192 x 3072 at 40-64 tokens
  // level to 50% slower); then, up to 128 tokens, the tensor-memory form with a fitted token tile; then the largest
  // token tile whose tiles still fit one wave of CTAs (a launch of one wave is bound by its per-tile latency, so
  // more, smaller tiles finish sooner): 64 tokens (form 4), 192 (form 6); above that, the 256-token prefill form
  (void)bits;
  if (M <= 32 || (M <= 64 && (long)N * K <= (4L << 20))) return 5;
  if (M <= 128) return 4;
  if (sms <= 0) sms = 148;
  const long rows = (N + 127) / 128;
  if (rows * ((M + 63) / 64) <= sms) return 4;
  if (rows * ((M + 191) / 192) <= sms) return 6;
  return 3;
}

// Persistent-form tile width: the fewer waves of BN-wide tiles over the SMs, weighing the narrower MMA's higher
// shared-memory traffic per flop.
static int pick_bn(dc_ctx *ctx, int M, int N) {
  const int sms = ctx->sms > 0 ? ctx->sms : 148;
  const long tm = (M + 127) / 128;
  const long w256 = ((N + 255) / 256 * tm + sms - 1) / sms, w128 = ((N + 127) / 128 * tm + sms - 1) / sms;
  return (double)w256 * 256 <= (double)w128 * 128 * 1.15 ? 256 : 128;
}

int qgemm_launch(dc_ctx *ctx, const void *X, const void *Wq, const void *S, void *Y, int M, int N, int K, int bits,
                 int form, int splits) {
  if (form == 5) return gemv_launch(ctx, X, Wq, S, Y, M, N, K, bits, splits);
  if (form == 3) {
    if (use_pair(M, N, K))
      return bits == 8 ? launch_pair<8, 0>(ctx, X, Wq, S, Y, M, N, K) : launch_pair<4, 0>(ctx, X, Wq, S, Y, M, N, K);
    if (bits == 8) return launch_ts<8, 256, 0, true>(ctx, X, Wq, S, Y, M, N, K, 1);
    return launch_ts<4, 256, 0, true>(ctx, X, Wq, S, Y, M, N, K, 1);
  }
  if (form == 7) return bits == 8 ? launch_pair<8, 0>(ctx, X, Wq, S, Y, M, N, K) : launch_pair<4, 0>(ctx, X, Wq, S, Y, M, N, K);
  if (form == 6) {
    if (bits == 8) return launch_ts<8, 192, 0>(ctx, X, Wq, S, Y, M, N, K, 1);
    return launch_ts<4, 192, 0>(ctx, X, Wq, S, Y, M, N, K, 1);
  }
  if (form == 4) {
    // the TS form with a token tile fitted to M and K split across CTAs (decode shapes)
    // token tile: 16 or 32 covers M in one or two tiles; above 64 tokens two 64-token tiles beat one 128-token
    // tile (more CTAs on the weight stream)
    const int bt = M <= 16 ? 16 : M <= 64 ? 32 : 64;
#define DC_TS(B, T) \
    if (bits == B && bt == T) return launch_ts<B, T, 0>(ctx, X, Wq, S, Y, M, N, K, splits);
    DC_TS(8, 16) DC_TS(8, 32) DC_TS(8, 64) DC_TS(8, 128)
    DC_TS(4, 16) DC_TS(4, 32) DC_TS(4, 64) DC_TS(4, 128)
#undef DC_TS
  }
  if (form == 2) {
    const int bn = pick_bn(ctx, M, N);
    if (bits == 8)
      return bn == 256 ? launch_persistent<8, 256, 0>(ctx, X, Wq, S, Y, M, N, K)
                       : launch_persistent<8, 128, 0>(ctx, X, Wq, S, Y, M, N, K);
    return bn == 256 ? launch_persistent<4, 256, 0>(ctx, X, Wq, S, Y, M, N, K)
                     : launch_persistent<4, 128, 0>(ctx, X, Wq, S, Y, M, N, K);
  }
  if (form == 0) {
    const long tiles256 = (long)((N + 255) / 256) * ((M + 127) / 128);
    const bool wide = tiles256 >= 2L * (ctx->sms > 0 ? ctx->sms : 148);
    if (bits == 8)
      return wide ? launch_cfg<8, 0, 256>(ctx, X, Wq, S, Y, M, N, K, 1) : launch_cfg<8, 0, 128>(ctx, X, Wq, S, Y, M, N, K, 1);
    return wide ? launch_cfg<4, 0, 256>(ctx, X, Wq, S, Y, M, N, K, 1) : launch_cfg<4, 0, 128>(ctx, X, Wq, S, Y, M, N, K, 1);
  }
  const int bt = M <= 16 ? 16 : M <= 32 ? 32 : M <= 64 ? 64 : 128;
  const int tiles = ((N + 127) / 128) * ((M + bt - 1) / bt);
  const int nkb = (K + BK - 1) / BK;
  if (splits <= 0) splits = pick_splits(ctx, tiles, nkb, (size_t)M * N);
  if (splits > nkb) splits = nkb;
  {  // every split must own at least one K block
    const int per = (nkb + splits - 1) / splits;
    splits = (nkb + per - 1) / per;
  }
#define DC_SKINNY(B, T) \
  if (bits == B && bt == T) return launch_cfg<B, 1, T>(ctx, X, Wq, S, Y, M, N, K, splits);
  DC_SKINNY(8, 16) DC_SKINNY(8, 32) DC_SKINNY(8, 64) DC_SKINNY(8, 128)
  DC_SKINNY(4, 16) DC_SKINNY(4, 32) DC_SKINNY(4, 64) DC_SKINNY(4, 128)
#undef DC_SKINNY
  return dc_fail(DC_EINVAL, "decision.js: no skinny matmul for bits=%d", bits);
}

// ------------------------------------------------------------------ allocation-free skinny matmul
// dc_qmatmul_skinny_noalloc: the skinny (split-K) form for callers that must not allocate device memory, e.g. a
// plug-in inside a host process that owns every byte of device memory and forbids cudaMalloc after start-up, or a
// latency-bound serving loop where cudaMalloc's implicit device synchronisation is not acceptable. Its split-K
// partials, tile counters and error word live in one file-scope static device array instead of the context's
// grow-only scratch, so the call needs no dc_ctx and allocates nothing.

namespace {

constexpr size_t kNoallocPartialBytes = (size_t)16 << 20;  // f32 split-K partials: splits * M * N * 4 <= 16 MiB
constexpr size_t kNoallocCounters = 4096;                   // one per output tile: ceil(N/128) * ceil(M/BT) <= 4096
constexpr size_t kNoallocCounterOff = kNoallocPartialBytes;
constexpr size_t kNoallocErrOff = kNoallocCounterOff + kNoallocCounters * sizeof(uint32_t);
constexpr size_t kNoallocBytes = kNoallocErrOff + 256;

// Every GPU that loads this library holds these bytes until the process exits.
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoallocBytes];

constexpr int kMaxDevices = 64;
static void *g_noalloc_addr[kMaxDevices];
static std::mutex g_noalloc_mu[kMaxDevices];

// The device address of g_noalloc_scratch on the current device (host code may not use the symbol itself: on the
// host it names a stand-in, not device memory). Looked up on the device's first call and kept once found; a failed
// lookup (e.g. a first call made during stream capture) is not kept, its error is cleared from the runtime, and
// the next call tries again.
int noalloc_scratch(int device, uint8_t **out) {
  DC_CHECK(device >= 0 && device < kMaxDevices, DC_EINVAL, "decision.js: device %d out of range", device);
  std::lock_guard<std::mutex> lock(g_noalloc_mu[device]);
  if (!g_noalloc_addr[device]) {
    void *p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p) {
      cudaGetLastError();
      return dc_fail(DC_ECUDA, "decision.js: cannot resolve the static scratch on device %d: %s", device,
                     cudaGetErrorString(e));
    }
    g_noalloc_addr[device] = p;
  }
  *out = static_cast<uint8_t *>(g_noalloc_addr[device]);
  return DC_OK;
}

template <int BITS, int BT>
int launch_skinny_noalloc(cudaStream_t stream, uint8_t *scratch, const void *X, const void *Wq, const void *S,
                          void *Y, int M, int N, int K, int splits) {
  using C = Cfg<BITS, 1, BT>;
  CUtensorMap tmX, tmW;
  int rc = make_map(&tmX, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, X, (uint64_t)K, (uint64_t)M, (uint64_t)K * 2, BK,
                    C::ROWS_X, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  const uint64_t wrow = (uint64_t)K * BITS / 8;
  rc = make_map(&tmW, CU_TENSOR_MAP_DATA_TYPE_UINT8, Wq, wrow, (uint64_t)N, wrow, BK * BITS / 8, C::ROWS_W,
                CU_TENSOR_MAP_SWIZZLE_NONE);
  if (rc) return rc;
  DC_CUDA(cudaFuncSetAttribute(qgemm_kernel<BITS, 1, BT>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM));
  GemmArgs a;
  a.Y = static_cast<__half *>(Y);
  a.S = static_cast<const __half *>(S);
  a.err = reinterpret_cast<uint32_t *>(scratch + kNoallocErrOff);
  a.M = M, a.N = N, a.K = K;
  a.nkb = (K + BK - 1) / BK;
  a.splits = splits;
  a.ws = reinterpret_cast<float *>(scratch);
  a.counters = reinterpret_cast<uint32_t *>(scratch + kNoallocCounterOff);
  const int tn = (N + C::ROWS_W - 1) / C::ROWS_W, tm = (M + C::ROWS_X - 1) / C::ROWS_X;
  // the tile counters must start at zero; the previous call leaves them at zero unless it was cut short
  DC_CUDA(cudaMemsetAsync(a.counters, 0, (size_t)tn * tm * sizeof(uint32_t), stream));
  qgemm_kernel<BITS, 1, BT><<<dim3(tn, splits, tm), THREADS, C::SMEM, stream>>>(tmX, tmW, a);
  return dc_launch_check("qgemm (no-alloc)");
}

}  // namespace

extern "C" int dc_qmatmul_skinny_noalloc(void *stream, const void *X, const void *Wq, const void *S, void *Y, int M,
                                         int N, int K, int bits, int splits) {
  DC_CHECK(X && Wq && S && Y, DC_EINVAL, "decision.js: qmatmul (no-alloc): null pointer");
  DC_CHECK(M > 0 && M <= 128 && N > 0 && K > 0 && K % 32 == 0, DC_EINVAL,
           "decision.js: qmatmul (no-alloc): needs 1 <= M <= 128 and K a multiple of 32 (M=%d N=%d K=%d)", M, N, K);
  DC_CHECK(bits == 8 || bits == 4, DC_EINVAL, "decision.js: qmatmul (no-alloc): bits must be 4 or 8 (got %d)", bits);
  DC_CHECK((((uintptr_t)X | (uintptr_t)Wq) & 15) == 0, DC_EINVAL,
           "decision.js: qmatmul (no-alloc): X and the codes must be 16-byte aligned");
  DC_CHECK((((uintptr_t)S | (uintptr_t)Y) & 1) == 0, DC_EINVAL,
           "decision.js: qmatmul (no-alloc): the scales and Y must be 2-byte aligned");
  int device = 0;
  DC_CUDA(cudaGetDevice(&device));
  uint8_t *scratch = nullptr;
  int rc = noalloc_scratch(device, &scratch);
  if (rc) return rc;
  const int bt = M <= 16 ? 16 : M <= 32 ? 32 : M <= 64 ? 64 : 128;
  const int tiles = ((N + 127) / 128) * ((M + bt - 1) / bt);
  DC_CHECK((size_t)tiles <= kNoallocCounters, DC_EINVAL,
           "decision.js: qmatmul (no-alloc): %d output tiles exceed the static limit of %zu (N <= %zu at M <= 16)",
           tiles, kNoallocCounters, kNoallocCounters * 128);
  const int nkb = (K + BK - 1) / BK;
  const size_t per_split = (size_t)M * N * sizeof(float);
  if (splits <= 0) {
    int sms = 148;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
    dc_ctx probe;
    probe.sms = sms;
    splits = pick_splits(&probe, tiles, nkb, (size_t)M * N);
    while (splits > 1 && (size_t)splits * per_split > kNoallocPartialBytes) splits--;
  }
  if (splits > nkb) splits = nkb;
  {  // every split must own at least one K block
    const int per = (nkb + splits - 1) / splits;
    splits = (nkb + per - 1) / per;
  }
  DC_CHECK(splits == 1 || (size_t)splits * per_split <= kNoallocPartialBytes, DC_EINVAL,
           "decision.js: qmatmul (no-alloc): %d splits x %d x %d f32 partials need %zu bytes, over the static "
           "limit of %zu",
           splits, M, N, (size_t)splits * per_split, kNoallocPartialBytes);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
#define DC_NOALLOC(B, T) \
  if (bits == B && bt == T) return launch_skinny_noalloc<B, T>(st, scratch, X, Wq, S, Y, M, N, K, splits);
  DC_NOALLOC(8, 16) DC_NOALLOC(8, 32) DC_NOALLOC(8, 64) DC_NOALLOC(8, 128)
  DC_NOALLOC(4, 16) DC_NOALLOC(4, 32) DC_NOALLOC(4, 64) DC_NOALLOC(4, 128)
#undef DC_NOALLOC
  return dc_fail(DC_EINVAL, "decision.js: qmatmul (no-alloc): unsupported shape");
}
