// The decode-shape quantized matmul (M <= 64 tokens): Y[M,N] = X[M,K] . deq(W)[N,K]^T with the semantics of
// MATMUL_PORTABLE_Q8/Q4 (src/kernels.ts:445-520: f16((code - Z) * scale) dequantisation, f32 accumulation,
// f16 out), as a pure weight stream: every code byte is read once from HBM by a 128-bit load, dequantized in
// registers and multiplied on the tensor pipe (mma.sync m16n8k16, f16 operands, f32 accumulators), so no shared
// memory round trip sits on the weight path and no shuffles are needed for the dot products.
//
// Layout of the work:
//  - a CTA owns 16 weight rows x a K part; its 8 warps take the part's steps in turn (warp w: steps w, w + 8,
//    ...), so the CTA reads 512 contiguous bytes of each row per round and the grid holds enough small CTAs
//    (few registers, four per SM) to keep HBM busy;
//  - per step (64 q8 or 128 q4 codes of 16 rows), lane (g = lane/4, t = lane%4) loads the 16-byte vector at byte
//    16t of rows g and g+8 (one warp load = 64 contiguous bytes of 8 rows; one scale group per row) and feeds it
//    to 4 (q8) or 8 (q4) m16n8k16 MMAs in which it supplies 4 codes of each of its two rows. The reduction
//    dimension may be permuted freely as long as the tokens (the B operand) follow: q8 keeps the natural order,
//    q4 pairs even and odd nibbles and the token fragments are permuted to match (0 2 1 3 within 4 codes);
//  - tokens are read straight from global memory through L1 (only lanes whose token exists load); the next
//    step's codes are in flight while the current one is multiplied;
//  - launched as a programmatic dependent launch: in the model passes (weights written before the pass) the first
//    codes are requested while the kernel before it in the stream drains, and the next kernel may launch as soon
//    as this one has started (griddepcontrol);
//  - the 8 warps' partial sums meet in shared memory (added in warp order); when K is split over several CTAs
//    (few rows, long K) those form a thread-block cluster (<= 8) and add their partials through distributed
//    shared memory in part order. Deterministic, no global scratch, no counters.
// Three kernels share this layout: qgemv_even_kernel (K a whole number of steps, up to 32 tokens: every load
// unconditional, the default), qgemv_kernel (any K, any token count up to 64) and qgemv_staged_kernel (codes by
// bulk copies into shared memory, for the 9-16-token shapes where it measured faster).
#include <atomic>

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "dc_internal.h"
#include "dc_ptx.cuh"

using namespace dcx;

namespace {

constexpr int GV_THREADS = 256;
constexpr int GV_WARPS = GV_THREADS / 32;
constexpr int GV_ROWS = 16;       // weight rows per CTA
// codes per warp step: one 16-byte vector per lane and row (q8 16 codes, q4 32 codes)
template <int BITS>
struct GvStep {
  static constexpr int CODES = BITS == 8 ? 64 : 128;
  static constexpr int PER_LANE = CODES / 4;
  static constexpr int MMAS = PER_LANE / 4;  // m16n8k16 per step (each takes 4 codes of a row from a lane)
};
constexpr int GV_MAX_PARTS = 8;   // portable cluster size



__device__ __forceinline__ uint4 ld_stream(const void *p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t h2u(__half2 h) { return *reinterpret_cast<uint32_t *>(&h); }

// Eight q4 codes (one word, low nibble first) -> {c0, c2}, {c4, c6}, {c1, c3}, {c5, c7}, each exactly
// f16((c - 8) * scale): the even nibbles and the odd nibbles each go through one 0x64 magic byte permute.
__device__ __forceinline__ void deq_q4_pairs(uint32_t w, __half2 s2, uint32_t (&o)[4]) {
  const uint32_t magic = 0x64646464u;
  const uint32_t lo = w & 0x0F0F0F0Fu;         // c0 c2 c4 c6
  const uint32_t hi = (w >> 4) & 0x0F0F0F0Fu;  // c1 c3 c5 c7
  uint32_t p[4];
  asm("prmt.b32 %0, %1, %2, 0x5150;" : "=r"(p[0]) : "r"(lo), "r"(magic));  // c0 c2
  asm("prmt.b32 %0, %1, %2, 0x5352;" : "=r"(p[1]) : "r"(lo), "r"(magic));  // c4 c6
  asm("prmt.b32 %0, %1, %2, 0x5150;" : "=r"(p[2]) : "r"(hi), "r"(magic));  // c1 c3
  asm("prmt.b32 %0, %1, %2, 0x5352;" : "=r"(p[3]) : "r"(hi), "r"(magic));  // c5 c7
  const __half2 z = __halves2half2(__ushort_as_half(0x6408), __ushort_as_half(0x6408));  // 1032
#pragma unroll
  for (int e = 0; e < 4; e++) o[e] = h2u(__hmul2(__hsub2(*reinterpret_cast<__half2 *>(&p[e]), z), s2));
}

// Eight q4 codes (one word, low nibble first) -> {c0, c4}, {c1, c5}, {c2, c6}, {c3, c7}, each exactly
// f16((c - 8) * scale). (w & 0x000F000F) | 0x64006400 is the half pair {1024 + c0, 1024 + c4}; the nibbles at bits
// 4 and 20 land as 1024 + 16 c, and 1/16 * (1024 + 16 c) - 72 = c - 8 is exact in one fused multiply-add.
__device__ __forceinline__ void deq_q4_spread(uint32_t w, __half2 s2, uint32_t (&o)[4]) {
  const uint32_t w8 = w >> 8;
  uint32_t p[4] = {(w & 0x000F000Fu) | 0x64006400u, (w & 0x00F000F0u) | 0x64006400u, (w8 & 0x000F000Fu) | 0x64006400u,
                   (w8 & 0x00F000F0u) | 0x64006400u};
  const __half2 z = __halves2half2(__ushort_as_half(0x6408), __ushort_as_half(0x6408));      // 1032
  const __half2 k16 = __halves2half2(__ushort_as_half(0x2C00), __ushort_as_half(0x2C00));    // 1/16
  const __half2 m72 = __halves2half2(__ushort_as_half(0xD480), __ushort_as_half(0xD480));    // -72
  o[0] = h2u(__hmul2(__hsub2(*reinterpret_cast<__half2 *>(&p[0]), z), s2));
  o[1] = h2u(__hmul2(__hfma2(*reinterpret_cast<__half2 *>(&p[1]), k16, m72), s2));
  o[2] = h2u(__hmul2(__hsub2(*reinterpret_cast<__half2 *>(&p[2]), z), s2));
  o[3] = h2u(__hmul2(__hfma2(*reinterpret_cast<__half2 *>(&p[3]), k16, m72), s2));
}

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ float ld_dsmem(const float *p, uint32_t rank) {
  uint32_t a = smem_u32(p), ra;
  float v;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(ra) : "r"(a), "r"(rank));
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(ra) : "memory");
  return v;
}

// Registers of one step: the lane's 16-byte vector of rows g and g + 8 and their scales (one group each).
struct Step {
  uint4 c[2];
  uint32_t s;  // scale of row g (low half) and row g + 8 (high half)
};

template <int BITS, int NT>
__global__ void __launch_bounds__(GV_THREADS, NT == 1 ? 4 : 2)
    qgemv_kernel(const __half *__restrict__ X, const uint8_t *__restrict__ W, const __half *__restrict__ S,
                 __half *__restrict__ Y, int M, int N, int K, int kc, int w_early) {
  constexpr int TOK = NT * 8;
  using G = GvStep<BITS>;
  using B = Step;
  __shared__ float red[GV_WARPS][TOK][GV_ROWS];
  __shared__ float part[TOK][GV_ROWS];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int n0 = blockIdx.x * GV_ROWS;
  const int k0 = blockIdx.y * kc, k1 = min(K, k0 + kc);
  const int nsteps = (k1 - k0 + G::CODES - 1) / G::CODES;

  const int r0 = n0 + g, r1 = r0 + 8;
  const bool v0 = r0 < N, v1 = r1 < N;
  const size_t rowb = (size_t)K * BITS / 8;
  const int kq = K / 32;
  const uint8_t *w0 = W + (size_t)(v0 ? r0 : 0) * rowb;
  const uint8_t *w1 = W + (size_t)(v1 ? r1 : 0) * rowb;
  const unsigned short *s0 = reinterpret_cast<const unsigned short *>(S) + (size_t)(v0 ? r0 : 0) * kq;
  const unsigned short *s1 = reinterpret_cast<const unsigned short *>(S) + (size_t)(v1 ? r1 : 0) * kq;
  // the lane's token rows (B operand column g of each 8-token tile)
  const __half *xr[NT];
  bool xv[NT];
#pragma unroll
  for (int j = 0; j < NT; j++) {
    xv[j] = j * 8 + g < M;
    xr[j] = X + (size_t)(xv[j] ? j * 8 + g : 0) * K;
  }

  // step s: the lane's codes [s * CODES + PER_LANE * t, +PER_LANE) of its two rows; zero codes and zero scales
  // beyond the K part or beyond N (they then contribute +-0)
  auto load = [&](int s, B &b) {
    const int kk = k0 + s * G::CODES + G::PER_LANE * t;
    const bool in = s < nsteps && kk < k1;
    const size_t off = (size_t)kk * BITS / 8;
    b.c[0] = (in && v0) ? ld_stream(w0 + off) : make_uint4(0, 0, 0, 0);
    b.c[1] = (in && v1) ? ld_stream(w1 + off) : make_uint4(0, 0, 0, 0);
    const uint32_t lo = (in && v0) ? __ldg(s0 + kk / 32) : 0u;
    const uint32_t hi = (in && v1) ? __ldg(s1 + kk / 32) : 0u;
    b.s = lo | (hi << 16);
  };

  float acc[NT][4];
#pragma unroll
  for (int j = 0; j < NT; j++) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;

  auto compute = [&](int s, const B &b) {
    if (s >= nsteps) return;
    const unsigned short slo = (unsigned short)(b.s & 0xFFFF), shi = (unsigned short)(b.s >> 16);
    const __half2 sg = __halves2half2(__ushort_as_half(slo), __ushort_as_half(slo));
    const __half2 sh = __halves2half2(__ushort_as_half(shi), __ushort_as_half(shi));
    // the lane's first code of this step (tokens beyond k1 multiply zero codes; X rows are K long, so the token
    // loads stay in bounds for kk < K)
    const int kb = k0 + s * G::CODES + G::PER_LANE * t;
#pragma unroll
    for (int h = 0; h < G::MMAS / 4; h++) {  // groups of 4 MMAs: token fragments for one group in flight
      // (up to 16 tokens the group's fragments are loaded up front; with more, each MMA's just before it, so the
      // registers hold one group of dequantized codes and the NT accumulators)
      constexpr int XF = NT <= 2 ? NT : 1;
      uint2 xf[XF][4];
      if (NT <= 2) {
#pragma unroll
        for (int e = 0; e < 4; e++) {
          const int xo = 4 * (4 * h + e);
#pragma unroll
          for (int j = 0; j < XF; j++)
            xf[j][e] = (xv[j] && kb + xo < K) ? __ldg(reinterpret_cast<const uint2 *>(xr[j] + kb + xo))
                                              : make_uint2(0, 0);
        }
      }
      uint32_t pg[4], ph[4];  // q4: the dequantized pairs of the current word of each row
#pragma unroll
      for (int e = 0; e < 4; e++) {  // one MMA per 4 codes of each row
        const int q = 4 * h + e;
        uint32_t a0, a1, a2, a3;
        if (BITS == 8) {
          // MMA q: word q of the vector (codes 16t + 4q .. +3)
          const uint32_t wg = (&b.c[0].x)[q], wh = (&b.c[1].x)[q];
          __half2 g01, g23, h01, h23;
          deq_q8_word(wg, sg, g01, g23);
          deq_q8_word(wh, sh, h01, h23);
          a0 = h2u(g01), a1 = h2u(h01), a2 = h2u(g23), a3 = h2u(h23);
        } else {
          // word q/2 holds 8 codes; MMA q uses pairs {c0,c2},{c1,c3} (q even) or {c4,c6},{c5,c7} (q odd)
          if ((q & 1) == 0) {
            deq_q4_pairs((&b.c[0].x)[q >> 1], sg, pg);
            deq_q4_pairs((&b.c[1].x)[q >> 1], sh, ph);
          }
          a0 = pg[q & 1], a1 = ph[q & 1], a2 = pg[2 + (q & 1)], a3 = ph[2 + (q & 1)];
        }
#pragma unroll
        for (int j = 0; j < NT; j++) {
          uint2 x2;
          if (NT <= 2) {
            x2 = xf[NT <= 2 ? j : 0][e];
          } else {
            const int xo = 4 * q;
            x2 = (xv[j] && kb + xo < K) ? __ldg(reinterpret_cast<const uint2 *>(xr[j] + kb + xo)) : make_uint2(0, 0);
          }
          uint32_t b0 = x2.x, b1 = x2.y;
          if (BITS == 4) {
            // tokens {x0 x1}, {x2 x3} -> {x0 x2}, {x1 x3}, the order of deq_q4_pairs
            const uint32_t p = b0, r = b1;
            asm("prmt.b32 %0, %1, %2, 0x5410;" : "=r"(b0) : "r"(p), "r"(r));
            asm("prmt.b32 %0, %1, %2, 0x7632;" : "=r"(b1) : "r"(p), "r"(r));
          }
          mma16816(acc[j], a0, a1, a2, a3, b0, b1);
        }
      }
    }
  };

  // programmatic dependent launch: let the next kernel in the stream launch now; with static weights (the model
  // passes) the first weight step is requested before waiting for the previous kernel's results
  asm volatile("griddepcontrol.launch_dependents;");
  B ba, bb;
  if (!w_early) asm volatile("griddepcontrol.wait;" ::: "memory");
  load(warp, ba);
  if (w_early) asm volatile("griddepcontrol.wait;" ::: "memory");  // X (and Y) only after the kernel before
  for (int s = warp; s < nsteps; s += 2 * GV_WARPS) {
    load(s + GV_WARPS, bb);
    compute(s, ba);
    load(s + 2 * GV_WARPS, ba);
    compute(s + GV_WARPS, bb);
  }

  // accumulator (m16n8): {c0, c1} = row g, tokens 2t, 2t+1; {c2, c3} = row g + 8
#pragma unroll
  for (int j = 0; j < NT; j++) {
    const int tk = j * 8 + 2 * t;
    red[warp][tk][g] = acc[j][0];
    red[warp][tk + 1][g] = acc[j][1];
    red[warp][tk][g + 8] = acc[j][2];
    red[warp][tk + 1][g + 8] = acc[j][3];
  }
  __syncthreads();
  const int parts = gridDim.y;
  // TOK x 16 outputs per CTA: one per thread up to 16 tokens, several beyond
  for (int i = threadIdx.x; i < TOK * GV_ROWS; i += GV_THREADS) {
    const int m = i / GV_ROWS, r = i % GV_ROWS;
    float v = 0.f;
#pragma unroll
    for (int w = 0; w < GV_WARPS; w++) v += red[w][m][r];
    if (parts == 1) {
      if (m < M && n0 + r < N) Y[(size_t)m * N + n0 + r] = __float2half_rn(v);
    } else {
      part[m][r] = v;
    }
  }
  if (parts == 1) return;
  // K parts: the cluster adds its partials in part order; CTA `rank` finishes every parts-th output
  cluster_sync();
  const uint32_t rank = cluster_rank();
  for (int i = threadIdx.x; i < TOK * GV_ROWS; i += GV_THREADS) {
    const int m = i / GV_ROWS, r = i % GV_ROWS;
    if (m < M && n0 + r < N && (uint32_t)(i % parts) == rank) {
      float sum = 0.f;
      for (int q = 0; q < parts; q++) sum += ld_dsmem(&part[m][r], (uint32_t)q);
      Y[(size_t)m * N + n0 + r] = __float2half_rn(sum);
    }
  }
  cluster_sync();  // no CTA leaves while a peer still reads its partial
}

// ------------------------------------------------------------------ staged form
// The same arithmetic with the weight stream landing in shared memory: a CTA (8 warps) owns 16 rows x one K part
// and, before anything else, has all of its part's codes and scales in flight: one bulk copy (cp.async.bulk) per row
// and K quarter, completing on the quarter's mbarrier, so issuing them costs 64 instructions per CTA and holds no
// registers. Only then does it wait for the kernel before it (griddepcontrol.wait) and read the tokens. A launch is
// thus one memory round trip deep instead of one per step pair, and as CTAs finish, the next launch's CTAs move in
// and start their copies while this one drains. The warps multiply a quarter as soon as its barrier completes,
// while the later quarters still stream in, alternating between two accumulator sets so consecutive MMAs do not
// wait on each other. Shared-memory rows are padded to 64 (mod 128) bytes: the 8 lanes of a quarter-warp (two
// rows, four 16-byte vectors each) hit 32 distinct banks. After the last step the code buffer holds the warps'
// partial sums. Every wait is bounded (an expired wait sets the device error word).
constexpr int GS_THREADS = 256;
constexpr int GS_WARPS = GS_THREADS / 32;
constexpr int GS_GROUPS = 4;

__host__ __device__ constexpr int gs_row_stride(int kcb) { return (kcb + 127) / 128 * 128 + 64; }
__host__ __device__ constexpr int gs_scale_stride(int kc) { return (kc / 32 + 7) / 8 * 8; }  // 16-byte rows

// codes, scales, GS_GROUPS barriers and an abort flag; the partial sums (GS_WARPS x TOK x 16 floats, then
// TOK x 16) reuse the code buffer
template <int NT>
__host__ __device__ constexpr int gs_smem_main(int kc, int bits) {
  return GV_ROWS * gs_row_stride(kc * bits / 8) + GV_ROWS * gs_scale_stride(kc) * 2;
}
template <int NT>
__host__ __device__ constexpr int gs_smem(int kc, int bits) {
  return (gs_smem_main<NT>(kc, bits) > (GS_WARPS + 1) * NT * 8 * GV_ROWS * 4 ? gs_smem_main<NT>(kc, bits)
                                                                              : (GS_WARPS + 1) * NT * 8 * GV_ROWS * 4) +
         8 * GS_GROUPS + 16;
}

__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void *src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
               "l"(src), "r"(bytes), "r"(bar)
               : "memory");
}

template <int BITS, int NT, bool EVEN>
__global__ void __launch_bounds__(GS_THREADS, BITS == 4 && NT == 2 ? 3 : 4)
    qgemv_staged_kernel(const __half *__restrict__ X, const uint8_t *__restrict__ W, const __half *__restrict__ S,
                        __half *__restrict__ Y, int M, int N, int K, int kc, int w_early, uint32_t *err) {
  constexpr int TOK = NT * 8;
  using G = GvStep<BITS>;
  extern __shared__ __align__(128) uint8_t gs_sm[];
  const int kcb = kc * BITS / 8, rs = gs_row_stride(kcb), kgp = gs_scale_stride(kc);
  uint8_t *codes = gs_sm;                                                         // [16][rs]
  unsigned short *scl = reinterpret_cast<unsigned short *>(gs_sm + GV_ROWS * rs);  // [16][kgp]
  const int main_bytes = GV_ROWS * rs + GV_ROWS * kgp * 2;
  const int red_bytes = (GS_WARPS + 1) * TOK * GV_ROWS * 4;
  const uint32_t bar0 = smem_u32(gs_sm + (main_bytes > red_bytes ? main_bytes : red_bytes));
  volatile int *abort = reinterpret_cast<volatile int *>(gs_sm + (main_bytes > red_bytes ? main_bytes : red_bytes) +
                                                         8 * GS_GROUPS);
  float *red = reinterpret_cast<float *>(gs_sm);  // [8][TOK][16], after the steps
  float *part = red + GS_WARPS * TOK * GV_ROWS;   // [TOK][16]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int n0 = blockIdx.x * GV_ROWS;
  const int k0 = blockIdx.y * kc, k1 = min(K, k0 + kc);
  const int vb = (k1 - k0) * BITS / 8;  // valid code bytes of each row's part (a multiple of 16: K % 32 == 0)
  const int kgv = (k1 - k0) / 32;       // valid scales of each row's part
  const int nsteps = (k1 - k0 + G::CODES - 1) / G::CODES;
  const int rows = min(GV_ROWS, N - n0);
  const size_t rowb = (size_t)K * BITS / 8;
  const int kq = K / 32;
  auto gend = [&](int grp) { return (nsteps * (grp + 1) + GS_GROUPS - 1) / GS_GROUPS; };  // in steps
  // the scale rows go by bulk copy when every source row is 16-byte aligned and a multiple of 16 bytes long
  const unsigned short *Su = reinterpret_cast<const unsigned short *>(S);
  const bool sbulk = ((reinterpret_cast<uintptr_t>(Su + k0 / 32) | (uintptr_t)kq * 2 | (uintptr_t)kgv * 2) & 15) == 0;

  asm volatile("griddepcontrol.launch_dependents;");
  if (threadIdx.x == 0) {
    for (int q = 0; q < GS_GROUPS; q++) mbar_init(bar0 + 8 * q, 1);
    *abort = 0;
    mbar_init_fence();
  }
  if (!w_early) asm volatile("griddepcontrol.wait;" ::: "memory");
  // zero what no copy writes: whole rows beyond N, each row's bytes beyond the part, the scales beyond the part
  // (all of them when they go by plain loads, written below)
  for (int r = rows; r < GV_ROWS; r++)
    for (int i = threadIdx.x; i < kcb / 16; i += GS_THREADS)
      *reinterpret_cast<uint4 *>(codes + r * rs + 16 * i) = make_uint4(0, 0, 0, 0);
  if (vb < kcb)
    for (int i = threadIdx.x; i < GV_ROWS * ((kcb - vb) / 16); i += GS_THREADS) {
      const int r = i / ((kcb - vb) / 16), c = i % ((kcb - vb) / 16);
      *reinterpret_cast<uint4 *>(codes + r * rs + vb + 16 * c) = make_uint4(0, 0, 0, 0);
    }
  for (int i = threadIdx.x; i < GV_ROWS * kgp; i += GS_THREADS) {
    const int r = i / kgp, q = i % kgp;
    if (!sbulk || r >= rows || q >= kgv) scl[i] = 0;
  }
  __syncthreads();  // barriers initialised, zero fills done
  if (threadIdx.x < GS_GROUPS * 16) {
    // thread (group q, row r): row r's bytes of quarter q; lane 0 of each group announces the group's bytes first
    const int q = threadIdx.x >> 4, r = threadIdx.x & 15;
    const int lo = q == 0 ? 0 : min(vb, 64 * gend(q - 1)), hi = min(vb, 64 * gend(q));
    const uint32_t bar = bar0 + 8 * q;
    if (r == 0) {
      uint32_t bytes = (uint32_t)(rows * (hi - lo));
      if (q == 0 && sbulk) bytes += (uint32_t)(rows * kgv * 2);
      mbar_expect_tx(bar, bytes);  // (the arrival: the phase cannot complete before it)
    }
    __syncwarp();
    if (r < rows) {
      if (hi > lo) bulk_g2s(smem_u32(codes + r * rs + lo), W + (size_t)(n0 + r) * rowb + (size_t)k0 * BITS / 8 + lo,
                            (uint32_t)(hi - lo), bar);
      if (q == 0 && sbulk && kgv > 0)
        bulk_g2s(smem_u32(scl + r * kgp), Su + (size_t)(n0 + r) * kq + k0 / 32, (uint32_t)(kgv * 2), bar);
    }
  }
  if (!sbulk) {
    // unaligned scale rows: plain loads, all in flight before any is stored
    constexpr int SB = 8;
    for (int b0 = 0; b0 < rows * kgv; b0 += GS_THREADS * SB) {
      unsigned short v[SB];
#pragma unroll
      for (int u = 0; u < SB; u++) {
        const int i = b0 + u * GS_THREADS + threadIdx.x;
        v[u] = i < rows * kgv ? __ldg(Su + (size_t)(n0 + i / kgv) * kq + k0 / 32 + i % kgv) : (unsigned short)0;
      }
#pragma unroll
      for (int u = 0; u < SB; u++) {
        const int i = b0 + u * GS_THREADS + threadIdx.x;
        if (i < rows * kgv) scl[(i / kgv) * kgp + i % kgv] = v[u];
      }
    }
    __syncthreads();
  }
  if (w_early) asm volatile("griddepcontrol.wait;" ::: "memory");  // X (and Y) only after the kernel before

  const __half *xr[NT];
  bool xv[NT];
#pragma unroll
  for (int j = 0; j < NT; j++) {
    xv[j] = j * 8 + g < M;
    xr[j] = X + (size_t)(xv[j] ? j * 8 + g : 0) * K + k0 + G::PER_LANE * t;
  }
  const uint8_t *cA = codes + g * rs + 16 * t, *cB = cA + 8 * rs;
  const unsigned short *sA = scl + g * kgp + G::PER_LANE * t / 32, *sB = sA + 8 * kgp;
  float acc[NT][2][4];
#pragma unroll
  for (int j = 0; j < NT; j++)
#pragma unroll
    for (int u = 0; u < 2; u++) acc[j][u][0] = acc[j][u][1] = acc[j][u][2] = acc[j][u][3] = 0.f;

  auto compute = [&](int s) {
    const uint4 c0 = *reinterpret_cast<const uint4 *>(cA + 64 * s);
    const uint4 c1 = *reinterpret_cast<const uint4 *>(cB + 64 * s);
    const unsigned short slo = sA[s * (G::CODES / 32)], shi = sB[s * (G::CODES / 32)];
    const __half2 sg = __halves2half2(__ushort_as_half(slo), __ushort_as_half(slo));
    const __half2 sh = __halves2half2(__ushort_as_half(shi), __ushort_as_half(shi));
    const int xo0 = s * G::CODES;  // the lane's tokens of this step start at xr + xo0 (PER_LANE of them)
#pragma unroll
    for (int h = 0; h < G::MMAS / 4; h++) {
      uint4 xq[NT][2];  // the 16 tokens of this group of 4 MMAs
#pragma unroll
      for (int j = 0; j < NT; j++)
#pragma unroll
        for (int u = 0; u < 2; u++) {
          const int xo = xo0 + 16 * h + 8 * u;
          xq[j][u] = (xv[j] && (EVEN || k0 + G::PER_LANE * t + xo < K))
                         ? __ldg(reinterpret_cast<const uint4 *>(xr[j] + xo))
                         : make_uint4(0, 0, 0, 0);
        }
      uint32_t pg[4], ph[4];
#pragma unroll
      for (int e = 0; e < 4; e++) {
        const int q = 4 * h + e;
        uint32_t a0, a1, a2, a3;
        if (BITS == 8) {
          const uint32_t wg = (&c0.x)[q], wh = (&c1.x)[q];
          __half2 g01, g23, h01, h23;
          deq_q8_word(wg, sg, g01, g23);
          deq_q8_word(wh, sh, h01, h23);
          a0 = h2u(g01), a1 = h2u(h01), a2 = h2u(g23), a3 = h2u(h23);
        } else {
          if ((q & 1) == 0) {
            deq_q4_pairs((&c0.x)[q >> 1], sg, pg);
            deq_q4_pairs((&c1.x)[q >> 1], sh, ph);
          }
          a0 = pg[q & 1], a1 = ph[q & 1], a2 = pg[2 + (q & 1)], a3 = ph[2 + (q & 1)];
        }
#pragma unroll
        for (int j = 0; j < NT; j++) {
          const uint32_t *xw = &xq[j][e >> 1].x + 2 * (e & 1);  // tokens 4q .. 4q + 3 of the lane's run
          uint32_t b0 = xw[0], b1 = xw[1];
          if (BITS == 4) {
            const uint32_t p = b0, r = b1;
            asm("prmt.b32 %0, %1, %2, 0x5410;" : "=r"(b0) : "r"(p), "r"(r));
            asm("prmt.b32 %0, %1, %2, 0x7632;" : "=r"(b1) : "r"(p), "r"(r));
          }
          mma16816(acc[j][e & 1], a0, a1, a2, a3, b0, b1);
        }
      }
    }
  };

  for (int grp = 0; grp < GS_GROUPS; grp++) {
    const int s0 = grp == 0 ? 0 : gend(grp - 1), s1 = gend(grp);
    if (s1 <= s0) continue;
    if (!mbar_wait(bar0 + 8 * grp, 0, abort, err, DC_DEVERR_GEMM_WAIT)) break;  // (the sums are then garbage)
    for (int s = s0 + warp; s < s1; s += GS_WARPS) compute(s);
  }
  __syncthreads();  // every warp done with the codes: the buffer takes the partial sums

#pragma unroll
  for (int j = 0; j < NT; j++) {
    const int tk = j * 8 + 2 * t;
    red[(warp * TOK + tk) * GV_ROWS + g] = acc[j][0][0] + acc[j][1][0];
    red[(warp * TOK + tk + 1) * GV_ROWS + g] = acc[j][0][1] + acc[j][1][1];
    red[(warp * TOK + tk) * GV_ROWS + g + 8] = acc[j][0][2] + acc[j][1][2];
    red[(warp * TOK + tk + 1) * GV_ROWS + g + 8] = acc[j][0][3] + acc[j][1][3];
  }
  __syncthreads();
  const int parts = gridDim.y;
  for (int i = threadIdx.x; i < TOK * GV_ROWS; i += GS_THREADS) {
    const int m = i / GV_ROWS, r = i % GV_ROWS;
    float v = 0.f;
#pragma unroll
    for (int w = 0; w < GS_WARPS; w++) v += red[(w * TOK + m) * GV_ROWS + r];
    if (parts == 1) {
      if (m < M && n0 + r < N) Y[(size_t)m * N + n0 + r] = __float2half_rn(v);
    } else {
      part[i] = v;
    }
  }
  if (parts == 1) return;
  // K parts: the cluster adds its partials in part order; CTA `rank` finishes every parts-th output
  cluster_sync();
  const uint32_t rank = cluster_rank();
  for (int i = threadIdx.x; i < TOK * GV_ROWS; i += GS_THREADS) {
    const int m = i / GV_ROWS, r = i % GV_ROWS;
    if (m < M && n0 + r < N && (uint32_t)(i % parts) == rank) {
      float sum = 0.f;
      for (int q = 0; q < parts; q++) sum += ld_dsmem(&part[i], (uint32_t)q);
      Y[(size_t)m * N + n0 + r] = __float2half_rn(sum);
    }
  }
  cluster_sync();  // no CTA leaves while a peer still reads its partial
}

template <int BITS, int NT, bool EVEN>
int launch_gemv_staged(dc_ctx *ctx, const void *X, const void *Wq, const void *S, void *Y, int M, int N, int K,
                       int parts) {
  constexpr int CODES = GvStep<BITS>::CODES;
  const int nrb = (N + GV_ROWS - 1) / GV_ROWS;
  const int nk = (K + CODES - 1) / CODES;
  if (parts <= 0) {
    // one part per row block while the row blocks cover the SMs twice (a cluster's reduction costs more than a
    // deeper part); fewer row blocks split K, at most into the cluster limit, down to 16 steps per part
    const int sms = ctx->sms > 0 ? ctx->sms : 148;
    parts = 1;
    while (parts < GV_MAX_PARTS && nrb * parts < 2 * sms && nk >= 2 * parts * 16) parts *= 2;
  }
  if (parts > GV_MAX_PARTS) parts = GV_MAX_PARTS;
  if (parts > nk) parts = nk;
  if (parts < 1) parts = 1;
  const int per = (nk + parts - 1) / parts;
  parts = (nk + per - 1) / per;
  const int kc = per * CODES;
  const int smem = gs_smem<NT>(kc, BITS);
  if (smem > 227 * 1024) return -1;  // (the register form takes it)
  auto kern = qgemv_staged_kernel<BITS, NT, EVEN>;
  if (smem > 48 * 1024) DC_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)nrb, (unsigned)parts, 1);
  cfg.blockDim = dim3(GS_THREADS, 1, 1);
  cfg.dynamicSmemBytes = (size_t)smem;
  cfg.stream = ctx->stream;
  cudaLaunchAttribute attr[2];
  int na = 0;
  attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[na].val.programmaticStreamSerializationAllowed = 1;
  na++;
  if (parts > 1) {
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = 1;
    attr[na].val.clusterDim.y = (unsigned)parts;
    attr[na].val.clusterDim.z = 1;
    na++;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  DC_CUDA(cudaLaunchKernelEx(&cfg, kern, static_cast<const __half *>(X), static_cast<const uint8_t *>(Wq),
                             static_cast<const __half *>(S), static_cast<__half *>(Y), M, N, K, kc,
                             ctx->static_weights ? 1 : 0, ctx->d_err));
  return dc_launch_check("qmatmul (decode, staged)");
}

template <int BITS, int NT>
int gemv_staged(dc_ctx *ctx, const void *X, const void *Wq, const void *S, void *Y, int M, int N, int K, int parts) {
  if (K % GvStep<BITS>::CODES == 0) return launch_gemv_staged<BITS, NT, true>(ctx, X, Wq, S, Y, M, N, K, parts);
  return launch_gemv_staged<BITS, NT, false>(ctx, X, Wq, S, Y, M, N, K, parts);
}

// ------------------------------------------------------------------ even form (K a multiple of the step)
// The register stream with nothing conditional on the weight path: when every K part is a whole number of steps,
// each lane's code, scale and token addresses advance by constants, rows beyond N repeat the last row and token rows
// beyond M repeat the last token (their MMA rows and columns are computed and never written: rows and columns of an
// MMA are independent), so every load is issued unpredicated and no branch sits between a load and its use. Only the
// warp-uniform step count decides whether a step (and the load one step ahead) exists. Tokens are read as 16-byte
// vectors through L1 (the CTAs of an SM share them), two (q8) or four (q4) per step and token tile; for q4 the
// nibbles are dequantised in the pairs {c_i, c_i+4} of a word (deq_q4_spread) and the token vectors permuted to match.
template <int BITS, int NT, bool DENSE>
__global__ void __launch_bounds__(GV_THREADS, DENSE ? (NT <= 2 ? 4 : 3) : (NT == 1 ? 4 : 2))
    qgemv_even_kernel(const __half *__restrict__ X, const uint8_t *__restrict__ W, const __half *__restrict__ S,
                      __half *__restrict__ Y, int M, int N, int K, int kc, int w_early) {
  constexpr int TOK = NT * 8;
  using G = GvStep<BITS>;
  constexpr int WB = GV_WARPS * G::CODES * BITS / 8;  // code bytes from one of a warp's steps to its next
  constexpr int WS = GV_WARPS * G::CODES / 32;        // scales from step to step
  constexpr int WX = GV_WARPS * G::CODES;             // tokens from step to step
  __shared__ float red[GV_WARPS][TOK][GV_ROWS];
  __shared__ float part[TOK][GV_ROWS];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int n0 = blockIdx.x * GV_ROWS;
  const int k0 = blockIdx.y * kc, k1 = min(K, k0 + kc);
  const int nsteps = (k1 - k0) / G::CODES;
  const int js = nsteps > warp ? (nsteps - warp + GV_WARPS - 1) / GV_WARPS : 0;  // this warp's steps

  const int r0 = min(n0 + g, N - 1), r1 = min(n0 + g + 8, N - 1);
  const int kl = k0 + warp * G::CODES + G::PER_LANE * t;  // the lane's first code of the warp's first step
  const uint8_t *pa = W + (size_t)r0 * ((size_t)K * BITS / 8) + (size_t)kl * BITS / 8;
  const uint8_t *pb = W + (size_t)r1 * ((size_t)K * BITS / 8) + (size_t)kl * BITS / 8;
  const unsigned short *sa = reinterpret_cast<const unsigned short *>(S) + (size_t)r0 * (K / 32) + kl / 32;
  const unsigned short *sb = reinterpret_cast<const unsigned short *>(S) + (size_t)r1 * (K / 32) + kl / 32;
  // the lane's token rows: one pointer per tile up to 4 tiles; with 8, a base and per-tile row offsets
  constexpr int NP = NT <= 4 ? NT : 1;
  const __half *xp[NP];
  int xo[NT];
#pragma unroll
  for (int j = 0; j < NT; j++) xo[j] = (NT <= 4 ? 0 : min(j * 8 + g, M - 1) * K);
#pragma unroll
  for (int j = 0; j < NP; j++) xp[j] = X + (NT <= 4 ? (size_t)min(j * 8 + g, M - 1) * K : 0) + kl;

  auto load = [&](Step &b) {
    b.c[0] = ld_stream(pa);
    b.c[1] = ld_stream(pb);
    b.s = (uint32_t)__ldg(sa) | ((uint32_t)__ldg(sb) << 16);
    pa += WB, pb += WB, sa += WS, sb += WS;
  };
  float acc[NT][4];
#pragma unroll
  for (int j = 0; j < NT; j++) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
  // the lane's 16 tokens of MMA group h of tile j as 8 B-operand words (q4: permuted to the nibble pairs)
  auto tokens = [&](const __half *p, uint32_t (&w)[8]) {
    const uint4 u0 = __ldg(reinterpret_cast<const uint4 *>(p));
    const uint4 u1 = __ldg(reinterpret_cast<const uint4 *>(p + 8));
    if (BITS == 8) {
      w[0] = u0.x, w[1] = u0.y, w[2] = u0.z, w[3] = u0.w, w[4] = u1.x, w[5] = u1.y, w[6] = u1.z, w[7] = u1.w;
    } else {  // per 8 tokens [x0 .. x7] -> {x0 x4} {x1 x5} {x2 x6} {x3 x7}
      asm("prmt.b32 %0, %1, %2, 0x5410;" : "=r"(w[0]) : "r"(u0.x), "r"(u0.z));
      asm("prmt.b32 %0, %1, %2, 0x7632;" : "=r"(w[1]) : "r"(u0.x), "r"(u0.z));
      asm("prmt.b32 %0, %1, %2, 0x5410;" : "=r"(w[2]) : "r"(u0.y), "r"(u0.w));
      asm("prmt.b32 %0, %1, %2, 0x7632;" : "=r"(w[3]) : "r"(u0.y), "r"(u0.w));
      asm("prmt.b32 %0, %1, %2, 0x5410;" : "=r"(w[4]) : "r"(u1.x), "r"(u1.z));
      asm("prmt.b32 %0, %1, %2, 0x7632;" : "=r"(w[5]) : "r"(u1.x), "r"(u1.z));
      asm("prmt.b32 %0, %1, %2, 0x5410;" : "=r"(w[6]) : "r"(u1.y), "r"(u1.w));
      asm("prmt.b32 %0, %1, %2, 0x7632;" : "=r"(w[7]) : "r"(u1.y), "r"(u1.w));
    }
  };
  // A fragments of MMA q (4 codes of rows g and g + 8 from the lane's vectors)
  auto afrag = [&](const Step &b, __half2 sg, __half2 sh, int q, uint32_t (&pg)[4], uint32_t (&ph)[4],
                   uint32_t (&a)[4]) {
    if (BITS == 8) {
      __half2 g01, g23, h01, h23;
      deq_q8_word((&b.c[0].x)[q], sg, g01, g23);
      deq_q8_word((&b.c[1].x)[q], sh, h01, h23);
      a[0] = h2u(g01), a[1] = h2u(h01), a[2] = h2u(g23), a[3] = h2u(h23);
    } else {
      if ((q & 1) == 0) {
        deq_q4_spread((&b.c[0].x)[q >> 1], sg, pg);
        deq_q4_spread((&b.c[1].x)[q >> 1], sh, ph);
      }
      a[0] = pg[2 * (q & 1)], a[1] = ph[2 * (q & 1)], a[2] = pg[2 * (q & 1) + 1], a[3] = ph[2 * (q & 1) + 1];
    }
  };
  auto compute = [&](const Step &b) {
    uint32_t sg2, sh2;
    asm("prmt.b32 %0, %1, 0, 0x1010;" : "=r"(sg2) : "r"(b.s));
    asm("prmt.b32 %0, %1, 0, 0x3232;" : "=r"(sh2) : "r"(b.s));
    const __half2 sg = *reinterpret_cast<__half2 *>(&sg2), sh = *reinterpret_cast<__half2 *>(&sh2);
#pragma unroll
    for (int h = 0; h < G::MMAS / 4; h++) {
      uint32_t pg[4], ph[4];
      if (NT <= 4) {
        // every tile's tokens of the group first, then the 4 MMAs, each over all tiles
        uint32_t xw[NP][8];
#pragma unroll
        for (int j = 0; j < NP; j++) tokens(xp[j] + 16 * h, xw[j]);
#pragma unroll
        for (int e = 0; e < 4; e++) {
          uint32_t a[4];
          afrag(b, sg, sh, 4 * h + e, pg, ph, a);
#pragma unroll
          for (int j = 0; j < NP; j++) mma16816(acc[j], a[0], a[1], a[2], a[3], xw[j][2 * e], xw[j][2 * e + 1]);
        }
      } else {
        // the group's 4 A fragments first, then tile by tile (the tokens of one tile live at a time)
        uint32_t a[4][4];
#pragma unroll
        for (int e = 0; e < 4; e++) afrag(b, sg, sh, 4 * h + e, pg, ph, a[e]);
#pragma unroll
        for (int j = 0; j < NT; j++) {
          uint32_t xw[8];
          tokens(xp[0] + xo[j] + 16 * h, xw);
#pragma unroll
          for (int e = 0; e < 4; e++) mma16816(acc[j], a[e][0], a[e][1], a[e][2], a[e][3], xw[2 * e], xw[2 * e + 1]);
        }
      }
    }
#pragma unroll
    for (int j = 0; j < NP; j++) xp[j] += WX;
  };

  asm volatile("griddepcontrol.launch_dependents;");
  Step ba, bb;
  if (!w_early) asm volatile("griddepcontrol.wait;" ::: "memory");
  if (js > 0) load(ba);
  if (w_early) asm volatile("griddepcontrol.wait;" ::: "memory");  // X (and Y) only after the kernel before
  for (int j = 0; j < js; j += 2) {
    if (j + 1 < js) load(bb);
    compute(ba);
    if (j + 1 >= js) break;
    if (j + 2 < js) load(ba);
    compute(bb);
  }

#pragma unroll
  for (int j = 0; j < NT; j++) {
    const int tk = j * 8 + 2 * t;
    red[warp][tk][g] = acc[j][0];
    red[warp][tk + 1][g] = acc[j][1];
    red[warp][tk][g + 8] = acc[j][2];
    red[warp][tk + 1][g + 8] = acc[j][3];
  }
  __syncthreads();
  const int parts = gridDim.y;
  for (int i = threadIdx.x; i < TOK * GV_ROWS; i += GV_THREADS) {  // (more outputs than threads beyond 16 tokens)
    const int m = i / GV_ROWS, r = i % GV_ROWS;
    float v = 0.f;
#pragma unroll
    for (int w = 0; w < GV_WARPS; w++) v += red[w][m][r];
    if (parts == 1) {
      if (m < M && n0 + r < N) Y[(size_t)m * N + n0 + r] = __float2half_rn(v);
    } else {
      part[m][r] = v;
    }
  }
  if (parts == 1) return;
  // K parts: the cluster adds its partials in part order; CTA `rank` finishes every parts-th output
  cluster_sync();
  const uint32_t rank = cluster_rank();
  for (int i = threadIdx.x; i < TOK * GV_ROWS; i += GV_THREADS) {
    const int m = i / GV_ROWS, r = i % GV_ROWS;
    if (m < M && n0 + r < N && (uint32_t)(i % parts) == rank) {
      float sum = 0.f;
      for (int q = 0; q < parts; q++) sum += ld_dsmem(&part[m][r], (uint32_t)q);
      Y[(size_t)m * N + n0 + r] = __float2half_rn(sum);
    }
  }
  cluster_sync();  // no CTA leaves while a peer still reads its partial
}

// resident CTAs per SM of a decode kernel (256 threads, static shared memory only), looked up once per kernel; a
// failed lookup (e.g. one refused during a stream capture) is not kept, its error is cleared, and the caller
// takes the uncapped build meanwhile (0)
template <typename Kern>
int gemv_occupancy(Kern kern, std::atomic<int> &cache) {
  int n = cache.load(std::memory_order_relaxed);
  if (n > 0) return n;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kern, GV_THREADS, 0) != cudaSuccess || n <= 0) {
    cudaGetLastError();
    return 0;
  }
  cache.store(n, std::memory_order_relaxed);
  return n;
}

template <int BITS, int NT>
int launch_gemv(dc_ctx *ctx, const void *X, const void *Wq, const void *S, void *Y, int M, int N, int K, int parts) {
  const int nrb = (N + GV_ROWS - 1) / GV_ROWS;
  const int nk = (K + GvStep<BITS>::CODES - 1) / GvStep<BITS>::CODES;
  const int sms = ctx->sms > 0 ? ctx->sms : 148;
  if (parts <= 0) {
    // resident CTAs: four per SM with one token tile, two with two. K is split (2 or 4 parts, a cluster each)
    // only while the row blocks fill at most half (a quarter) of those slots and every part keeps >= 12 steps:
    // the cluster reduction costs more than it gains otherwise (measured: 1024 x 3072 q8 gains 17-28% from 4
    // parts, 1280 x 768 loses 16% from 2).
    const int slots = (NT == 1 ? 4 : 2) * sms;
    parts = 1;
    while (parts < 4 && nrb * parts * 2 <= slots && nk >= parts * 2 * 12) parts *= 2;
  }
  if (parts > GV_MAX_PARTS) parts = GV_MAX_PARTS;
  if (parts > nk) parts = nk;
  if (parts < 1) parts = 1;
  const int per = (nk + parts - 1) / parts;  // steps per part
  parts = (nk + per - 1) / per;              // every part owns at least one step
  const int kc = per * GvStep<BITS>::CODES;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)nrb, (unsigned)parts, 1);
  cfg.blockDim = dim3(GV_THREADS, 1, 1);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = ctx->stream;
  cudaLaunchAttribute attr[2];
  int na = 0;
  attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;  // may overlap the kernel before (see above)
  attr[na].val.programmaticStreamSerializationAllowed = 1;
  na++;
  if (parts > 1) {  // K parts form a cluster
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = 1;
    attr[na].val.clusterDim.y = (unsigned)parts;
    attr[na].val.clusterDim.z = 1;
    na++;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  // K a whole number of steps: the form without conditional loads
  auto kern = qgemv_kernel<BITS, NT>;
  if (K % GvStep<BITS>::CODES == 0) {
    kern = qgemv_even_kernel<BITS, NT, false>;
    if constexpr (NT == 2 || NT == 4) {
      // the register-capped build of the same kernel (four or three CTAs per SM instead of two or three; a little
      // slower per CTA) where that alone brings the grid into one wave
      static std::atomic<int> cache[2];
      const int occ0 = gemv_occupancy(qgemv_even_kernel<BITS, NT, false>, cache[0]);
      const int occ1 = gemv_occupancy(qgemv_even_kernel<BITS, NT, true>, cache[1]);
      const long grid = (long)nrb * parts;
      if (occ0 > 0 && grid > (long)occ0 * sms && grid <= (long)occ1 * sms) kern = qgemv_even_kernel<BITS, NT, true>;
    }
  }
  DC_CUDA(cudaLaunchKernelEx(&cfg, kern, static_cast<const __half *>(X),
                             static_cast<const uint8_t *>(Wq), static_cast<const __half *>(S),
                             static_cast<__half *>(Y), M, N, K, kc, ctx->static_weights ? 1 : 0));
  return dc_launch_check("qmatmul (decode)");
}

}  // namespace

int gemv_launch(dc_ctx *ctx, const void *X, const void *Wq, const void *S, void *Y, int M, int N, int K, int bits,
                int parts) {
  if (M > 64) return dc_fail(DC_EINVAL, "decision.js: qmatmul: the decode form takes M <= 64 (got %d)", M);
  if (M > 16) {  // 17-64 tokens: the register stream with 4 or 8 token tiles (small weights, qgemm_pick_form)
    if (bits == 8)
      return M <= 32 ? launch_gemv<8, 4>(ctx, X, Wq, S, Y, M, N, K, parts) : launch_gemv<8, 8>(ctx, X, Wq, S, Y, M, N, K, parts);
    return M <= 32 ? launch_gemv<4, 4>(ctx, X, Wq, S, Y, M, N, K, parts) : launch_gemv<4, 8>(ctx, X, Wq, S, Y, M, N, K, parts);
  }
  // the staged form where the sweep of the decode shapes measured it faster than the register stream at 9-16
  // tokens: q8 weights of 16M codes or more in at most three row blocks per SM, and q4 weights of 8M codes or more
  // in more than two and at most three (more row blocks go to the register form's four-CTA-per-SM build, which
  // holds up to four per SM in one wave)
  const long nk = (long)N * K;
  const int sms = ctx->sms > 0 ? ctx->sms : 148;
  const int nrb = (N + GV_ROWS - 1) / GV_ROWS;
  const bool staged = M > 8 && nrb <= 3 * sms && (bits == 8 ? nk >= (16L << 20) : nk >= (8L << 20) && nrb > 2 * sms);
  if (staged) {
    const int rc = bits == 8 ? gemv_staged<8, 2>(ctx, X, Wq, S, Y, M, N, K, parts)
                             : gemv_staged<4, 2>(ctx, X, Wq, S, Y, M, N, K, parts);
    if (rc != -1) return rc;  // -1: a K part too long for shared memory
  }
  if (bits == 8)
    return M <= 8 ? launch_gemv<8, 1>(ctx, X, Wq, S, Y, M, N, K, parts) : launch_gemv<8, 2>(ctx, X, Wq, S, Y, M, N, K, parts);
  return M <= 8 ? launch_gemv<4, 1>(ctx, X, Wq, S, Y, M, N, K, parts) : launch_gemv<4, 2>(ctx, X, Wq, S, Y, M, N, K, parts);
}
