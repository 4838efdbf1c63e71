// The decode-shape quantized matmul (M <= 16 tokens): Y[M,N] = X[M,K] . deq(W)[N,K]^T with the semantics of
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
      uint2 xf[NT][4];
#pragma unroll
      for (int e = 0; e < 4; e++) {
        const int xo = 4 * (4 * h + e);
#pragma unroll
        for (int j = 0; j < NT; j++)
          xf[j][e] = (xv[j] && kb + xo < K) ? __ldg(reinterpret_cast<const uint2 *>(xr[j] + kb + xo))
                                            : make_uint2(0, 0);
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
          uint32_t b0 = xf[j][e].x, b1 = xf[j][e].y;
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
  const int i = threadIdx.x, m = i / GV_ROWS, r = i % GV_ROWS;
  float v = 0.f;
  if (i < TOK * GV_ROWS) {
#pragma unroll
    for (int w = 0; w < GV_WARPS; w++) v += red[w][m][r];
  }
  if (parts == 1) {
    if (i < TOK * GV_ROWS && m < M && n0 + r < N) Y[(size_t)m * N + n0 + r] = __float2half_rn(v);
    return;
  }
  // K parts: the cluster adds its partials in part order; CTA `rank` finishes every parts-th output
  if (i < TOK * GV_ROWS) part[m][r] = v;
  cluster_sync();
  const uint32_t rank = cluster_rank();
  if (i < TOK * GV_ROWS && m < M && n0 + r < N && (uint32_t)(i % parts) == rank) {
    float sum = 0.f;
    for (int q = 0; q < parts; q++) sum += ld_dsmem(&part[m][r], (uint32_t)q);
    Y[(size_t)m * N + n0 + r] = __float2half_rn(sum);
  }
  cluster_sync();  // no CTA leaves while a peer still reads its partial
}

template <int BITS, int NT>
int launch_gemv(dc_ctx *ctx, const void *X, const void *Wq, const void *S, void *Y, int M, int N, int K, int parts) {
  const int nrb = (N + GV_ROWS - 1) / GV_ROWS;
  const int nk = (K + GvStep<BITS>::CODES - 1) / GvStep<BITS>::CODES;
  const int sms = ctx->sms > 0 ? ctx->sms : 148;
  if (parts <= 0) {
    // resident CTAs: four per SM with one token tile, two with two. K is split (2 or 4 parts, a cluster each)
    // only while the row blocks fill at most half (a quarter) of those slots and every warp keeps >= 2 steps
    // per part: the cluster reduction costs more than it gains otherwise.
    const int slots = (NT == 1 ? 4 : 2) * sms;
    parts = 1;
    while (parts < 4 && nrb * parts * 2 <= slots && nk >= parts * 2 * 2 * GV_WARPS) parts *= 2;
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
  DC_CUDA(cudaLaunchKernelEx(&cfg, qgemv_kernel<BITS, NT>, static_cast<const __half *>(X),
                             static_cast<const uint8_t *>(Wq), static_cast<const __half *>(S),
                             static_cast<__half *>(Y), M, N, K, kc, ctx->static_weights ? 1 : 0));
  return dc_launch_check("qmatmul (decode)");
}

}  // namespace

int gemv_launch(dc_ctx *ctx, const void *X, const void *Wq, const void *S, void *Y, int M, int N, int K, int bits,
                int parts) {
  if (M > 16) return dc_fail(DC_EINVAL, "decision.js: qmatmul: the decode form takes M <= 16 (got %d)", M);
  if (bits == 8)
    return M <= 8 ? launch_gemv<8, 1>(ctx, X, Wq, S, Y, M, N, K, parts) : launch_gemv<8, 2>(ctx, X, Wq, S, Y, M, N, K, parts);
  return M <= 8 ? launch_gemv<4, 1>(ctx, X, Wq, S, Y, M, N, K, parts) : launch_gemv<4, 2>(ctx, X, Wq, S, Y, M, N, K, parts);
}
