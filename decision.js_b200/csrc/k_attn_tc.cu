// Attention on the 5th-generation tensor cores (src/eg2-kernels.ts:104-163 `attention`, src/kernels.ts:117-147
// `ATTENTION`): query token t reads the keys of [lo0, hi0) union [lo1, hi1) (sequence, causal prefix, window, or a
// tree branch's trunk plus its own branch). GQA: query head h reads kv head h / (heads / kv).
//
// One CTA takes 128 consecutive query tokens of one head and walks the union of their key ranges in blocks of
// KB = 64 keys:
//   warp 8  TMA: the Q tile once, then K blocks (lane 0) and V blocks (lane 1) into two-stage rings of their own,
//           each freed as soon as its MMA has read it (128-byte swizzle, straight from the packed
//           q|k|v rows);
//   warp 9  MMA (and TMEM owner): S_j = Q K_j^T (both operands in shared memory) into one of two S buffers in
//           TMEM; then O += P_j V_j with P_j read from TMEM as the A operand and V_j as an MN-major B operand;
//   warps 0-7  softmax, two warps per TMEM lane quadrant (thread = query row), one per half of the block: the
//           half's scores read once into registers, a 32-bit visibility mask per row (no branches), scale into
//           the exp2 domain, partial row max exchanged with the partner warp, P = exp2(s - m) written back over
//           S_j as f16, row sums in f32. O is rescaled (each warp its half of the columns) only when the row max
//           grows by more than 8 (a factor 256), so P stays in f16 range and most blocks skip the rescale; at the
//           end the partners add their row sums and stage the normalised tile in shared memory (the Q tile's
//           layout), which one thread writes out with TMA stores.
// TMEM columns: S_0 | S_1 (KB each) | O (D); two CTAs per SM at D = 64 and 128. Every wait is bounded (an expired
// wait sets the device error word).
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <float.h>

#include "dc_internal.h"
#include "dc_ptx.cuh"

using namespace dcx;

namespace {

constexpr int AT_SOFT_WARPS = 8;                 // two per TMEM lane quadrant, one per half of a key block
constexpr int AT_WARP_TMA = AT_SOFT_WARPS;
constexpr int AT_WARP_MMA = AT_SOFT_WARPS + 1;
constexpr int AT_THREADS = (AT_SOFT_WARPS + 2) * 32;

template <int D>
struct ACfg {
  static constexpr int KB = 64;                     // keys per block
  static constexpr int NA = D / 64;                 // 64-wide swizzle atoms along D
  static constexpr int Q_BYTES = 128 * D * 2;
  static constexpr int KV_BYTES = KB * D * 2;       // one of K or V per stage
  static constexpr int Q_OFF = 0;
  static constexpr int K_OFF = Q_BYTES;             // K stage s at K_OFF + s * 2 * KV_BYTES, V right after it
  static constexpr int BAR_OFF = K_OFF + 4 * KV_BYTES;
  // q, kfull[2], kempty[2], sfull[2], pfull[2], oready, odone, pair exchange[4], vfull[2], vempty[2]
  static constexpr int NBARS = 1 + 2 + 2 + 2 + 2 + 1 + 1 + 4 + 2 + 2;
  static constexpr int MISC_OFF = BAR_OFF + NBARS * 8;
  static constexpr int XCH_OFF = MISC_OFF + 32;  // float [2 parity][2 halves][128 rows]: partial row maxima / sums
  static constexpr int SMEM = XCH_OFF + 2 * 2 * 128 * 4 + 1024;
  static constexpr int S_COL = 0, O_COL = 2 * KB;
  // D = 128: 256 columns and about 97 KB of shared memory, so two CTAs share an SM and one's loads, softmax and
  // epilogue overlap the other's MMAs (the key loops of short sequences are only a few blocks long)
  static constexpr int TCOLS = O_COL + D <= 256 ? 256 : 512;
  static constexpr int CTAS_PER_SM = TCOLS == 256 ? 2 : 1;
  static_assert(O_COL + D <= TCOLS, "tensor memory");
  static_assert(KB <= 64, "one 64-bit visibility mask per row and block");
  static_assert(SMEM * CTAS_PER_SM <= 227 * 1024, "shared memory");
};

// Shared-memory descriptor of an MN-major operand stored as TMA writes a {64, rows} box with 128-byte swizzling:
// 8-row (K) groups 1024 bytes apart, 64-element MN chunks `lbo` bytes apart (one box after the other).
__device__ __forceinline__ uint64_t desc_sw128_mn(uint32_t saddr, uint32_t lbo) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr & 0x3FFFFu) >> 4);
  d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)(1024 >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

__device__ __forceinline__ int4 clamp_rng(int4 r, int T) {
  r.x = min(max(r.x, 0), T), r.y = min(max(r.y, 0), T);
  r.z = min(max(r.z, 0), T), r.w = min(max(r.w, 0), T);
  return r;
}

// bar.red.and over the 8 softmax warps (barrier 1, 256 threads): every softmax thread passes, returns whether all of
// them passed `pred`
__device__ __forceinline__ int __syncthreads_and_softmax(bool pred) {
  uint32_t r;
  asm volatile("{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n bar.red.and.pred q, 1, %2, p;\n selp.u32 %0, 1, 0, q;\n}\n"
               : "=r"(r)
               : "r"((uint32_t)pred), "n"(AT_SOFT_WARPS * 32)
               : "memory");
  return (int)r;
}

struct AArgs {
  const int4 *rng;
  __half *Y;
  const __half *Z;  // the rows, for the output gates
  uint32_t *err;
  long zstride;     // elements per token row of Z
  int T, heads, kv;
  int gate;         // 1: Y = attention * sigmoid(gate), the gate heads after the v heads (d3-lite)
  float scale_log2;
};

template <int D>
__global__ void __launch_bounds__(AT_THREADS, ACfg<D>::CTAS_PER_SM)
    attention_tc(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmKV,
                 const __grid_constant__ CUtensorMap tmY, AArgs a) {
  dc_pdl_launch_dependents();
  using C = ACfg<D>;
  constexpr int KB = C::KB;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bars = sbase + C::BAR_OFF;
  const uint32_t QF = bars;
  // K and V have rings of their own: a K stage is free once Q K^T of its block is done, a V stage once P V of
  // its block is, so the next K blocks load while P V still runs
  auto KF = [&](int s) { return bars + 8u * (1 + s); };
  auto KE = [&](int s) { return bars + 8u * (3 + s); };
  auto VF = [&](int s) { return bars + 8u * (15 + s); };
  auto VE = [&](int s) { return bars + 8u * (17 + s); };
  auto SF = [&](int b) { return bars + 8u * (5 + b); };
  auto PF = [&](int b) { return bars + 8u * (7 + b); };
  const uint32_t OR = bars + 8u * 9;   // one phase per P.V block (waited on only while at most one is pending)
  const uint32_t OD = bars + 8u * 10;  // one phase: every P.V block done (the epilogue's wait)
  auto XB = [&](int q) { return bars + 8u * (11 + q); };  // the two softmax warps of lane quadrant q meet
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + C::MISC_OFF);
  volatile int *abort = reinterpret_cast<volatile int *>(smem + C::MISC_OFF + 4);
  int *s_kmin = reinterpret_cast<int *>(smem + C::MISC_OFF + 8);
  int *s_kmax = reinterpret_cast<int *>(smem + C::MISC_OFF + 12);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // query tiles in reverse order: in causal passes the later tiles of a sequence walk the most key blocks, so the
  // longest CTAs start first and the launch ends on short ones
  const int h = blockIdx.y, t0 = (gridDim.x - 1 - blockIdx.x) * 128;
  const int kvh = h / (a.heads / a.kv);

  if (threadIdx.x == 0) {
    mbar_init(QF, 1);
    for (int s = 0; s < 2; s++) {
      mbar_init(KF(s), 1);
      mbar_init(KE(s), 1);
      mbar_init(VF(s), 1);
      mbar_init(VE(s), 1);
      mbar_init(SF(s), 1);
      mbar_init(PF(s), AT_SOFT_WARPS);
    }
    mbar_init(OR, 1);
    mbar_init(OD, 1);
    for (int q = 0; q < 4; q++) mbar_init(XB(q), 2);
    *abort = 0;
    *s_kmin = 0x7fffffff;
    *s_kmax = -1;
    mbar_init_fence();
  }
  if (warp == AT_WARP_MMA) tmem_alloc(smem_u32(tmem_slot), C::TCOLS);
  if (warp == AT_WARP_TMA && lane == 0) { tma_prefetch_desc(&tmQ); tma_prefetch_desc(&tmKV); }
  dc_pdl_wait();  // the q|k|v rows and the key ranges are written by the kernels before this one
  __syncthreads();
  // the Q tile does not depend on the key ranges: its load overlaps their gathering
  if (warp == AT_WARP_TMA && lane == 0) {
    mbar_expect_tx(QF, C::Q_BYTES);
    for (int j = 0; j < C::NA; j++) tma_load_2d(sbase + C::Q_OFF + j * 128 * 128, &tmQ, h * D + 64 * j, t0, QF);
  }
  // the tile's key span: the union of its rows' ranges. Softmax thread (warp w, lane) owns row 32 (w % 4) + lane
  int4 myr = make_int4(0, 0, 0, 0);
  const int row = 32 * (warp & 3) + lane;
  const int t = t0 + row;
  if (warp < AT_SOFT_WARPS && t < a.T) {
    myr = clamp_rng(a.rng[t], a.T);
    int lo = 0x7fffffff, hi = -1;
    if (myr.y > myr.x) lo = min(lo, myr.x), hi = max(hi, myr.y);
    if (myr.w > myr.z) lo = min(lo, myr.z), hi = max(hi, myr.w);
    if (hi >= 0 && warp < 4) { atomicMin(s_kmin, lo); atomicMax(s_kmax, hi); }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int kmin = *s_kmin, kmax = *s_kmax;
  const int nblk = kmax > kmin ? (kmax - kmin + KB - 1) / KB : 0;

  if (warp == AT_WARP_TMA) {
    // no keys: nothing waits for the Q tile, so its load is waited for here (no copy outlives the CTA)
    if (lane == 0 && nblk == 0) mbar_wait(QF, 0, abort, a.err, DC_DEVERR_ATTN_WAIT);
    // lane 0 loads the K blocks, lane 1 the V blocks, each as its ring frees a stage
    if (lane < 2 && nblk > 0) {
      const bool isk = lane == 0;
      for (int jb = 0; jb < nblk; jb++) {
        const int s = jb & 1;
        if (!mbar_wait(isk ? KE(s) : VE(s), ((jb >> 1) & 1) ^ 1, abort, a.err, DC_DEVERR_ATTN_WAIT)) break;
        const uint32_t full = isk ? KF(s) : VF(s);
        mbar_expect_tx(full, C::KV_BYTES);
        const uint32_t st = sbase + C::K_OFF + s * 2 * C::KV_BYTES + (isk ? 0u : (uint32_t)C::KV_BYTES);
        const int col = (isk ? a.heads + kvh : a.heads + a.kv + kvh) * D, kc = kmin + jb * KB;
        for (int j = 0; j < C::NA; j++) tma_load_2d(st + j * KB * 128, &tmKV, col + 64 * j, kc, full);
      }
    }
  } else if (warp == AT_WARP_MMA) {
    if (lane == 0 && nblk > 0) {
      constexpr uint32_t idesc_qk = idesc_f16_f32(128, KB);
      constexpr uint32_t idesc_pv = idesc_f16_f32(128, D) | (1u << 16);  // B (V) MN-major
      bool ok = mbar_wait(QF, 0, abort, a.err, DC_DEVERR_ATTN_WAIT);
      auto pv = [&](int jb) -> bool {
        const int s = jb & 1;
        if (!mbar_wait(PF(s), (jb >> 1) & 1, abort, a.err, DC_DEVERR_ATTN_WAIT) ||
            !mbar_wait(VF(s), (jb >> 1) & 1, abort, a.err, DC_DEVERR_ATTN_WAIT))
          return false;
        tc_fence_after();
        const uint32_t vst = sbase + C::K_OFF + s * 2 * C::KV_BYTES + C::KV_BYTES;
        const uint32_t pcol = tmem + (uint32_t)(C::S_COL + s * KB);
#pragma unroll
        for (int kk = 0; kk < KB / 16; kk++)
          mma_f16_ts(tmem + C::O_COL, pcol + 8 * kk, desc_sw128_mn(vst + kk * 2048, KB * 128), idesc_pv,
                     (jb > 0 || kk > 0) ? 1u : 0u);
        mma_commit(VE(s));
        mma_commit(OR);
        return true;
      };
      for (int jb = 0; ok && jb < nblk; jb++) {
        const int s = jb & 1;
        if (!mbar_wait(KF(s), (jb >> 1) & 1, abort, a.err, DC_DEVERR_ATTN_WAIT)) { ok = false; break; }
        tc_fence_after();
        const uint32_t kst = sbase + C::K_OFF + s * 2 * C::KV_BYTES;
#pragma unroll
        for (int kd = 0; kd < D / 16; kd++) {
          const uint64_t qd = desc_sw128(sbase + C::Q_OFF + (kd >> 2) * 128 * 128 + (kd & 3) * 32);
          const uint64_t kdsc = desc_sw128(kst + (kd >> 2) * KB * 128 + (kd & 3) * 32);
          mma_f16(tmem + (uint32_t)(C::S_COL + s * KB), qd, kdsc, idesc_qk, kd > 0 ? 1u : 0u);
        }
        mma_commit(SF(s));
        mma_commit(KE(s));  // S(jb + 2) overwrites this S buffer only after P V(jb) read it: one thread issues both
        if (jb > 0 && !pv(jb - 1)) { ok = false; break; }
      }
      if (ok && pv(nblk - 1)) mma_commit(OD);
    }
  } else {
    // softmax and epilogue. Warp w handles the 32 rows of TMEM lane quadrant q = w % 4 (thread = row) and half
    // hf = w / 4 of each 64-key block (and of O's columns); the two warps of a quadrant exchange partial row
    // maxima (and, at the end, row sums) through shared memory, meeting on an mbarrier.
    const int q = warp & 3, hf = warp >> 2;
    const uint32_t lrow = (uint32_t)(32 * q) << 16;
    float *xch = reinterpret_cast<float *>(smem + C::XCH_OFF);  // [parity][half][row]
    float m_ref = -FLT_MAX, l = 0.f;
    bool ok = true;
    auto meet = [&](int phase) -> bool {  // both warps of the quadrant have written their partials
      __syncwarp();
      if (lane == 0) mbar_arrive(XB(q));
      return __all_sync(0xffffffffu, mbar_wait(XB(q), phase & 1, abort, a.err, DC_DEVERR_ATTN_WAIT));
    };
    for (int jb = 0; jb < nblk; jb++) {
      const int s = jb & 1;
      const int kc = kmin + jb * KB;
      // tcgen05.ld / st are warp-collective: every decision in front of them is made by the whole warp, and they
      // are issued from warp-converged code only
      if (!__all_sync(0xffffffffu, mbar_wait(SF(s), (jb >> 1) & 1, abort, a.err, DC_DEVERR_ATTN_WAIT))) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t scol = tmem + lrow + (uint32_t)(C::S_COL + s * KB);
      uint32_t r[32];
      __syncwarp();
      tmem_ld32(scol + 32 * hf, r);
      tmem_ld_wait(r);
      // the row's visible keys of this half block as a 32-bit mask (its two ranges clipped to it)
      const int kh = kc + 32 * hf;
      auto span = [&](int lo, int hi) -> uint32_t {
        const int a0 = min(max(lo - kh, 0), 32), b0 = min(max(hi - kh, 0), 32);
        if (b0 <= a0) return 0u;
        const uint32_t upto_b = b0 >= 32 ? ~0u : ((1u << b0) - 1u);
        const uint32_t upto_a = a0 >= 32 ? ~0u : ((1u << a0) - 1u);
        return upto_b & ~upto_a;
      };
      const uint32_t vis = span(myr.x, myr.y) | span(myr.z, myr.w);
      float m4[4] = {-FLT_MAX, -FLT_MAX, -FLT_MAX, -FLT_MAX};
#pragma unroll
      for (int e = 0; e < 32; e++) {
        const float v = __uint_as_float(r[e]) * a.scale_log2;
        r[e] = __float_as_uint(v);
        m4[e & 3] = fmaxf(m4[e & 3], ((vis >> e) & 1u) ? v : -FLT_MAX);
      }
      const float pmx = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3]));
      xch[(s * 2 + hf) * 128 + row] = pmx;
      if (!meet(jb)) { ok = false; break; }
      const float mx = fmaxf(pmx, xch[(s * 2 + (hf ^ 1)) * 128 + row]);
      // a row whose max grew past its reference by more than a factor 2^8 moves O and l to the new reference
      // (both warps of the quadrant see the same maxima, so they decide alike); the warp rescales its half of O
      // together when any of its rows needs it (factor 1 for the others)
      const bool grow = mx > m_ref + 8.0f;
      const bool resc = grow && m_ref > -FLT_MAX && jb > 0;
      if (__any_sync(0xffffffffu, resc)) {
        if (!__all_sync(0xffffffffu, mbar_wait(OR, (jb - 1) & 1, abort, a.err, DC_DEVERR_ATTN_WAIT))) {
          ok = false;
          break;
        }
        tc_fence_after();
        const float f = resc ? ex2_approx(m_ref - mx) : 1.0f;
        l *= f;
        const uint32_t ocol = tmem + lrow + (uint32_t)(C::O_COL + hf * (D / 2));
#pragma unroll 1
        for (int c = 0; c < D / 2; c += 16) {
          uint32_t o[16];
          __syncwarp();
          tmem_ld16(ocol + c, o);
          tmem_ld_wait(o);
#pragma unroll
          for (int e = 0; e < 16; e++) o[e] = __float_as_uint(__uint_as_float(o[e]) * f);
          __syncwarp();
          tmem_st16(ocol + c, o);
        }
        tmem_st_wait();
      }
      if (grow) m_ref = mx;
      // P = exp2(s - m_ref) as f16 pairs for this half: 16 words written over S columns 16 hf .. 16 hf + 15 (the
      // partner warp's scores there were read before the meeting above)
      float r4[4] = {0.f, 0.f, 0.f, 0.f};
      const uint32_t live = m_ref > -FLT_MAX ? vis : 0u;
#pragma unroll
      for (int e = 0; e < 32; e += 2) {
        const float p0 = ((live >> e) & 1u) ? ex2_approx(__uint_as_float(r[e]) - m_ref) : 0.f;
        const float p1 = ((live >> (e + 1)) & 1u) ? ex2_approx(__uint_as_float(r[e + 1]) - m_ref) : 0.f;
        const __half2 hp = __floats2half2_rn(p0, p1);
        const float2 back = __half22float2(hp);  // the row sum adds what the MMA multiplies
        r4[(e >> 1) & 3] += back.x + back.y;
        r[e / 2] = *reinterpret_cast<const uint32_t *>(&hp);
      }
      l += (r4[0] + r4[1]) + (r4[2] + r4[3]);
      __syncwarp();
      tmem_st16(scol + 16 * hf, *reinterpret_cast<const uint32_t (*)[16]>(&r[0]));
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(PF(s));
    }
    // OD, not OR: when the last block's softmax ends, the P.V of the block before may still be running, and OR's
    // parity could not tell its phase from the last one
    bool staged = false;
    if (ok && nblk > 0 && __all_sync(0xffffffffu, mbar_wait(OD, 0, abort, a.err, DC_DEVERR_ATTN_WAIT))) {
      tc_fence_after();
      xch[(2 * (nblk & 1) + hf) * 128 + row] = l;
      if (meet(nblk)) {
        const float lt = l + xch[(2 * (nblk & 1) + (hf ^ 1)) * 128 + row];
        const float inv = lt > 0.f ? 1.0f / lt : 0.f;
        const uint32_t ocol = tmem + lrow + (uint32_t)(C::O_COL + hf * (D / 2));
        const __half *grow = a.Z + (size_t)t * a.zstride + (size_t)(a.heads + 2 * a.kv) * D + (size_t)h * D;
        const bool gated = a.gate && t < a.T;
        // this half of the normalised f16 row goes to shared memory (the Q tile's space: every MMA that read Q is
        // done) in the Q tile's own layout, 64-column atoms of 128 rows x 128 bytes, 16-byte chunk c of row r at
        // c ^ (r % 8); the tile then leaves by TMA stores, one per atom
        for (int c = 0; c < D / 2; c += 32) {
          uint32_t rr[32];
          __syncwarp();
          tmem_ld32(ocol + c, rr);
          tmem_ld_wait(rr);
#pragma unroll
          for (int qq = 0; qq < 4; qq++) {
            const int ch = hf * (D / 16) + c / 8 + qq;  // 16-byte chunk of the row, 0 .. D/8 - 1
            __half2 hv[4];
            if (gated) {  // times sigmoid(gate): the gate heads follow the v heads in the row
              const uint4 gv = *reinterpret_cast<const uint4 *>(grow + 8 * ch);
              const __half2 *gh = reinterpret_cast<const __half2 *>(&gv);
#pragma unroll
              for (int e = 0; e < 4; e++) {
                const float2 f = __half22float2(gh[e]);
                hv[e] = __floats2half2_rn(__uint_as_float(rr[8 * qq + 2 * e]) * inv / (1.0f + expf(-f.x)),
                                          __uint_as_float(rr[8 * qq + 2 * e + 1]) * inv / (1.0f + expf(-f.y)));
              }
            } else {
#pragma unroll
              for (int e = 0; e < 4; e++)
                hv[e] = __floats2half2_rn(__uint_as_float(rr[8 * qq + 2 * e]) * inv,
                                          __uint_as_float(rr[8 * qq + 2 * e + 1]) * inv);
            }
            uint8_t *dst = smem + C::Q_OFF + (ch >> 3) * (128 * 128) + row * 128 + (((ch & 7) ^ (row & 7)) << 4);
            *reinterpret_cast<uint4 *>(dst) = *reinterpret_cast<uint4 *>(hv);
          }
        }
        fence_proxy_async_smem();  // the TMA stores read what these threads wrote
        staged = true;
      }
    } else if (t < a.T && nblk == 0) {
      for (int c = hf * (D / 2); c < (hf + 1) * (D / 2); c += 8)
        *reinterpret_cast<uint4 *>(a.Y + (size_t)t * a.heads * D + (size_t)h * D + c) = make_uint4(0, 0, 0, 0);
    }
    // every softmax warp passes here once, on every path; when all of them staged their rows, one thread stores
    // the tile (rows past T are clipped by the TMA) and waits until the stores have read the shared memory
    const int all_staged = __syncthreads_and_softmax(staged);
    if (warp == 0 && lane == 0 && all_staged) {
      for (int j = 0; j < C::NA; j++) tma_store_2d(&tmY, h * D + 64 * j, t0, sbase + C::Q_OFF + j * 128 * 128);
      bulk_commit();
      bulk_store_read_wait();
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == AT_WARP_MMA) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TCOLS);
  }
}

typedef CUresult (*EncodeTiledA)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                 const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

int z_map(CUtensorMap *m, const void *Z, int W, int T, int rows) {
  static EncodeTiledA enc = nullptr;
  if (!enc) {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      enc = reinterpret_cast<EncodeTiledA>(p);
  }
  DC_CHECK(enc, DC_ECUDA, "decision.js: cuTensorMapEncodeTiled is unavailable");
  cuuint64_t dims[2] = {(cuuint64_t)W, (cuuint64_t)T};
  cuuint64_t strides[1] = {(cuuint64_t)W * 2};
  cuuint32_t box[2] = {64, (cuuint32_t)rows};
  cuuint32_t es[2] = {1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void *>(Z), dims, strides, box, es,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  DC_CHECK(r == CUDA_SUCCESS, DC_ECUDA, "decision.js: attention tensor map encode failed (%d)", (int)r);
  return DC_OK;
}

template <int D>
int launch(dc_ctx *ctx, const void *Z, const int *rng, void *Y, int T, int heads, int kv, float scale, long zstride,
           int gate) {
  using C = ACfg<D>;
  CUtensorMap tq, tkv;
  const int W = (int)zstride;
  int rc = z_map(&tq, Z, W, T, 128);
  if (rc) return rc;
  rc = z_map(&tkv, Z, W, T, C::KB);
  if (rc) return rc;
  CUtensorMap ty;  // the output rows [T, heads * D], stored 128 rows x 64 columns at a time
  rc = z_map(&ty, Y, heads * D, T, 128);
  if (rc) return rc;
  static uint64_t attr_done = 0;
  if (!(attr_done & (1ull << ctx->device))) {
    DC_CUDA(cudaFuncSetAttribute(attention_tc<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM));
    attr_done |= 1ull << ctx->device;
  }
  AArgs a;
  a.rng = reinterpret_cast<const int4 *>(rng);
  a.Y = static_cast<__half *>(Y);
  a.Z = static_cast<const __half *>(Z);
  a.err = ctx->d_err;
  a.zstride = zstride, a.gate = gate;
  a.T = T, a.heads = heads, a.kv = kv;
  a.scale_log2 = scale * 1.4426950408889634f;
  dim3 grid((T + 127) / 128, heads);
  DC_CUDA(dc_launch_pdl(ctx->stream, attention_tc<D>, grid, dim3(AT_THREADS), C::SMEM, tq, tkv, ty, a));
  return dc_launch_check("attention (tcgen05)");
}

}  // namespace

// The tensor-core attention for D = 64, 128 or 256 (D = 512 takes the mma.sync kernel: its O alone would fill the
// 512 TMEM columns). Z (rows of `zstride` halves: q | k | v heads, then with `gate` the output gates) and Y (rows
// of heads * D halves) must be 16-byte aligned.
int attn_tc_launch(dc_ctx *ctx, const void *Z, const int *rng, void *Y, int T, int heads, int kv, int D, float scale,
                   long zstride, int gate) {
  DC_CHECK(((uintptr_t)Z & 15) == 0 && ((uintptr_t)Y & 15) == 0 && zstride % 8 == 0, DC_EINVAL,
           "decision.js: attention: Z and Y must be 16-byte aligned, the row stride a multiple of 8");
  if (D == 256) return launch<256>(ctx, Z, rng, Y, T, heads, kv, scale, zstride, gate);
  if (D == 128) return launch<128>(ctx, Z, rng, Y, T, heads, kv, scale, zstride, gate);
  if (D == 64) return launch<64>(ctx, Z, rng, Y, T, heads, kv, scale, zstride, gate);
  return dc_fail(DC_EINVAL, "decision.js: tensor-core attention takes D = 64, 128 or 256 (got %d)", D);
}
