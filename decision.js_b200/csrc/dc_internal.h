// Internal declarations shared by the library's translation units.
#pragma once
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include <stdio.h>
#include <stdarg.h>
#include <string>
#include <vector>

#include "../../include/decision_cuda.h"

// Thread-local last error (dc_last_error). Returns `code` so call sites read `return dc_fail(DC_EINVAL, ...)`.
int dc_fail(int code, const char *fmt, ...);
int dc_ok();

#define DC_CUDA(call)                                                                                 \
  do {                                                                                                \
    cudaError_t e_ = (call);                                                                          \
    if (e_ != cudaSuccess) return dc_fail(DC_ECUDA, "decision.js: %s: %s (%s:%d)", #call,             \
                                          cudaGetErrorString(e_), __FILE__, __LINE__);                \
  } while (0)

#define DC_CHECK(cond, code, ...)                                                                     \
  do {                                                                                                \
    if (!(cond)) return dc_fail(code, __VA_ARGS__);                                                   \
  } while (0)

// Programmatic dependent launch. Kernels launched with dc_launch_pdl begin with dc_pdl_begin(): they let the next
// kernel of the stream launch at once (its blocks then wait in their own dc_pdl_begin) and wait for the kernel
// before them to complete before touching memory, so a kernel's launch and prologue overlap its predecessor's
// drain. Without the launch attribute both instructions are no-ops.
__device__ __forceinline__ void dc_pdl_begin() {
  asm volatile("griddepcontrol.launch_dependents;");
  asm volatile("griddepcontrol.wait;" ::: "memory");
}
// The two halves, for kernels whose setup (barriers, tensor memory) touches no global memory and can run before
// the predecessor completes.
__device__ __forceinline__ void dc_pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;"); }
__device__ __forceinline__ void dc_pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// GELU with erf by Abramowitz & Stegun 7.1.26 (|error of erf| < 1.5e-7), as the reference writes it in
// src/kernels.ts:202-206, src/encoder-kernels.ts:31-35 and src/eg2-head.ts: 0.5 x (1 + erf(x / sqrt 2)).
__device__ __forceinline__ float dc_gelu_erf_as(float x) {
  const float z = x * 0.70710678f;
  const float t = 1.0f / (1.0f + 0.3275911f * fabsf(z));
  const float y = 1.0f - ((((1.061405429f * t - 1.453152027f) * t + 1.421413741f) * t - 0.284496736f) * t +
                          0.254829592f) * t * expf(-z * z);
  return 0.5f * x * (1.0f + (z >= 0.f ? y : -y));
}

// Launches `kernel` on ctx's stream with the programmatic-stream-serialization attribute (see dc_pdl_begin).
template <typename... KArgs, typename... Args>
cudaError_t dc_launch_pdl(cudaStream_t stream, void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                          Args &&...args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

// Device error word bits written by kernels whose bounded waits expire (read back by dc_sync).
enum {
  DC_DEVERR_GEMM_WAIT = 1,
  DC_DEVERR_ATTN_WAIT = 2,
  DC_DEVERR_TOKEN_ID = 4,
  DC_DEVERR_BOUNDS = 8,
  DC_DEVERR_WAIT_PROBE = 16,  // dc_selftest_wait's expired wait
};

struct dc_profile_slot {
  cudaEvent_t a, b;
  int kind;
  double flops, bytes;
};

struct dc_ctx {
  int device = 0;
  cudaStream_t stream = nullptr;
  int sms = 0;
  // Kernel-visible error word (device memory, one uint32) and its pinned host copy, read back on the stream before
  // dc_sync's wait so one synchronisation covers both.
  uint32_t *d_err = nullptr;
  uint32_t *h_err = nullptr;
  // Grow-only scratch for split-K partials and tile counters.
  void *scratch = nullptr;
  size_t scratch_bytes = 0;
  uint32_t *counters = nullptr;  // zero between launches
  size_t counters_n = 0;
  // Set by the model passes around their matmuls: the weights were written before the pass (and the stream
  // synchronised since), so a matmul may start reading its codes and scales before the kernel before it completes.
  bool static_weights = false;
  // Profiling.
  bool profiling = false;
  std::vector<dc_profile_slot> pending;
  std::vector<cudaEvent_t> free_events;
  double prof_ms[DC_K_KINDS] = {}, prof_flops[DC_K_KINDS] = {}, prof_bytes[DC_K_KINDS] = {};
  long long prof_n[DC_K_KINDS] = {};
};

// Make `ctx`'s device current on this thread.
int dc_use(dc_ctx *ctx);
// Scratch of at least `bytes` (grow-only; the stream is synced before a regrow) and `ncounters` zeroed words.
int dc_scratch(dc_ctx *ctx, size_t bytes, size_t ncounters, void **scratch, uint32_t **counters);
// Profiling brackets around one launch (no-ops unless profiling).
void dc_prof_begin(dc_ctx *ctx, int kind, double flops, double bytes);
void dc_prof_end(dc_ctx *ctx);
// Launch-error check after a <<<>>> launch.
int dc_launch_check(const char *what);

// EmbeddingGemma 2's decision head (src/eg2-head.ts): device pointers of its f32 tensors (the manifest's "host"
// section) and its scalars (config.head).
struct Eg2HeadW {
  const float *state_w, *state_b, *question_w, *question_b, *option_w, *option_b;
  const float *field0_w, *field0_b, *field3_w, *field3_b, *type_emb, *field_norm_w, *field_norm_b;
  const float *option_norm_w, *option_norm_b, *res0_w, *res0_b, *res3_w;
  int W, E, ntypes;
  float ln_eps, prior_scale, joint_scale, gate, residual_bias;
};

// Kernel hosts (implemented in the k_*.cu files); arguments already validated by the API layer.
int qgemm_launch(dc_ctx *ctx, const void *X, const void *Wq, const void *S, void *Y, int M, int N, int K, int bits,
                 int form, int splits);
int qgemm_pick_form(int M, int N, int K, int bits, int sms);
// Decode form (M <= 16): tensor-pipe weight stream, K split over a cluster of `parts` CTAs (<= 0 picks).
int gemv_launch(dc_ctx *ctx, const void *X, const void *Wq, const void *S, void *Y, int M, int N, int K, int bits,
                int parts);
// Y[M, N/2] = act(gate) * up over interleaved gate|up weight rows (act 1 = GELU-tanh, 2 = SiLU); N % 128 == 0.
int qgemm_launch_glu(dc_ctx *ctx, const void *X, const void *Wq, const void *S, void *Y, int M, int N, int K,
                     int bits, int act);
// the direct form: Y = X . W16^T on weights dequantized to f16 at load (act 0 plain, 1 GeGLU, 2 SwiGLU)
int qgemm_direct_launch(dc_ctx *ctx, const void *X, const void *W16, void *Y, int M, int N, int K, int act);
