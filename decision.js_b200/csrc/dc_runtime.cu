// Context, memory, errors, synchronisation and profiling: the part of the reference's device layer
// (src/gpu.ts:38-54 requestDevice, :148-174 buffers, :177-281 recorder bookkeeping) that is not a kernel.
#include <chrono>
#include <thread>
#include <string.h>

#include "dc_internal.h"

static thread_local char g_err[1024];

int dc_fail(int code, const char *fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof g_err, fmt, ap);
  va_end(ap);
  return code;
}

int dc_ok() { return DC_OK; }

extern "C" const char *dc_last_error(void) { return g_err; }

int dc_launch_check(const char *what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return dc_fail(DC_ECUDA, "decision.js: launch of %s failed: %s", what, cudaGetErrorString(e));
  return DC_OK;
}

int dc_use(dc_ctx *ctx) {
  DC_CHECK(ctx, DC_EINVAL, "decision.js: null context");
  DC_CUDA(cudaSetDevice(ctx->device));
  return DC_OK;
}

extern "C" int dc_device_count(int *out) {
  DC_CHECK(out, DC_EINVAL, "decision.js: null output");
  int n = 0;
  cudaError_t e = cudaGetDeviceCount(&n);
  if (e != cudaSuccess) n = 0;
  *out = n;
  return DC_OK;
}

extern "C" int dc_init(int device, dc_ctx **out) {
  DC_CHECK(out, DC_EINVAL, "decision.js: null output");
  *out = nullptr;
  int n = 0;
  cudaError_t e = cudaGetDeviceCount(&n);
  DC_CHECK(e == cudaSuccess && n > 0, DC_ECUDA, "decision.js: no CUDA device is available (%s)",
           cudaGetErrorString(e));
  DC_CHECK(device >= 0 && device < n, DC_EINVAL, "decision.js: device %d out of range (%d devices)", device, n);
  DC_CUDA(cudaSetDevice(device));
  cudaDeviceProp prop;
  DC_CUDA(cudaGetDeviceProperties(&prop, device));
  DC_CHECK(prop.major == 10, DC_ECUDA, "decision.js: device %d is sm_%d%d; this library is built for sm_100a",
           device, prop.major, prop.minor);
  dc_ctx *c = new dc_ctx();
  c->device = device;
  c->sms = prop.multiProcessorCount;
  if (cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking) != cudaSuccess ||
      cudaMalloc(&c->d_err, sizeof(uint32_t)) != cudaSuccess ||
      cudaHostAlloc((void **)&c->h_err, sizeof(uint32_t), cudaHostAllocDefault) != cudaSuccess ||
      cudaMemsetAsync(c->d_err, 0, sizeof(uint32_t), c->stream) != cudaSuccess) {
    cudaError_t le = cudaGetLastError();
    dc_destroy(c);
    return dc_fail(DC_ECUDA, "decision.js: context setup on device %d failed: %s", device, cudaGetErrorString(le));
  }
  *out = c;
  return DC_OK;
}

extern "C" int dc_destroy(dc_ctx *ctx) {
  if (!ctx) return DC_OK;
  cudaSetDevice(ctx->device);
  if (ctx->stream) cudaStreamSynchronize(ctx->stream);
  for (auto &p : ctx->pending) { cudaEventDestroy(p.a); cudaEventDestroy(p.b); }
  for (auto e : ctx->free_events) cudaEventDestroy(e);
  if (ctx->scratch) cudaFree(ctx->scratch);
  if (ctx->counters) cudaFree(ctx->counters);
  if (ctx->d_err) cudaFree(ctx->d_err);
  if (ctx->h_err) cudaFreeHost(ctx->h_err);
  if (ctx->stream) cudaStreamDestroy(ctx->stream);
  delete ctx;
  return DC_OK;
}

extern "C" int dc_alloc(dc_ctx *ctx, size_t bytes, void **d_out) {
  DC_CHECK(d_out, DC_EINVAL, "decision.js: null output");
  int rc = dc_use(ctx);
  if (rc) return rc;
  *d_out = nullptr;
  cudaError_t e = cudaMalloc(d_out, bytes ? bytes : 16);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return dc_fail(DC_ENOMEM, "decision.js: cannot allocate %zu bytes on device %d: %s", bytes, ctx->device,
                   cudaGetErrorString(e));
  }
  return DC_OK;
}

extern "C" int dc_free(dc_ctx *ctx, void *d_ptr) {
  int rc = dc_use(ctx);
  if (rc) return rc;
  if (d_ptr) DC_CUDA(cudaFree(d_ptr));
  return DC_OK;
}

extern "C" int dc_upload(dc_ctx *ctx, void *d_dst, const void *h_src, size_t bytes) {
  int rc = dc_use(ctx);
  if (rc) return rc;
  DC_CHECK(bytes == 0 || (d_dst && h_src), DC_EINVAL, "decision.js: null pointer in upload");
  if (!bytes) return DC_OK;
  DC_CUDA(cudaMemcpyAsync(d_dst, h_src, bytes, cudaMemcpyHostToDevice, ctx->stream));
  DC_CUDA(cudaStreamSynchronize(ctx->stream));
  return DC_OK;
}

extern "C" int dc_download(dc_ctx *ctx, void *h_dst, const void *d_src, size_t bytes) {
  int rc = dc_use(ctx);
  if (rc) return rc;
  DC_CHECK(bytes == 0 || (h_dst && d_src), DC_EINVAL, "decision.js: null pointer in download");
  if (!bytes) return DC_OK;
  DC_CUDA(cudaMemcpyAsync(h_dst, d_src, bytes, cudaMemcpyDeviceToHost, ctx->stream));
  DC_CUDA(cudaStreamSynchronize(ctx->stream));
  return DC_OK;
}

extern "C" int dc_memset(dc_ctx *ctx, void *d_dst, int value, size_t bytes) {
  int rc = dc_use(ctx);
  if (rc) return rc;
  if (bytes) DC_CUDA(cudaMemsetAsync(d_dst, value, bytes, ctx->stream));
  return DC_OK;
}

extern "C" void *dc_stream(dc_ctx *ctx) { return ctx ? (void *)ctx->stream : nullptr; }

extern "C" int dc_static_weights(dc_ctx *ctx, int on) {
  DC_CHECK(ctx, DC_EINVAL, "decision.js: static_weights: null context");
  ctx->static_weights = on != 0;
  return DC_OK;
}

// The error word as of the launches enqueued so far: its copy is enqueued here, and read after the caller's wait.
static int enqueue_error_read(dc_ctx *ctx) {
  *ctx->h_err = 0;
  DC_CUDA(cudaMemcpyAsync(ctx->h_err, ctx->d_err, sizeof(uint32_t), cudaMemcpyDeviceToHost, ctx->stream));
  return DC_OK;
}

static int check_device_error(dc_ctx *ctx) {
  const uint32_t err = *ctx->h_err;
  if (err) {
    DC_CUDA(cudaMemsetAsync(ctx->d_err, 0, sizeof(uint32_t), ctx->stream));
    // A split-K CTA that gave up on a wait skips its ticket on the tile counter, so the counter never returns to
    // zero; the next launch on that tile would then reduce too early or never. Every counter is cleared here,
    // which keeps the context usable after an expired wait.
    if ((err & (DC_DEVERR_GEMM_WAIT | DC_DEVERR_ATTN_WAIT | DC_DEVERR_WAIT_PROBE)) && ctx->counters)
      DC_CUDA(cudaMemsetAsync(ctx->counters, 0, ctx->counters_n * sizeof(uint32_t), ctx->stream));
    DC_CUDA(cudaStreamSynchronize(ctx->stream));
    if (err & (DC_DEVERR_TOKEN_ID | DC_DEVERR_BOUNDS))
      return dc_fail(DC_EINVAL, "decision.js: a kernel met %s (device error word 0x%x)",
                     (err & DC_DEVERR_TOKEN_ID) ? "a token id or readout row out of range" : "malformed sequence bounds",
                     err);
    return dc_fail(DC_ETIMEOUT, "decision.js: a kernel's bounded wait expired (device error word 0x%x)", err);
  }
  return DC_OK;
}

extern "C" int dc_sync(dc_ctx *ctx, int timeout_ms) {
  int rc = dc_use(ctx);
  if (rc) return rc;
  rc = enqueue_error_read(ctx);
  if (rc) return rc;
  if (timeout_ms < 0) {
    DC_CUDA(cudaStreamSynchronize(ctx->stream));
  } else {
    auto t0 = std::chrono::steady_clock::now();
    for (;;) {
      cudaError_t e = cudaStreamQuery(ctx->stream);
      if (e == cudaSuccess) break;
      if (e != cudaErrorNotReady)
        return dc_fail(DC_ECUDA, "decision.js: stream error: %s", cudaGetErrorString(e));
      auto ms = std::chrono::duration_cast<std::chrono::milliseconds>(std::chrono::steady_clock::now() - t0).count();
      if (ms > timeout_ms) return dc_fail(DC_ETIMEOUT, "decision.js: dc_sync timed out after %d ms", timeout_ms);
      std::this_thread::sleep_for(std::chrono::microseconds(50));
    }
  }
  return check_device_error(ctx);
}

// ------------------------------------------------------------------ scratch

int dc_scratch(dc_ctx *ctx, size_t bytes, size_t ncounters, void **scratch, uint32_t **counters) {
  if (bytes > ctx->scratch_bytes) {
    DC_CUDA(cudaStreamSynchronize(ctx->stream));
    if (ctx->scratch) DC_CUDA(cudaFree(ctx->scratch));
    ctx->scratch = nullptr;
    ctx->scratch_bytes = 0;
    size_t want = bytes < (1u << 20) ? (1u << 20) : bytes;
    cudaError_t e = cudaMalloc(&ctx->scratch, want);
    if (e != cudaSuccess) {
      cudaGetLastError();
      return dc_fail(DC_ENOMEM, "decision.js: cannot allocate %zu bytes of scratch", want);
    }
    ctx->scratch_bytes = want;
  }
  if (ncounters > ctx->counters_n) {
    DC_CUDA(cudaStreamSynchronize(ctx->stream));
    if (ctx->counters) DC_CUDA(cudaFree(ctx->counters));
    ctx->counters = nullptr;
    ctx->counters_n = 0;
    size_t want = ncounters < 4096 ? 4096 : ncounters;
    cudaError_t e = cudaMalloc(&ctx->counters, want * sizeof(uint32_t));
    if (e != cudaSuccess) {
      cudaGetLastError();
      return dc_fail(DC_ENOMEM, "decision.js: cannot allocate %zu tile counters", want);
    }
    DC_CUDA(cudaMemsetAsync(ctx->counters, 0, want * sizeof(uint32_t), ctx->stream));
    ctx->counters_n = want;
  }
  *scratch = ctx->scratch;
  *counters = ctx->counters;
  return DC_OK;
}

// ------------------------------------------------------------------ profiling

static cudaEvent_t take_event(dc_ctx *ctx) {
  if (!ctx->free_events.empty()) {
    cudaEvent_t e = ctx->free_events.back();
    ctx->free_events.pop_back();
    return e;
  }
  cudaEvent_t e;
  cudaEventCreate(&e);
  return e;
}

void dc_prof_begin(dc_ctx *ctx, int kind, double flops, double bytes) {
  if (!ctx->profiling) return;
  dc_profile_slot s;
  s.a = take_event(ctx);
  s.b = take_event(ctx);
  s.kind = kind;
  s.flops = flops;
  s.bytes = bytes;
  cudaEventRecord(s.a, ctx->stream);
  ctx->pending.push_back(s);
}

void dc_prof_end(dc_ctx *ctx) {
  if (!ctx->profiling || ctx->pending.empty()) return;
  cudaEventRecord(ctx->pending.back().b, ctx->stream);
}

static void drain(dc_ctx *ctx) {
  for (auto &s : ctx->pending) {
    cudaEventSynchronize(s.b);
    float ms = 0;
    cudaEventElapsedTime(&ms, s.a, s.b);
    ctx->prof_ms[s.kind] += ms;
    ctx->prof_n[s.kind] += 1;
    ctx->prof_flops[s.kind] += s.flops;
    ctx->prof_bytes[s.kind] += s.bytes;
    ctx->free_events.push_back(s.a);
    ctx->free_events.push_back(s.b);
  }
  ctx->pending.clear();
}

extern "C" int dc_profile(dc_ctx *ctx, int enable) {
  int rc = dc_use(ctx);
  if (rc) return rc;
  drain(ctx);
  for (int k = 0; k < DC_K_KINDS; k++) ctx->prof_ms[k] = ctx->prof_flops[k] = ctx->prof_bytes[k] = 0, ctx->prof_n[k] = 0;
  ctx->profiling = enable != 0;
  return DC_OK;
}

extern "C" int dc_profile_read(dc_ctx *ctx, int kind, double *ms, long long *launches, double *flops,
                               double *bytes) {
  int rc = dc_use(ctx);
  if (rc) return rc;
  DC_CHECK(kind >= 0 && kind < DC_K_KINDS, DC_EINVAL, "decision.js: bad profile kind %d", kind);
  drain(ctx);
  if (ms) *ms = ctx->prof_ms[kind];
  if (launches) *launches = ctx->prof_n[kind];
  if (flops) *flops = ctx->prof_flops[kind];
  if (bytes) *bytes = ctx->prof_bytes[kind];
  return DC_OK;
}
