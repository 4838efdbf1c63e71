// Models: the reference's manifest.json + weights.bin format read into device memory (loadWeights,
// src/gpu.ts:57-88), and the engine graphs:
//   - encoder: Eg2Engine.embed (src/eg2-engine.ts:72-141), with or without per-layer embeddings (PLE);
//   - decoder: D13BEngine.run  (src/d1-3b-engine.ts:44-108), attention and LFM2 short-conv layers;
//   - d3:      D3Engine.logits (src/d3-engine.ts:67-139), Gated DeltaNet and gated attention layers, code readout;
//   - omni:    D1OmniEngine.logits (src/omni-engine.ts:56-141), the LFM2 backbone, a transformer head, the scorer;
//   - laya:    LayaEngine.logits (src/laya-engine.ts:47-141), a ModernBERT encoder and the same head.
// Weights live in one device allocation laid out exactly as weights.bin (every tensor 256-byte aligned by the
// exporter), so a tensor's device address is base + its manifest offset. Activation buffers are grow-only
// per model, like the reference's ensure() (src/eg2-engine.ts:56-69).
#include <errno.h>
#include <fcntl.h>
#include <string.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cmath>
#include <fstream>
#include <sstream>

#include "dc_internal.h"
#include "dc_json.h"

int ops_add_rmsnorm(dc_ctx *, void *, const void *, const void *, void *, int, int, int, float);
int ops_sandwich(dc_ctx *, void *, const void *, const void *, const void *, void *, int, int, float, float);
int ops_qkv_norm_rope(dc_ctx *, void *, const void *, const void *, const int *, int, int, int, int, float, float,
                      int);
int ops_glu(dc_ctx *, const void *, void *, int, int, int, int);
int ops_interleave_rows(dc_ctx *, const void *, void *, long, long);
int ops_gather(dc_ctx *, const int *, const void *, const void *, void *, int, int, int, int);
int ops_encoder_meta(dc_ctx *, const int *, int, int, int, int *, int *, int *);
int ops_pool(dc_ctx *, const void *, const int *, const void *, float *, int, int, int);
int ops_leaf_logits(dc_ctx *, const void *, const int *, const void *, const int *, const void *, const void *,
                    float *, int, int, int, int, float, int, int);
int attn_launch(dc_ctx *, const void *, const int *, void *, int, int, int, int, float);
int ops_short_conv(dc_ctx *, const void *, const void *, const int *, void *, int, int);
int ops_conv_taps(dc_ctx *, const int *, int *, int);
int ops_ple_mix(dc_ctx *, const void *, const void *, const void *, void *, int, int, float);
int ops_gdn(dc_ctx *, const void *, long, long, int, const void *, const void *, const void *, const void *,
            const uint32_t *, int, float, void *, int);
int ops_qk_rope(dc_ctx *, void *, const void *, const void *, const int *, int, int, int, int, long, int, int, float,
                float);
int attn_launch_ex(dc_ctx *, const void *, const int *, void *, int, int, int, int, float, int, long, int);
int ops_readout(dc_ctx *, const void *, const float *, const int *, float *, int, int, int, int);
int ops_add_rows(dc_ctx *, const void *, const int *, const void *, void *, int, int, int);
int ops_bias_act(dc_ctx *, void *, const void *, int, int, int);
int ops_add_layernorm(dc_ctx *, void *, const void *, const void *, const void *, void *, int, int, int, float);
int ops_gather_rows(dc_ctx *, const void *, const int *, void *, int, int, int);
int ops_score(dc_ctx *, const void *, const void *, const void *, float *, int, int);

struct dc_tensor {
  int dtype = 0;  // 4, 8 (quantized), 16 (f16), 32 (f32)
  int64_t rows = 0, cols = 0;
  int64_t offset = 0, bytes = 0, scales = -1, scales_bytes = 0;
  bool glu_interleaved = false;  // fused gate|up rows stored as alternating gate, up rows
};

struct dc_model {
  dc_ctx *ctx = nullptr;
  dcj::Value manifest;
  std::map<std::string, dc_tensor> tensors;
  uint8_t *base = nullptr;  // device copy of weights.bin
  size_t size = 0;
  // activations (grow-only)
  size_t cap = 0;
  __half *x = nullptr, *normed = nullptr, *z = nullptr, *y = nullptr, *h = nullptr, *o = nullptr;
  // per-layer embeddings (encoders with ple > 0): the embedding rows xe [T, H], and gate / e / mix [T, ple]
  __half *xe = nullptr, *pg = nullptr, *pe = nullptr, *pm = nullptr;
  size_t ple_cap = 0;
  int32_t *meta = nullptr;  // ids | pos | rng (2 layer kinds) | bounds | leaves | leaf ids
  size_t meta_cap = 0;
  float *out = nullptr;
  size_t out_cap = 0;
  void *pinned = nullptr;
  size_t pinned_cap = 0;
  void *dmeta = nullptr;  // per-token metadata built on the device
  size_t dmeta_bytes = 0;
  double attn_keys = 0;  // sum over tokens of visible keys (profiling flops), 0 when unknown
  // One captured forward pass per model kind (see run_graphed).
  struct Graph {
    std::vector<uintptr_t> key, seen;  // key of the instantiated graph; key of the last pass run directly
    cudaGraphExec_t exec = nullptr;
  } genc, gdec, gd3, gomni, glaya;
};

// A forward pass is ~10 kernel launches per layer; replaying it as one CUDA graph removes the launch gaps. The
// graph is captured on the second consecutive pass with the same key -- the shape, every pointer the pass reads or
// writes (arguments, activations, metadata, split-K scratch) -- and replayed while the key stays the same. Every
// buffer only ever grows, so a pointer equal to the captured one still holds at least what the graph touches.
// Passes under profiling (per-launch events) and passes whose capture fails run directly.
template <class F>
static int run_graphed(dc_model *m, dc_model::Graph &gc, const std::vector<uintptr_t> &key, F &&core) {
  dc_ctx *ctx = m->ctx;
  if (ctx->profiling) return core();
  if (gc.exec && key == gc.key) {
    DC_CUDA(cudaGraphLaunch(gc.exec, ctx->stream));
    return DC_OK;
  }
  if (key != gc.seen) {
    gc.seen = key;
    return core();
  }
  cudaGraph_t graph = nullptr;
  DC_CUDA(cudaStreamBeginCapture(ctx->stream, cudaStreamCaptureModeThreadLocal));
  const int rc = core();
  const cudaError_t e = cudaStreamEndCapture(ctx->stream, &graph);
  cudaGraphExec_t exec = nullptr;
  if (!rc && e == cudaSuccess && graph && cudaGraphInstantiate(&exec, graph, 0) == cudaSuccess) {
    cudaGraphDestroy(graph);
    if (gc.exec) cudaGraphExecDestroy(gc.exec);
    gc.exec = exec;
    gc.key = key;
    DC_CUDA(cudaGraphLaunch(exec, ctx->stream));
    return DC_OK;
  }
  if (graph) cudaGraphDestroy(graph);
  cudaGetLastError();
  gc.seen.clear();
  return core();  // run it directly (and report its own error, if any)
}

static std::vector<uintptr_t> pass_key(dc_model *m, int kind, std::initializer_list<uintptr_t> args) {
  std::vector<uintptr_t> k = {(uintptr_t)kind};
  k.insert(k.end(), args.begin(), args.end());
  for (const void *p : {(const void *)m->x, (const void *)m->normed, (const void *)m->z, (const void *)m->y,
                        (const void *)m->h, (const void *)m->o, (const void *)m->meta, (const void *)m->out,
                        (const void *)m->dmeta, (const void *)m->ctx->scratch, (const void *)m->ctx->counters,
                        (const void *)m->xe, (const void *)m->pg, (const void *)m->pe, (const void *)m->pm})
    k.push_back((uintptr_t)p);
  return k;
}

static const dcj::Value *cfg(dc_model *m, const char *k) {
  const dcj::Value *c = m->manifest.get("config");
  return c ? c->get(k) : nullptr;
}

static bool cfg_num(dc_model *m, const std::string &path, double &out) {
  const dcj::Value *v = m->manifest.get("config");
  size_t p = 0;
  while (v && p <= path.size()) {
    size_t q = path.find('.', p);
    std::string key = path.substr(p, q == std::string::npos ? std::string::npos : q - p);
    if (v->kind == dcj::Value::Arr) {
      char *end = nullptr;
      long i = strtol(key.c_str(), &end, 10);
      v = (*end == 0 && i >= 0 && (size_t)i < v->arr.size()) ? &v->arr[i] : nullptr;
    } else {
      v = v->get(key);
    }
    if (q == std::string::npos) break;
    p = q + 1;
  }
  if (!v) return false;
  if (v->kind == dcj::Value::Num) { out = v->num; return true; }
  if (v->kind == dcj::Value::Bool) { out = v->b ? 1 : 0; return true; }
  return false;
}

// ------------------------------------------------------------------ loading

static int read_file(const std::string &path, std::string &out) {
  std::ifstream f(path, std::ios::binary);
  if (!f) return dc_fail(DC_EIO, "decision.js: cannot open %s", path.c_str());
  std::stringstream ss;
  ss << f.rdbuf();
  out = ss.str();
  return DC_OK;
}

static int parse_section(dc_model *m, const dcj::Value *ts, int64_t file_size);

// The manifest's "tensors" and, when present, its "host" section (EmbeddingGemma 2's decision head in f32,
// scripts/export-eg2.py:119-123; the reference reads those on the host, here they are uploaded with the rest).
static int parse_tensors(dc_model *m, int64_t file_size) {
  const dcj::Value *ts = m->manifest.get("tensors");
  DC_CHECK(ts && ts->kind == dcj::Value::Obj, DC_EFORMAT, "decision.js: manifest.json has no tensors");
  int rc = parse_section(m, ts, file_size);
  if (rc) return rc;
  const dcj::Value *host = m->manifest.get("host");
  if (host) {
    DC_CHECK(host->kind == dcj::Value::Obj, DC_EFORMAT, "decision.js: manifest.json: host must be an object");
    rc = parse_section(m, host, file_size);
  }
  return rc;
}

static int parse_section(dc_model *m, const dcj::Value *ts, int64_t file_size) {
  for (auto &kv : ts->obj) {
    const dcj::Value &t = kv.second;
    const dcj::Value *dt = t.get("dtype"), *sh = t.get("shape"), *off = t.get("offset"), *by = t.get("bytes");
    DC_CHECK(dt && dt->kind == dcj::Value::Str && sh && sh->kind == dcj::Value::Arr && off && off->is_num() && by &&
                 by->is_num(),
             DC_EFORMAT, "decision.js: tensor %s: dtype, shape, offset and bytes are required", kv.first.c_str());
    dc_tensor d;
    const std::string &s = dt->str;
    d.dtype = s == "q4" ? 4 : s == "q8" ? 8 : s == "f16" ? 16 : s == "f32" ? 32 : 0;
    DC_CHECK(d.dtype, DC_EFORMAT, "decision.js: tensor %s: unknown dtype %s", kv.first.c_str(), s.c_str());
    int64_t numel = 1;
    for (auto &e : sh->arr) {
      DC_CHECK(e.is_num() && e.num >= 0, DC_EFORMAT, "decision.js: tensor %s: bad shape", kv.first.c_str());
      numel *= (int64_t)e.num;
    }
    d.rows = sh->arr.empty() ? 1 : (int64_t)sh->arr[0].num;
    d.cols = sh->arr.size() >= 2 ? numel / (d.rows ? d.rows : 1) : numel;
    d.offset = (int64_t)off->num;
    d.bytes = (int64_t)by->num;
    int64_t want = d.dtype == 8 ? numel : d.dtype == 4 ? numel / 2 : d.dtype == 16 ? 2 * numel : 4 * numel;
    DC_CHECK(d.bytes == want, DC_EFORMAT, "decision.js: tensor %s: %lld bytes for %lld values of %s",
             kv.first.c_str(), (long long)d.bytes, (long long)numel, s.c_str());
    DC_CHECK(d.offset >= 0 && d.offset + d.bytes <= file_size, DC_EIO,
             "decision.js: tensor %s lies past the end of weights.bin (%lld + %lld > %lld)", kv.first.c_str(),
             (long long)d.offset, (long long)d.bytes, (long long)file_size);
    // the kernels move rows in 16-byte vectors (the reference's writer pads every blob to 256 bytes)
    DC_CHECK(d.offset % 16 == 0, DC_EFORMAT, "decision.js: tensor %s: offset %lld is not 16-byte aligned",
             kv.first.c_str(), (long long)d.offset);
    if (d.dtype == 4 || d.dtype == 8) {
      const dcj::Value *sc = t.get("scales"), *sb = t.get("scales_bytes");
      DC_CHECK(sh->arr.size() == 2 && d.cols % 32 == 0, DC_EFORMAT,
               "decision.js: tensor %s: a quantized tensor is [N, K] with K a multiple of 32", kv.first.c_str());
      DC_CHECK(sc && sc->is_num() && sb && sb->is_num(), DC_EFORMAT, "decision.js: tensor %s: scales missing",
               kv.first.c_str());
      d.scales = (int64_t)sc->num;
      d.scales_bytes = (int64_t)sb->num;
      DC_CHECK(d.scales_bytes == d.rows * (d.cols / 32) * 2, DC_EFORMAT,
               "decision.js: tensor %s: %lld scale bytes, wanted %lld", kv.first.c_str(), (long long)d.scales_bytes,
               (long long)(d.rows * (d.cols / 32) * 2));
      DC_CHECK(d.scales >= 0 && d.scales + d.scales_bytes <= file_size, DC_EIO,
               "decision.js: tensor %s: scales lie past the end of weights.bin", kv.first.c_str());
      DC_CHECK(d.scales % 2 == 0, DC_EFORMAT, "decision.js: tensor %s: scales must be 2-byte aligned",
               kv.first.c_str());
    }
    m->tensors[kv.first] = d;
  }
  return DC_OK;
}

// Fused gate|up weights (`*.gu` of the encoder, `*.w13` of the decoder) are re-laid out once at load so that the
// gate and up rows of every output are adjacent (rows 2i, 2i + 1): the GEMM's epilogue then gates in place (the reference re-lays out its SwiGLU weights for the same purpose, src/kernels.ts:525-538).
static int interleave_glu(dc_model *m) {
  for (auto &kv : m->tensors) {
    dc_tensor &t = kv.second;
    const std::string &n = kv.first;
    const bool fused = (n.size() > 3 && n.compare(n.size() - 3, 3, ".gu") == 0) ||
                       (n.size() > 4 && n.compare(n.size() - 4, 4, ".w13") == 0);
    if (!fused || (t.dtype != 4 && t.dtype != 8) || t.rows % 128 != 0) continue;
    const long row_codes = t.cols * t.dtype / 8, row_scales = t.cols / 32 * 2;
    void *tmp = nullptr;
    if (cudaMalloc(&tmp, (size_t)t.bytes) != cudaSuccess) {
      cudaGetLastError();
      return dc_fail(DC_ENOMEM, "decision.js: cannot allocate %lld bytes to re-lay out %s", (long long)t.bytes,
                     n.c_str());
    }
    int rc = ops_interleave_rows(m->ctx, m->base + t.offset, tmp, t.rows, row_codes);
    if (!rc && cudaMemcpyAsync(m->base + t.offset, tmp, (size_t)t.bytes, cudaMemcpyDeviceToDevice, m->ctx->stream))
      rc = dc_fail(DC_ECUDA, "decision.js: re-layout copy failed");
    if (!rc) rc = ops_interleave_rows(m->ctx, m->base + t.scales, tmp, t.rows, row_scales);
    if (!rc && cudaMemcpyAsync(m->base + t.scales, tmp, (size_t)t.scales_bytes, cudaMemcpyDeviceToDevice,
                               m->ctx->stream))
      rc = dc_fail(DC_ECUDA, "decision.js: re-layout copy failed");
    cudaStreamSynchronize(m->ctx->stream);
    cudaFree(tmp);
    if (rc) return rc;
    t.glu_interleaved = true;
  }
  return DC_OK;
}

extern "C" int dc_check_weights(const char *dir) {
  DC_CHECK(dir, DC_EINVAL, "decision.js: null argument");
  std::string d(dir);
  if (!d.empty() && d.back() != '/') d += '/';
  std::string text;
  int rc = read_file(d + "manifest.json", text);
  if (rc) return rc;
  dc_model m;
  std::string err;
  if (!dcj::Parser(text).parse(m.manifest, err)) return dc_fail(DC_EFORMAT, "decision.js: manifest.json: %s", err.c_str());
  struct stat st;
  if (stat((d + "weights.bin").c_str(), &st) != 0)
    return dc_fail(DC_EIO, "decision.js: cannot open %sweights.bin: %s", d.c_str(), strerror(errno));
  rc = parse_tensors(&m, st.st_size);
  if (rc) return rc;
  const dcj::Value *total = m.manifest.get("bytes");
  if (total && total->is_num() && (int64_t)total->num > (int64_t)st.st_size)
    return dc_fail(DC_EIO, "decision.js: weights.bin holds %lld bytes, the manifest says %lld", (long long)st.st_size,
                   (long long)total->num);
  return DC_OK;
}

extern "C" int dc_load_weights(dc_ctx *ctx, const char *dir, dc_model **out) {
  DC_CHECK(dir && out, DC_EINVAL, "decision.js: null argument");
  *out = nullptr;
  int rc = dc_use(ctx);
  if (rc) return rc;
  std::string d(dir);
  if (!d.empty() && d.back() != '/') d += '/';
  std::string text;
  rc = read_file(d + "manifest.json", text);
  if (rc) return rc;
  dc_model *m = new dc_model();
  m->ctx = ctx;
  std::string err;
  if (!dcj::Parser(text).parse(m->manifest, err)) {
    delete m;
    return dc_fail(DC_EFORMAT, "decision.js: manifest.json: %s", err.c_str());
  }
  const std::string bin = d + "weights.bin";
  int fd = open(bin.c_str(), O_RDONLY);
  if (fd < 0) {
    delete m;
    return dc_fail(DC_EIO, "decision.js: cannot open %s: %s", bin.c_str(), strerror(errno));
  }
  struct stat st;
  fstat(fd, &st);
  const int64_t fsize = st.st_size;
  rc = parse_tensors(m, fsize);
  const dcj::Value *total = m->manifest.get("bytes");
  if (!rc && total && total->is_num() && (int64_t)total->num > fsize)
    rc = dc_fail(DC_EIO, "decision.js: weights.bin holds %lld bytes, the manifest says %lld", (long long)fsize,
                 (long long)total->num);
  if (rc) {
    close(fd);
    delete m;
    return rc;
  }
  m->size = (size_t)fsize;
  if (cudaMalloc(&m->base, m->size ? m->size : 16) != cudaSuccess) {
    cudaGetLastError();
    close(fd);
    delete m;
    return dc_fail(DC_ENOMEM, "decision.js: cannot allocate %zu bytes of weights on device %d", (size_t)fsize,
                   ctx->device);
  }
  // stream the file through two pinned chunks
  const size_t CH = 64u << 20;
  void *pin[2] = {nullptr, nullptr};
  cudaEvent_t ev[2];
  rc = DC_OK;
  if (cudaHostAlloc(&pin[0], CH, cudaHostAllocDefault) != cudaSuccess ||
      cudaHostAlloc(&pin[1], CH, cudaHostAllocDefault) != cudaSuccess) {
    cudaGetLastError();
    rc = dc_fail(DC_ENOMEM, "decision.js: cannot allocate pinned staging memory");
  }
  cudaEventCreate(&ev[0]);
  cudaEventCreate(&ev[1]);
  for (size_t o = 0, i = 0; !rc && o < m->size; o += CH, i++) {
    const size_t n = std::min(CH, m->size - o);
    cudaEventSynchronize(ev[i & 1]);
    size_t got = 0;
    while (got < n) {
      ssize_t r = pread(fd, (uint8_t *)pin[i & 1] + got, n - got, (off_t)(o + got));
      if (r <= 0) break;
      got += (size_t)r;
    }
    if (got != n) {
      rc = dc_fail(DC_EIO, "decision.js: short read of weights.bin at byte %zu", o + got);
      break;
    }
    if (cudaMemcpyAsync(m->base + o, pin[i & 1], n, cudaMemcpyHostToDevice, ctx->stream) != cudaSuccess ||
        cudaEventRecord(ev[i & 1], ctx->stream) != cudaSuccess) {
      rc = dc_fail(DC_ECUDA, "decision.js: weight upload failed: %s", cudaGetErrorString(cudaGetLastError()));
      break;
    }
  }
  cudaStreamSynchronize(ctx->stream);
  cudaEventDestroy(ev[0]);
  cudaEventDestroy(ev[1]);
  if (pin[0]) cudaFreeHost(pin[0]);
  if (pin[1]) cudaFreeHost(pin[1]);
  close(fd);
  if (!rc) rc = interleave_glu(m);
  if (rc) {
    dc_model_free(m);
    return rc;
  }
  *out = m;
  return DC_OK;
}

extern "C" int dc_model_free(dc_model *m) {
  if (!m) return DC_OK;
  cudaSetDevice(m->ctx->device);
  cudaStreamSynchronize(m->ctx->stream);
  for (void *p : {(void *)m->base, (void *)m->x, (void *)m->normed, (void *)m->z, (void *)m->y, (void *)m->h,
                  (void *)m->o, (void *)m->meta, (void *)m->out, m->dmeta, (void *)m->xe, (void *)m->pg,
                  (void *)m->pe, (void *)m->pm})
    if (p) cudaFree(p);
  if (m->pinned) cudaFreeHost(m->pinned);
  for (dc_model::Graph *g : {&m->genc, &m->gdec, &m->gd3, &m->gomni, &m->glaya})
    if (g->exec) cudaGraphExecDestroy(g->exec);
  delete m;
  return DC_OK;
}

extern "C" int dc_model_kind(dc_model *m, char *buf, size_t len) {
  DC_CHECK(m && buf && len, DC_EINVAL, "decision.js: null argument");
  const dcj::Value *k = cfg(m, "model");
  std::string s = k && k->kind == dcj::Value::Str ? k->str : "";
  // the reference's rule (src/d1.ts:63-64): no explicit model and no head_layers means d1-3B
  if (s.empty()) s = cfg(m, "head_layers") ? "d1-omni" : "d1-3b";
  snprintf(buf, len, "%s", s.c_str());
  return DC_OK;
}

extern "C" int dc_model_config_f(dc_model *m, const char *key, double *out) {
  DC_CHECK(m && key && out, DC_EINVAL, "decision.js: null argument");
  DC_CHECK(cfg_num(m, key, *out), DC_EINVAL, "decision.js: config has no number at %s", key);
  return DC_OK;
}

extern "C" int dc_model_tensor(dc_model *m, const char *name, void **data, void **scales, int *dtype, int64_t *rows,
                               int64_t *cols) {
  DC_CHECK(m && name, DC_EINVAL, "decision.js: null argument");
  auto it = m->tensors.find(name);
  DC_CHECK(it != m->tensors.end(), DC_EINVAL, "decision.js: the model has no tensor %s", name);
  const dc_tensor &t = it->second;
  if (data) *data = m->base + t.offset;
  if (scales) *scales = t.scales >= 0 ? (void *)(m->base + t.scales) : nullptr;
  if (dtype) *dtype = t.dtype;
  if (rows) *rows = t.rows;
  if (cols) *cols = t.cols;
  return DC_OK;
}

// ------------------------------------------------------------------ graphs

namespace {

struct Q {
  const void *codes = nullptr, *scales = nullptr;
  int N = 0, K = 0, bits = 0;
  bool glu = false;  // rows interleaved for the gated epilogue
};

int qw(dc_model *m, const std::string &name, Q &q, int K = -1) {
  auto it = m->tensors.find(name);
  DC_CHECK(it != m->tensors.end(), DC_EFORMAT, "decision.js: the model has no tensor %s", name.c_str());
  const dc_tensor &t = it->second;
  DC_CHECK(t.dtype == 4 || t.dtype == 8, DC_EFORMAT, "decision.js: %s must be q4 or q8", name.c_str());
  DC_CHECK(K < 0 || t.cols == K, DC_EFORMAT, "decision.js: %s has K=%lld, the graph needs %d", name.c_str(),
           (long long)t.cols, K);
  q.codes = m->base + t.offset;
  q.scales = m->base + t.scales;
  q.N = (int)t.rows;
  q.K = (int)t.cols;
  q.bits = t.dtype;
  q.glu = t.glu_interleaved;
  return DC_OK;
}

int fw(dc_model *m, const std::string &name, const void *&p, int64_t numel) {
  auto it = m->tensors.find(name);
  DC_CHECK(it != m->tensors.end(), DC_EFORMAT, "decision.js: the model has no tensor %s", name.c_str());
  const dc_tensor &t = it->second;
  DC_CHECK(t.dtype == 16 && t.bytes == 2 * numel, DC_EFORMAT, "decision.js: %s must be f16 with %lld values",
           name.c_str(), (long long)numel);
  p = m->base + t.offset;
  return DC_OK;
}

// A model's weights are written at load time and the stream is synchronised after, so its matmuls may request
// their codes and scales before the kernel before them completes (dc_ctx::static_weights).
struct StaticWeights {
  dc_ctx *c;
  bool was;
  explicit StaticWeights(dc_ctx *ctx) : c(ctx), was(ctx->static_weights) { c->static_weights = true; }
  ~StaticWeights() { c->static_weights = was; }
};

int matmul(dc_model *m, const __half *X, const Q &w, __half *Y, int M) {
  dc_ctx *ctx = m->ctx;
  StaticWeights sw(ctx);
  const int form = qgemm_pick_form(M, w.N, w.K, w.bits, ctx->sms);
  dc_prof_begin(ctx, M > 128 ? DC_K_QGEMM : DC_K_QGEMV, 2.0 * M * w.N * w.K,
                (double)w.N * w.K * w.bits / 8 + (double)w.N * w.K / 16 + 2.0 * M * w.K + 2.0 * M * w.N);
  int rc = qgemm_launch(ctx, X, w.codes, w.scales, Y, M, w.N, w.K, w.bits, form, 0);
  dc_prof_end(ctx);
  return rc;
}

// h[M, I] = act(gate) * up for a fused gate|up weight: one persistent GEMM with the gated epilogue when the rows
// are interleaved and M is a prefill shape; otherwise the matmul into z, then the gating kernel.
int gated(dc_model *m, const __half *X, const Q &w, __half *z, __half *h, int M, int act) {
  dc_ctx *ctx = m->ctx;
  const int I = w.N / 2;
  if (w.glu && M > 128) {
    dc_prof_begin(ctx, DC_K_QGEMM, 2.0 * M * w.N * w.K,
                  (double)w.N * w.K * w.bits / 8 + (double)w.N * w.K / 16 + 2.0 * M * w.K + 2.0 * M * I);
    StaticWeights sw(ctx);
    int rc = qgemm_launch_glu(ctx, X, w.codes, w.scales, h, M, w.N, w.K, w.bits, act == DC_ACT_GELU_TANH ? 1 : 2);
    dc_prof_end(ctx);
    return rc;
  }
  int rc = matmul(m, X, w, z, M);
  if (rc) return rc;
  dc_prof_begin(ctx, DC_K_OTHER, 0, 6.0 * M * I);
  rc = ops_glu(ctx, z, h, M, I, act, w.glu ? 1 : 0);
  dc_prof_end(ctx);
  return rc;
}

template <class T>
int grow(T *&p, size_t &cap, size_t want, size_t elem) {
  if (want <= cap) return DC_OK;
  if (p) cudaFree(p);
  p = nullptr;
  cap = 0;
  if (cudaMalloc((void **)&p, want * elem) != cudaSuccess) {
    cudaGetLastError();
    return dc_fail(DC_ENOMEM, "decision.js: cannot allocate %zu bytes of activations", want * elem);
  }
  cap = want;
  return DC_OK;
}

// Activation buffers for T tokens: x, normed, o [T,H]; z [T,zc]; y [T,yc]; h [T,I].
int ensure(dc_model *m, int T, int H, int zc, int yc, int I) {
  if ((size_t)T <= m->cap && m->x) return DC_OK;
  cudaStreamSynchronize(m->ctx->stream);
  for (__half **p : {&m->x, &m->normed, &m->z, &m->y, &m->h, &m->o}) {
    if (*p) cudaFree(*p);
    *p = nullptr;
  }
  const size_t cap = std::max<size_t>((size_t)T, 256);
  size_t c;
  int rc = DC_OK;
  c = 0; rc = rc ? rc : grow(m->x, c, cap * H, 2);
  c = 0; rc = rc ? rc : grow(m->normed, c, cap * H, 2);
  c = 0; rc = rc ? rc : grow(m->o, c, cap * H, 2);
  c = 0; rc = rc ? rc : grow(m->z, c, cap * zc, 2);
  c = 0; rc = rc ? rc : grow(m->y, c, cap * yc, 2);
  c = 0; rc = rc ? rc : grow(m->h, c, cap * I, 2);
  if (rc) return rc;
  m->cap = cap;
  return DC_OK;
}

// The per-layer-embedding buffers for T tokens: xe [T, H], gate / e / mix [T, P].
int ensure_ple(dc_model *m, int T, int H, int P) {
  if ((size_t)T <= m->ple_cap && m->xe) return DC_OK;
  cudaStreamSynchronize(m->ctx->stream);
  for (__half **p : {&m->xe, &m->pg, &m->pe, &m->pm}) {
    if (*p) cudaFree(*p);
    *p = nullptr;
  }
  const size_t cap = std::max<size_t>((size_t)T, 256);
  size_t c;
  int rc = DC_OK;
  c = 0; rc = rc ? rc : grow(m->xe, c, cap * H, 2);
  c = 0; rc = rc ? rc : grow(m->pg, c, cap * P, 2);
  c = 0; rc = rc ? rc : grow(m->pe, c, cap * P, 2);
  c = 0; rc = rc ? rc : grow(m->pm, c, cap * P, 2);
  if (rc) return rc;
  m->ple_cap = cap;
  return DC_OK;
}

// Per-token device metadata (grow-only, m->dmeta): at least `bytes`.
int ensure_dmeta(dc_model *m, size_t bytes) {
  if (bytes <= m->dmeta_bytes) return DC_OK;
  DC_CUDA(cudaStreamSynchronize(m->ctx->stream));
  if (m->dmeta) cudaFree(m->dmeta);
  m->dmeta = nullptr;
  m->dmeta_bytes = 0;
  if (cudaMalloc(&m->dmeta, bytes) != cudaSuccess) {
    cudaGetLastError();
    return dc_fail(DC_ENOMEM, "decision.js: cannot allocate token metadata");
  }
  m->dmeta_bytes = bytes;
  return DC_OK;
}

// Copies host metadata into the model's device metadata buffer through pinned memory; returns device pointers.
int upload_meta(dc_model *m, const std::vector<std::pair<const void *, size_t>> &parts,
                std::vector<int32_t *> &dptr) {
  size_t total = 0;
  for (auto &p : parts) total += (p.second + 255) & ~size_t(255);
  int rc = grow(m->meta, m->meta_cap, total / 4 + 64, 4);
  if (rc) return rc;
  if (total > m->pinned_cap) {
    cudaStreamSynchronize(m->ctx->stream);
    if (m->pinned) cudaFreeHost(m->pinned);
    m->pinned = nullptr;
    m->pinned_cap = 0;
    if (cudaHostAlloc(&m->pinned, total, cudaHostAllocDefault) != cudaSuccess) {
      cudaGetLastError();
      return dc_fail(DC_ENOMEM, "decision.js: cannot allocate pinned metadata");
    }
    m->pinned_cap = total;
  }
  DC_CUDA(cudaStreamSynchronize(m->ctx->stream));  // the staging buffer is reused
  size_t off = 0;
  dptr.clear();
  for (auto &p : parts) {
    if (p.second) memcpy((uint8_t *)m->pinned + off, p.first, p.second);
    dptr.push_back((int32_t *)((uint8_t *)m->meta + off));
    off += (p.second + 255) & ~size_t(255);
  }
  DC_CUDA(cudaMemcpyAsync(m->meta, m->pinned, off, cudaMemcpyHostToDevice, m->ctx->stream));
  return DC_OK;
}

int download_out(dc_model *m, float *h_out, size_t n) {
  if (n * sizeof(float) > m->pinned_cap) {
    DC_CUDA(cudaStreamSynchronize(m->ctx->stream));
    if (m->pinned) cudaFreeHost(m->pinned);
    m->pinned = nullptr;
    m->pinned_cap = 0;
    if (cudaHostAlloc(&m->pinned, n * sizeof(float), cudaHostAllocDefault) != cudaSuccess) {
      cudaGetLastError();
      return dc_fail(DC_ENOMEM, "decision.js: cannot allocate pinned output");
    }
    m->pinned_cap = n * sizeof(float);
  }
  DC_CUDA(cudaMemcpyAsync(m->pinned, m->out, n * sizeof(float), cudaMemcpyDeviceToHost, m->ctx->stream));
  int rc = dc_sync(m->ctx, -1);
  if (rc) return rc;
  memcpy(h_out, m->pinned, n * sizeof(float));
  return DC_OK;
}

#define RC(x)              \
  do {                     \
    int rc_ = (x);         \
    if (rc_) return rc_;   \
  } while (0)

}  // namespace

namespace {

// The encoder's configuration, read once per call from the manifest.
struct EncGeom {
  int H = 0, I = 0, heads = 0, L = 0, window = 0, zc = 0, yc = 0, N = 0, vnorm = 1, ple = 0;
  float eps = 1e-6f, attn_scale = 1.0f;
  bool proj = false;
};

int encoder_geom(dc_model *m, EncGeom &g) {
  double v;
  auto num = [&](const std::string &k, double dflt) { return cfg_num(m, k, v) ? v : dflt; };
  DC_CHECK(cfg_num(m, "hidden", v), DC_EFORMAT, "decision.js: encoder config needs hidden");
  g.H = (int)v;
  g.I = (int)num("intermediate", 0), g.heads = (int)num("heads", 0);
  g.eps = (float)num("eps", 1e-6);
  g.attn_scale = (float)num("attn_scale", 1.0);
  g.vnorm = (int)num("v_norm", 1);
  g.ple = (int)num("ple", 0);
  DC_CHECK(g.ple >= 0 && g.ple % 8 == 0 && g.ple <= 1024, DC_EFORMAT,
           "decision.js: per-layer embedding width ple=%d must be a multiple of 8, at most 1024", g.ple);
  const dcj::Value *lt = cfg(m, "layer_types");
  DC_CHECK(lt && lt->kind == dcj::Value::Arr && !lt->arr.empty() && g.I > 0 && g.heads > 0, DC_EFORMAT,
           "decision.js: encoder config needs layer_types, intermediate, heads");
  g.L = (int)num("layers", (double)lt->arr.size());
  DC_CHECK(g.L <= (int)lt->arr.size(), DC_EFORMAT, "decision.js: fewer layer_types than layers");
  g.window = (int)num("window", 0);
  g.zc = 2 * g.I, g.yc = 0;
  for (int i = 0; i < g.L; i++) {
    const std::string t = lt->arr[i].str;
    const int D = (int)num("head_dim." + t, 0), kv = (int)num("kv_heads." + t, 0);
    DC_CHECK(D > 0 && kv > 0 && g.heads % kv == 0, DC_EFORMAT, "decision.js: bad head_dim/kv_heads for %s",
             t.c_str());
    g.zc = std::max(g.zc, (g.heads + 2 * kv) * D);
    g.yc = std::max(g.yc, g.heads * D);
  }
  g.proj = m->tensors.count("projection") > 0;
  g.N = g.proj ? (int)m->tensors["projection"].rows : g.H;
  return DC_OK;
}

// The per-token metadata the device builds for itself: positions and two key-range tables.
int32_t *dmeta_ptr(dc_model *m, int T, int part) {
  // layout: pos [T] | full [T,4] | slide [T,4], each 256-byte aligned
  const size_t a = ((size_t)T * 4 + 255) & ~size_t(255), b = ((size_t)T * 16 + 255) & ~size_t(255);
  uint8_t *base = (uint8_t *)m->dmeta;
  return (int32_t *)(part == 0 ? base : part == 1 ? base + a : base + a + b);
}

// Eg2Engine.embed's GPU part on device-resident inputs (src/eg2-engine.ts:103-131): gather, the layer loop,
// then mean pooling into d_out [S, N].
int encoder_core(dc_model *m, const EncGeom &g, const int32_t *d_ids, const int32_t *d_bounds, int T, int S,
                 float *d_out) {
  dc_ctx *ctx = m->ctx;
  double v;
  auto num = [&](const std::string &k, double dflt) { return cfg_num(m, k, v) ? v : dflt; };
  const dcj::Value *lt = cfg(m, "layer_types");
  const int H = g.H, I = g.I, heads = g.heads, L = g.L;
  Q emb;
  RC(qw(m, "embed", emb, H));
  RC(ensure(m, T, H, g.zc, g.yc, I));
  RC(ensure_dmeta(m, (((size_t)T * 4 + 255) & ~size_t(255)) + 2 * (((size_t)T * 16 + 255) & ~size_t(255))));
  if (g.ple) RC(ensure_ple(m, T, H, g.ple));
  int32_t *d_pos = dmeta_ptr(m, T, 0), *d_full = dmeta_ptr(m, T, 1), *d_slide = dmeta_ptr(m, T, 2);
  dc_prof_begin(ctx, DC_K_OTHER, 0, (double)T * 36);
  RC(ops_encoder_meta(ctx, d_bounds, S, T, g.window, d_pos, d_full, d_slide));
  dc_prof_end(ctx);
  dc_prof_begin(ctx, DC_K_OTHER, 0, (double)T * H * 3);
  RC(ops_gather(ctx, d_ids, emb.codes, emb.scales, m->x, T, H, emb.bits, emb.N));
  dc_prof_end(ctx);
  const void *plen = nullptr;
  if (g.ple) {  // the embedding rows again: each layer projects its own per-layer embedding from them
    RC(fw(m, "ple.norm", plen, g.ple));
    DC_CUDA(cudaMemcpyAsync(m->xe, m->x, (size_t)T * H * 2, cudaMemcpyDeviceToDevice, ctx->stream));
  }
  const void *w0;
  RC(fw(m, "layers.0.input_layernorm", w0, H));
  dc_prof_begin(ctx, DC_K_NORM, 0, 4.0 * T * H);
  RC(ops_add_rmsnorm(ctx, m->x, nullptr, w0, m->normed, T, H, 0, g.eps));
  dc_prof_end(ctx);
  for (int i = 0; i < L; i++) {
    const std::string p = "layers." + std::to_string(i) + ".";
    const std::string typ = lt->arr[i].str;
    const int D = (int)num("head_dim." + typ, 0), kv = (int)num("kv_heads." + typ, 0);
    const float theta = (float)num("rope_theta." + typ, 10000.0);
    const bool sliding = typ == "sliding_attention" && g.window > 0;
    Q wqkv, wo, wgu, wdown;
    RC(qw(m, p + "qkv", wqkv, H));
    RC(qw(m, p + "o", wo, heads * D));
    RC(qw(m, p + "gu", wgu, H));
    RC(qw(m, p + "down", wdown, I));
    DC_CHECK(wqkv.N == (heads + 2 * kv) * D && wo.N == H && wgu.N == 2 * I && wdown.N == H, DC_EFORMAT,
             "decision.js: layer %d: matmul shapes do not match the config", i);
    const void *qn, *kn, *n1, *n2, *n3, *nx;
    RC(fw(m, p + "q_norm", qn, D));
    RC(fw(m, p + "k_norm", kn, D));
    RC(fw(m, p + "post_attention_layernorm", n1, H));
    RC(fw(m, p + "pre_feedforward_layernorm", n2, H));
    RC(fw(m, p + "post_feedforward_layernorm", n3, H));
    RC(fw(m, i + 1 < L ? "layers." + std::to_string(i + 1) + ".input_layernorm" : std::string("final_norm"), nx, H));
    const float lscale = (float)num("layer_scalars." + std::to_string(i), 1.0);

    RC(matmul(m, m->normed, wqkv, m->z, T));
    dc_prof_begin(ctx, DC_K_NORM, 0, 4.0 * T * (heads + 2 * kv) * D);
    RC(ops_qkv_norm_rope(ctx, m->z, qn, kn, d_pos, T, heads, kv, D, g.eps, theta, g.vnorm));
    dc_prof_end(ctx);
    dc_prof_begin(ctx, DC_K_ATTN, m->attn_keys * 4.0 * heads * D, 0);
    RC(attn_launch(ctx, m->z, sliding ? d_slide : d_full, m->y, T, heads, kv, D, g.attn_scale));
    dc_prof_end(ctx);
    RC(matmul(m, m->y, wo, m->o, T));
    dc_prof_begin(ctx, DC_K_NORM, 0, 10.0 * T * H);
    RC(ops_sandwich(ctx, m->x, m->o, n1, n2, m->normed, T, H, g.eps, 1.0f));
    dc_prof_end(ctx);
    RC(gated(m, m->normed, wgu, m->z, m->h, T, DC_ACT_GELU_TANH));
    RC(matmul(m, m->h, wdown, m->o, T));
    if (!g.ple) {
      dc_prof_begin(ctx, DC_K_NORM, 0, 10.0 * T * H);
      RC(ops_sandwich(ctx, m->x, m->o, n3, nx, m->normed, T, H, g.eps, lscale));
      dc_prof_end(ctx);
      continue;
    }
    // per-layer embedding (src/eg2-engine.ts:123-128): the MLP's post-norm alone, then
    // x = (x + norm(proj(gelu(gate(x)) * norm(ple_in(xe))))) * layer scalar, and the next layer's input norm
    Q wpg, wpi, wpp;
    RC(qw(m, p + "ple_gate", wpg, H));
    RC(qw(m, p + "ple_in", wpi, H));
    RC(qw(m, p + "ple_proj", wpp, g.ple));
    DC_CHECK(wpg.N == g.ple && wpi.N == g.ple && wpp.N == H, DC_EFORMAT,
             "decision.js: layer %d: per-layer embedding shapes do not match the config", i);
    const void *npl;
    RC(fw(m, p + "ple_norm", npl, H));
    dc_prof_begin(ctx, DC_K_NORM, 0, 6.0 * T * H);
    RC(ops_sandwich(ctx, m->x, m->o, n3, nullptr, nullptr, T, H, g.eps, 1.0f));
    dc_prof_end(ctx);
    RC(matmul(m, m->x, wpg, m->pg, T));
    RC(matmul(m, m->xe, wpi, m->pe, T));
    dc_prof_begin(ctx, DC_K_NORM, 0, 6.0 * T * g.ple);
    RC(ops_ple_mix(ctx, m->pg, m->pe, plen, m->pm, T, g.ple, g.eps));
    dc_prof_end(ctx);
    RC(matmul(m, m->pm, wpp, m->o, T));
    dc_prof_begin(ctx, DC_K_NORM, 0, 10.0 * T * H);
    RC(ops_sandwich(ctx, m->x, m->o, npl, nx, m->normed, T, H, g.eps, lscale));
    dc_prof_end(ctx);
  }
  const void *pw = nullptr;
  if (g.proj) RC(fw(m, "projection", pw, (int64_t)g.N * H));
  dc_prof_begin(ctx, DC_K_OTHER, 0, 2.0 * T * H);
  RC(ops_pool(ctx, m->normed, d_bounds, pw, d_out, S, H, g.N));
  dc_prof_end(ctx);
  return DC_OK;
}

struct DecGeom {
  int H = 0, I = 0, heads = 0, kv = 0, D = 0, L = 0;
  float eps = 1e-5f, theta = 10000.f, scale = 1.f;
  bool conv = false;  // any LFM2 short-conv layer
};

int decoder_geom(dc_model *m, DecGeom &g) {
  double v;
  auto num = [&](const std::string &k, double dflt) { return cfg_num(m, k, v) ? v : dflt; };
  g.H = (int)num("hidden", 0), g.I = (int)num("intermediate", 0), g.heads = (int)num("heads", 0);
  g.kv = (int)num("kv_heads", 0), g.D = (int)num("head_dim", 0);
  g.eps = (float)num("eps", 1e-5), g.theta = (float)num("rope_theta", 10000.0);
  g.scale = (float)num("attn_scale", 1.0 / std::sqrt((double)(g.D > 0 ? g.D : 1)));
  DC_CHECK(g.H > 0 && g.I > 0 && g.heads > 0 && g.kv > 0 && g.D > 0 && g.heads % g.kv == 0, DC_EFORMAT,
           "decision.js: decoder config needs hidden, intermediate, heads, kv_heads, head_dim");
  const dcj::Value *lt = cfg(m, "layer_types");
  DC_CHECK(lt && lt->kind == dcj::Value::Arr && !lt->arr.empty(), DC_EFORMAT,
           "decision.js: decoder needs layer_types");
  g.L = (int)lt->arr.size();
  for (auto &t : lt->arr) {
    DC_CHECK(t.kind == dcj::Value::Str, DC_EFORMAT, "decision.js: layer_types must be strings");
    g.conv = g.conv || t.str == "conv";
  }
  return DC_OK;
}

// The LFM2 / attention backbone shared by D13BEngine.run (src/d1-3b-engine.ts:86-106) and D1OmniEngine.logits
// (src/omni-engine.ts:98-114): the embedding gather, the operator norm, per layer a short-conv or an attention
// mixer, the ffn norm and the SwiGLU MLP; on return x holds the residual stream and normed its final norm.
int lfm2_backbone(dc_model *m, const DecGeom &g, const int32_t *d_ids, const int32_t *d_pos, const int32_t *d_rng,
                  const int32_t *d_taps, int T) {
  dc_ctx *ctx = m->ctx;
  const int H = g.H, I = g.I, heads = g.heads, kv = g.kv, D = g.D;
  Q emb;
  RC(qw(m, "embed", emb, H));
  const dcj::Value *lt = cfg(m, "layer_types");
  const void *w0;
  RC(fw(m, "layers.0.operator_norm", w0, H));
  dc_prof_begin(ctx, DC_K_OTHER, 0, (double)T * H * 3);
  RC(ops_gather(ctx, d_ids, emb.codes, emb.scales, m->x, T, H, emb.bits, emb.N));
  dc_prof_end(ctx);
  dc_prof_begin(ctx, DC_K_NORM, 0, 4.0 * T * H);
  RC(ops_add_rmsnorm(ctx, m->x, nullptr, w0, m->normed, T, H, 0, g.eps));
  dc_prof_end(ctx);
  for (int i = 0; i < g.L; i++) {
    const std::string p = "layers." + std::to_string(i) + ".";
    Q w13, w2;
    RC(qw(m, p + "w13", w13, H));
    RC(qw(m, p + "w2", w2, I));
    DC_CHECK(w13.N == 2 * I && w2.N == H, DC_EFORMAT, "decision.js: layer %d: MLP shapes do not match the config",
             i);
    const void *fn, *nx;
    RC(fw(m, p + "ffn_norm", fn, H));
    RC(fw(m, i + 1 < g.L ? "layers." + std::to_string(i + 1) + ".operator_norm" : std::string("final_norm"), nx, H));
    if (lt->arr[i].str == "conv") {
      // LFM2 short convolution (src/d1-3b-engine.ts:89-92): in_proj to B | C | U, SHORT_CONV, out_proj
      Q win, wout;
      RC(qw(m, p + "in_proj", win, H));
      RC(qw(m, p + "out_proj", wout, H));
      DC_CHECK(win.N == 3 * H && wout.N == H, DC_EFORMAT, "decision.js: layer %d: conv shapes do not match", i);
      const void *wc;
      RC(fw(m, p + "conv", wc, (int64_t)3 * H));
      RC(matmul(m, m->normed, win, m->z, T));
      dc_prof_begin(ctx, DC_K_NORM, 0, 8.0 * T * H);
      RC(ops_short_conv(ctx, m->z, wc, d_taps, m->y, T, H));
      dc_prof_end(ctx);
      RC(matmul(m, m->y, wout, m->o, T));
    } else {
      Q wqkv, wo;
      RC(qw(m, p + "qkv", wqkv, H));
      RC(qw(m, p + "o_proj", wo, heads * D));
      DC_CHECK(wqkv.N == (heads + 2 * kv) * D && wo.N == H, DC_EFORMAT,
               "decision.js: layer %d: attention shapes do not match the config", i);
      const void *qn, *kn;
      RC(fw(m, p + "q_norm", qn, D));
      RC(fw(m, p + "k_norm", kn, D));
      RC(matmul(m, m->normed, wqkv, m->z, T));
      dc_prof_begin(ctx, DC_K_NORM, 0, 4.0 * T * (heads + 2 * kv) * D);
      RC(ops_qkv_norm_rope(ctx, m->z, qn, kn, d_pos, T, heads, kv, D, g.eps, g.theta, 0));
      dc_prof_end(ctx);
      dc_prof_begin(ctx, DC_K_ATTN, m->attn_keys * 4.0 * heads * D, 0);
      RC(attn_launch(ctx, m->z, d_rng, m->y, T, heads, kv, D, g.scale));
      dc_prof_end(ctx);
      RC(matmul(m, m->y, wo, m->o, T));
    }
    dc_prof_begin(ctx, DC_K_NORM, 0, 8.0 * T * H);
    RC(ops_add_rmsnorm(ctx, m->x, m->o, fn, m->normed, T, H, 1, g.eps));
    dc_prof_end(ctx);
    RC(gated(m, m->normed, w13, m->z, m->h, T, DC_ACT_SILU));
    RC(matmul(m, m->h, w2, m->o, T));
    dc_prof_begin(ctx, DC_K_NORM, 0, 8.0 * T * H);
    RC(ops_add_rmsnorm(ctx, m->x, m->o, nx, m->normed, T, H, 1, g.eps));
    dc_prof_end(ctx);
  }
  return DC_OK;
}

// D13BEngine.run's GPU part on device-resident inputs (src/d1-3b-engine.ts:86-108).
int decoder_core(dc_model *m, const DecGeom &g, const int32_t *d_ids, const int32_t *d_pos, const int32_t *d_rng,
                 int T, const int32_t *d_leaves, const int32_t *d_leaf_ids, int Lv, int nIds, float *d_out) {
  dc_ctx *ctx = m->ctx;
  const int H = g.H, I = g.I, heads = g.heads, kv = g.kv, D = g.D;
  Q emb;
  RC(qw(m, "embed", emb, H));
  RC(ensure(m, T, H, std::max(std::max((heads + 2 * kv) * D, 2 * I), g.conv ? 3 * H : 0),
            std::max(heads * D, g.conv ? H : 0), I));
  int32_t *d_taps = nullptr;
  if (g.conv) {  // the short convolution's taps, from the key ranges (src/d1-3b-engine.ts:53-62)
    RC(ensure_dmeta(m, (size_t)T * 16));
    d_taps = (int32_t *)m->dmeta;
    dc_prof_begin(ctx, DC_K_OTHER, 0, (double)T * 32);
    RC(ops_conv_taps(ctx, d_rng, d_taps, T));
    dc_prof_end(ctx);
  }
  RC(lfm2_backbone(m, g, d_ids, d_pos, d_rng, d_taps, T));
  const void *fnorm;
  RC(fw(m, "final_norm", fnorm, H));
  dc_prof_begin(ctx, DC_K_OTHER, 0, 0);
  RC(ops_leaf_logits(ctx, m->x, d_leaves, fnorm, d_leaf_ids, emb.codes, emb.scales, d_out, Lv, H, nIds, emb.bits,
                     g.eps, T, emb.N));
  dc_prof_end(ctx);
  return DC_OK;
}

}  // namespace

extern "C" int dc_forward_encoder(dc_model *m, const int32_t *h_ids, const int32_t *h_bounds, int T, int S,
                                  float *h_out) {
  DC_CHECK(m && h_ids && h_bounds && h_out && T > 0 && S > 0, DC_EINVAL, "decision.js: encoder: bad arguments");
  RC(dc_use(m->ctx));
  EncGeom g;
  RC(encoder_geom(m, g));
  Q emb;
  RC(qw(m, "embed", emb, g.H));
  for (int t = 0; t < T; t++)
    DC_CHECK(h_ids[t] >= 0 && h_ids[t] < emb.N, DC_EINVAL, "decision.js: token id %d out of range", h_ids[t]);
  double keys = 0;
  for (int s = 0; s < S; s++) {
    const int a = h_bounds[2 * s], b = h_bounds[2 * s + 1];
    DC_CHECK(a >= 0 && b > a && b <= T && (s == 0 || a >= h_bounds[2 * s - 1]), DC_EINVAL,
             "decision.js: encoder: sequence %d has bounds [%d, %d)", s, a, b);
    keys += (double)(b - a) * (b - a);
  }
  m->attn_keys = keys;
  std::vector<int32_t *> d;
  RC(upload_meta(m, {{h_ids, 4 * (size_t)T}, {h_bounds, 8 * (size_t)S}}, d));
  RC(grow(m->out, m->out_cap, (size_t)S * g.N, 4));
  RC(run_graphed(m, m->genc, pass_key(m, 0, {(uintptr_t)T, (uintptr_t)S, (uintptr_t)d[0], (uintptr_t)d[1]}),
                 [&] { return encoder_core(m, g, d[0], d[1], T, S, m->out); }));
  return download_out(m, h_out, (size_t)S * g.N);
}

extern "C" int dc_forward_encoder_device(dc_model *m, const int32_t *d_ids, const int32_t *d_bounds, int T, int S,
                                         float *d_out) {
  DC_CHECK(m && d_ids && d_bounds && d_out && T > 0 && S > 0, DC_EINVAL, "decision.js: encoder: bad arguments");
  RC(dc_use(m->ctx));
  EncGeom g;
  RC(encoder_geom(m, g));
  m->attn_keys = 0;  // unknown without reading the bounds back
  return run_graphed(m, m->genc,
                     pass_key(m, 0, {(uintptr_t)T, (uintptr_t)S, (uintptr_t)d_ids, (uintptr_t)d_bounds, (uintptr_t)d_out}),
                     [&] { return encoder_core(m, g, d_ids, d_bounds, T, S, d_out); });
}

extern "C" int dc_forward_decoder(dc_model *m, const int32_t *h_ids, const int32_t *h_pos, const int32_t *h_rng,
                                  int T, const int32_t *h_leaves, const int32_t *h_leaf_ids, int Lv, int nIds,
                                  float *h_out) {
  DC_CHECK(m && h_ids && h_pos && h_rng && h_leaves && h_leaf_ids && h_out && T > 0 && Lv > 0 && nIds > 0,
           DC_EINVAL, "decision.js: decoder: bad arguments");
  RC(dc_use(m->ctx));
  DecGeom g;
  RC(decoder_geom(m, g));
  Q emb;
  RC(qw(m, "embed", emb, g.H));
  double keys = 0;
  for (int t = 0; t < T; t++) {
    DC_CHECK(h_ids[t] >= 0 && h_ids[t] < emb.N, DC_EINVAL, "decision.js: token id %d out of range", h_ids[t]);
    const int *r = h_rng + 4 * t;
    DC_CHECK(r[0] >= 0 && r[1] <= T && r[2] >= 0 && r[3] <= T && (r[1] > r[0] || r[3] > r[2]), DC_EINVAL,
             "decision.js: token %d has no keys or keys out of range", t);
    keys += std::max(0, r[1] - r[0]) + std::max(0, r[3] - r[2]);
  }
  for (int l = 0; l < Lv; l++) DC_CHECK(h_leaves[l] >= 0 && h_leaves[l] < T, DC_EINVAL, "decision.js: bad leaf row");
  for (long j = 0; j < (long)Lv * nIds; j++)
    DC_CHECK(h_leaf_ids[j] >= 0 && h_leaf_ids[j] < emb.N, DC_EINVAL, "decision.js: readout id out of range");
  m->attn_keys = keys;
  std::vector<int32_t *> d;
  RC(upload_meta(m, {{h_ids, 4 * (size_t)T}, {h_pos, 4 * (size_t)T}, {h_rng, 16 * (size_t)T},
                     {h_leaves, 4 * (size_t)Lv}, {h_leaf_ids, 4 * (size_t)Lv * nIds}},
                 d));
  RC(grow(m->out, m->out_cap, (size_t)Lv * nIds, 4));
  RC(run_graphed(m, m->gdec,
                 pass_key(m, 1, {(uintptr_t)T, (uintptr_t)Lv, (uintptr_t)nIds, (uintptr_t)d[0], (uintptr_t)d[1],
                                 (uintptr_t)d[2], (uintptr_t)d[3], (uintptr_t)d[4]}),
                 [&] { return decoder_core(m, g, d[0], d[1], d[2], T, d[3], d[4], Lv, nIds, m->out); }));
  return download_out(m, h_out, (size_t)Lv * nIds);
}

extern "C" int dc_forward_decoder_device(dc_model *m, const int32_t *d_ids, const int32_t *d_pos,
                                         const int32_t *d_rng, int T, const int32_t *d_leaves,
                                         const int32_t *d_leaf_ids, int Lv, int nIds, float *d_out) {
  DC_CHECK(m && d_ids && d_pos && d_rng && d_leaves && d_leaf_ids && d_out && T > 0 && Lv > 0 && nIds > 0,
           DC_EINVAL, "decision.js: decoder: bad arguments");
  RC(dc_use(m->ctx));
  DecGeom g;
  RC(decoder_geom(m, g));
  m->attn_keys = 0;
  return run_graphed(m, m->gdec,
                     pass_key(m, 1, {(uintptr_t)T, (uintptr_t)Lv, (uintptr_t)nIds, (uintptr_t)d_ids, (uintptr_t)d_pos,
                                     (uintptr_t)d_rng, (uintptr_t)d_leaves, (uintptr_t)d_leaf_ids, (uintptr_t)d_out}),
                     [&] { return decoder_core(m, g, d_ids, d_pos, d_rng, T, d_leaves, d_leaf_ids, Lv, nIds, d_out); });
}

namespace {

// d3-lite's configuration (scripts/export-d3.py:55-61), read once per call from the manifest.
struct D3Geom {
  int H = 0, I = 0, heads = 0, kv = 0, D = 0, rot = 0, LH = 0, rows = 0, L = 0, codes = 0;
  float eps = 1e-6f, theta = 10000.f;
  const float *R = nullptr;  // the code readout [codes, H] f32
};

int d3_geom(dc_model *m, D3Geom &g) {
  double v;
  auto num = [&](const std::string &k, double dflt) { return cfg_num(m, k, v) ? v : dflt; };
  g.H = (int)num("hidden", 0), g.I = (int)num("intermediate", 0), g.heads = (int)num("heads", 0);
  g.kv = (int)num("kv_heads", 0), g.D = (int)num("head_dim", 0), g.rot = (int)num("rotary_dim", g.D);
  g.LH = (int)num("linear_heads", 0), g.rows = (int)num("linear_rows", 0);
  g.eps = (float)num("eps", 1e-6), g.theta = (float)num("rope_theta", 10000.0);
  DC_CHECK(g.H > 0 && g.I > 0 && g.heads > 0 && g.kv > 0 && g.heads % g.kv == 0 && g.D > 0, DC_EFORMAT,
           "decision.js: d3 config needs hidden, intermediate, heads, kv_heads, head_dim");
  DC_CHECK(num("linear_key_dim", 128) == 128 && num("linear_value_dim", 128) == 128 && num("conv_kernel", 4) == 4,
           DC_EFORMAT, "decision.js: d3 linear attention takes 128-wide key and value heads and a 4-tap conv");
  const dcj::Value *lt = cfg(m, "layer_types");
  DC_CHECK(lt && lt->kind == dcj::Value::Arr && !lt->arr.empty(), DC_EFORMAT, "decision.js: d3 needs layer_types");
  g.L = (int)lt->arr.size();
  bool linear = false;
  for (auto &t : lt->arr) {
    DC_CHECK(t.kind == dcj::Value::Str && (t.str == "linear_attention" || t.str == "full_attention"), DC_EFORMAT,
             "decision.js: d3 layer types are linear_attention or full_attention");
    linear = linear || t.str == "linear_attention";
  }
  DC_CHECK(!linear || (g.LH > 0 && g.rows >= 4 * g.LH * 128 + 2 * g.LH && g.rows % 8 == 0), DC_EFORMAT,
           "decision.js: d3 linear_rows %d cannot hold q|k|v|z|b|a of %d heads", g.rows, g.LH);
  auto it = m->tensors.find("readout");
  DC_CHECK(it != m->tensors.end() && it->second.dtype == 32 && it->second.cols == g.H, DC_EFORMAT,
           "decision.js: d3 needs an f32 readout [codes, %d]", g.H);
  g.codes = (int)it->second.rows;
  g.R = reinterpret_cast<const float *>(m->base + it->second.offset);
  return DC_OK;
}

// D3Engine.logits's GPU part on device-resident inputs (src/d3-engine.ts:103-131).
int d3_core(dc_model *m, const D3Geom &g, const int32_t *d_ids, const int32_t *d_pos, const int32_t *d_rng, int T,
            const uint32_t *d_spans, int nseq, const int32_t *d_pairs, int P, float *d_out) {
  dc_ctx *ctx = m->ctx;
  const int H = g.H, I = g.I, heads = g.heads, kv = g.kv, D = g.D, LH = g.LH;
  const long astride = (long)(2 * heads + 2 * kv) * D;  // q | k | v | gate heads
  Q emb;
  RC(qw(m, "embed", emb, H));
  RC(ensure(m, T, H, std::max(std::max(g.rows, 2 * I), (int)astride), std::max(LH * 128, heads * D), I));
  const dcj::Value *lt = cfg(m, "layer_types");
  dc_prof_begin(ctx, DC_K_OTHER, 0, (double)T * H * 3);
  RC(ops_gather(ctx, d_ids, emb.codes, emb.scales, m->x, T, H, emb.bits, emb.N));
  dc_prof_end(ctx);
  for (int i = 0; i < g.L; i++) {
    const std::string p = "layers." + std::to_string(i) + ".";
    const void *in_n, *post_n;
    RC(fw(m, p + "input_norm", in_n, H));
    RC(fw(m, p + "post_norm", post_n, H));
    // the input norm adds the previous layer's MLP output
    dc_prof_begin(ctx, DC_K_NORM, 0, (i > 0 ? 8.0 : 4.0) * T * H);
    RC(ops_add_rmsnorm(ctx, m->x, i > 0 ? m->o : nullptr, in_n, m->normed, T, H, i > 0 ? 1 : 0, g.eps));
    dc_prof_end(ctx);
    if (lt->arr[i].str == "linear_attention") {
      Q win, wout;
      RC(qw(m, p + "in", win, H));
      RC(qw(m, p + "out", wout, LH * 128));
      DC_CHECK(win.N == g.rows && wout.N == H, DC_EFORMAT, "decision.js: layer %d: linear shapes do not match", i);
      const void *wc, *alog, *dtb, *gw;
      RC(fw(m, p + "conv", wc, (int64_t)3 * LH * 128 * 4));
      RC(fw(m, p + "A_log", alog, LH));
      RC(fw(m, p + "dt_bias", dtb, LH));
      RC(fw(m, p + "gnorm", gw, 128));
      RC(matmul(m, m->normed, win, m->z, T));
      dc_prof_begin(ctx, DC_K_OTHER, 0, 2.0 * T * g.rows + 2.0 * T * LH * 128);
      RC(ops_gdn(ctx, m->z, g.rows, 3L * LH * 128, LH, wc, alog, dtb, gw, d_spans, nseq, g.eps, m->y, T));
      dc_prof_end(ctx);
      RC(matmul(m, m->y, wout, m->o, T));
    } else {
      Q wqkvg, wo;
      RC(qw(m, p + "qkvg", wqkvg, H));
      RC(qw(m, p + "o", wo, heads * D));
      DC_CHECK(wqkvg.N == astride && wo.N == H, DC_EFORMAT, "decision.js: layer %d: attention shapes do not match",
               i);
      const void *qn, *kn;
      RC(fw(m, p + "q_norm", qn, D));
      RC(fw(m, p + "k_norm", kn, D));
      RC(matmul(m, m->normed, wqkvg, m->z, T));
      dc_prof_begin(ctx, DC_K_NORM, 0, 4.0 * T * (heads + kv) * D);
      RC(ops_qk_rope(ctx, m->z, qn, kn, d_pos, T, heads, kv, D, astride, g.rot, 1, g.eps, g.theta));
      dc_prof_end(ctx);
      dc_prof_begin(ctx, DC_K_ATTN, m->attn_keys * 4.0 * heads * D, 0);
      RC(attn_launch_ex(ctx, m->z, d_rng, m->y, T, heads, kv, D, 1.0f / std::sqrt((float)D), -1, astride, 1));
      dc_prof_end(ctx);
      RC(matmul(m, m->y, wo, m->o, T));
    }
    Q w13, w2;
    RC(qw(m, p + "w13", w13, H));
    RC(qw(m, p + "w2", w2, I));
    DC_CHECK(w13.N == 2 * I && w2.N == H, DC_EFORMAT, "decision.js: layer %d: MLP shapes do not match", i);
    dc_prof_begin(ctx, DC_K_NORM, 0, 8.0 * T * H);
    RC(ops_add_rmsnorm(ctx, m->x, m->o, post_n, m->normed, T, H, 1, g.eps));
    dc_prof_end(ctx);
    RC(gated(m, m->normed, w13, m->z, m->h, T, DC_ACT_SILU));
    RC(matmul(m, m->h, w2, m->o, T));
  }
  const void *fnorm;
  RC(fw(m, "final_norm", fnorm, H));
  dc_prof_begin(ctx, DC_K_NORM, 0, 8.0 * T * H);
  RC(ops_add_rmsnorm(ctx, m->x, m->o, fnorm, m->normed, T, H, 1, g.eps));
  dc_prof_end(ctx);
  dc_prof_begin(ctx, DC_K_OTHER, 0, 0);
  RC(ops_readout(ctx, m->normed, g.R, d_pairs, d_out, P, H, T, g.codes));
  dc_prof_end(ctx);
  return DC_OK;
}

}  // namespace

extern "C" int dc_forward_d3(dc_model *m, const int32_t *h_ids, const int32_t *h_pos, const int32_t *h_rng, int T,
                             const uint32_t *h_spans, int nseq, const int32_t *h_pairs, int P, float *h_out) {
  DC_CHECK(m && h_ids && h_pos && h_rng && h_spans && h_pairs && h_out && T > 0 && nseq > 0 && P > 0, DC_EINVAL,
           "decision.js: d3: bad arguments");
  RC(dc_use(m->ctx));
  D3Geom g;
  RC(d3_geom(m, g));
  Q emb;
  RC(qw(m, "embed", emb, g.H));
  double keys = 0;
  for (int t = 0; t < T; t++) {
    DC_CHECK(h_ids[t] >= 0 && h_ids[t] < emb.N, DC_EINVAL, "decision.js: token id %d out of range", h_ids[t]);
    const int *r = h_rng + 4 * t;
    DC_CHECK(r[0] >= 0 && r[1] <= T && r[2] >= 0 && r[3] <= T && (r[1] > r[0] || r[3] > r[2]), DC_EINVAL,
             "decision.js: token %d has no keys or keys out of range", t);
    keys += std::max(0, r[1] - r[0]) + std::max(0, r[3] - r[2]);
  }
  for (int q = 0; q < nseq; q++) {
    const uint32_t *sp = h_spans + 4 * q;
    DC_CHECK((uint64_t)sp[0] + (sp[1] & 0x7fffffffu) <= (uint64_t)T && (uint64_t)sp[2] + sp[3] <= (uint64_t)T,
             DC_EINVAL, "decision.js: d3: sequence %d spans past the %d tokens", q, T);
  }
  for (int k = 0; k < P; k++)
    DC_CHECK(h_pairs[2 * k] >= 0 && h_pairs[2 * k] < T && h_pairs[2 * k + 1] >= 0 && h_pairs[2 * k + 1] < g.codes,
             DC_EINVAL, "decision.js: d3: readout pair %d out of range", k);
  m->attn_keys = keys;
  std::vector<int32_t *> d;
  RC(upload_meta(m, {{h_ids, 4 * (size_t)T}, {h_pos, 4 * (size_t)T}, {h_rng, 16 * (size_t)T},
                     {h_spans, 16 * (size_t)nseq}, {h_pairs, 8 * (size_t)P}},
                 d));
  RC(grow(m->out, m->out_cap, (size_t)P, 4));
  RC(run_graphed(m, m->gd3,
                 pass_key(m, 2, {(uintptr_t)T, (uintptr_t)nseq, (uintptr_t)P, (uintptr_t)d[0], (uintptr_t)d[1],
                                 (uintptr_t)d[2], (uintptr_t)d[3], (uintptr_t)d[4]}),
                 [&] {
                   return d3_core(m, g, d[0], d[1], d[2], T, reinterpret_cast<const uint32_t *>(d[3]), nseq, d[4], P,
                                  m->out);
                 }));
  return download_out(m, h_out, (size_t)P);
}

namespace {

// An f16 tensor of exactly n values (a bias, a norm weight).
int fw_opt(dc_model *m, const std::string &name, const void *&p, int64_t n) { return fw(m, name, p, n); }

// The decision head of d1-omni and Laya (src/omni-engine.ts:115-131, src/laya-engine.ts:112-130) over the
// encoder's final-normed rows in `normed`: the question type embedding, the pre-norm transformer head (LayerNorms
// with biases, biased projections, 64-wide heads over each whole sequence, ReLU FFN), the scorer's norm, the option
// markers' rows, fc + bias + GELU, and the score.
int decision_head(dc_model *m, int H, const int32_t *d_rng, int T, const int32_t *d_qtype, const int32_t *d_markers,
                  int M, float *d_out) {
  dc_ctx *ctx = m->ctx;
  double v;
  const int hl = cfg_num(m, "head_layers", v) ? (int)v : 0, hh = cfg_num(m, "head_heads", v) ? (int)v : 0;
  const int ff = cfg_num(m, "head_ff", v) ? (int)v : 0;
  const float ln_eps = cfg_num(m, "ln_eps", v) ? (float)v : 1e-5f;
  DC_CHECK(hl > 0 && hh > 0 && H == 64 * hh && ff > 0 && ff % 8 == 0, DC_EFORMAT,
           "decision.js: the decision head needs head_layers, head_heads of 64 dims (hidden %d) and head_ff", H);
  auto it = m->tensors.find("head.type_emb");
  DC_CHECK(it != m->tensors.end() && it->second.dtype == 16 && it->second.cols == H, DC_EFORMAT,
           "decision.js: the decision head needs head.type_emb [types, %d] f16", H);
  dc_prof_begin(ctx, DC_K_OTHER, 0, 6.0 * T * H);
  RC(ops_add_rows(ctx, m->normed, d_qtype, m->base + it->second.offset, m->x, T, H, (int)it->second.rows));
  dc_prof_end(ctx);
  auto ln = [&](__half *X, int rows, bool add, const std::string &name, __half *O) -> int {
    const void *w, *b;
    RC(fw(m, name, w, H));
    RC(fw(m, name + "_bias", b, H));
    dc_prof_begin(ctx, DC_K_NORM, 0, (add ? 6.0 : 4.0) * rows * H);
    RC(ops_add_layernorm(ctx, X, add ? m->o : nullptr, w, b, O, rows, H, add ? 1 : 0, ln_eps));
    dc_prof_end(ctx);
    return DC_OK;
  };
  auto bias = [&](__half *Y, int rows, const std::string &name, int n, int act) -> int {
    const void *b;
    RC(fw(m, name, b, n));
    dc_prof_begin(ctx, DC_K_OTHER, 0, 4.0 * rows * n);
    RC(ops_bias_act(ctx, Y, b, rows, n, act));
    dc_prof_end(ctx);
    return DC_OK;
  };
  for (int i = 0; i < hl; i++) {
    const std::string p = "head." + std::to_string(i) + ".";
    Q win, wout, w1, w2;
    RC(qw(m, p + "in_proj", win, H));
    RC(qw(m, p + "out_proj", wout, H));
    RC(qw(m, p + "linear1", w1, H));
    RC(qw(m, p + "linear2", w2, ff));
    DC_CHECK(win.N == 3 * H && wout.N == H && w1.N == ff && w2.N == H, DC_EFORMAT,
             "decision.js: head layer %d: shapes do not match the config", i);
    RC(ln(m->x, T, i > 0, p + "norm1", m->normed));  // i > 0: adds the previous layer's FFN output
    RC(matmul(m, m->normed, win, m->z, T));
    RC(bias(m->z, T, p + "in_proj_bias", 3 * H, 0));
    dc_prof_begin(ctx, DC_K_ATTN, m->attn_keys * 4.0 * hh * 64, 0);
    RC(attn_launch(ctx, m->z, d_rng, m->y, T, hh, hh, 64, 0.125f));
    dc_prof_end(ctx);
    RC(matmul(m, m->y, wout, m->o, T));
    RC(bias(m->o, T, p + "out_proj_bias", H, 0));
    RC(ln(m->x, T, true, p + "norm2", m->normed));
    RC(matmul(m, m->normed, w1, m->h, T));
    RC(bias(m->h, T, p + "linear1_bias", ff, 1));
    RC(matmul(m, m->h, w2, m->o, T));
    RC(bias(m->o, T, p + "linear2_bias", H, 0));
  }
  RC(ln(m->x, T, true, "scorer.norm", m->normed));
  // the markers' rows into y, the scorer's fc into o (M <= T rows each)
  Q fc;
  RC(qw(m, "scorer.fc", fc, H));
  DC_CHECK(fc.N == H, DC_EFORMAT, "decision.js: scorer.fc must be [%d, %d]", H, H);
  dc_prof_begin(ctx, DC_K_OTHER, 0, 4.0 * M * H);
  RC(ops_gather_rows(ctx, m->normed, d_markers, m->y, M, H, T));
  dc_prof_end(ctx);
  RC(matmul(m, m->y, fc, m->o, M));
  RC(bias(m->o, M, "scorer.fc_bias", H, 2));
  const void *ws, *bs;
  RC(fw(m, "scorer.out", ws, H));
  RC(fw(m, "scorer.out_bias", bs, 2));
  dc_prof_begin(ctx, DC_K_OTHER, 0, 2.0 * M * H);
  RC(ops_score(ctx, m->o, ws, bs, d_out, M, H));
  dc_prof_end(ctx);
  return DC_OK;
}

// D1OmniEngine.logits's GPU part (src/omni-engine.ts:98-131) on device-resident inputs: the backbone, then the head.
int omni_core(dc_model *m, const DecGeom &g, const int32_t *d_ids, const int32_t *d_pos, const int32_t *d_rng,
              const int32_t *d_taps, int T, const int32_t *d_qtype, const int32_t *d_markers, int M, float *d_out) {
  double v;
  const int ff = cfg_num(m, "head_ff", v) ? (int)v : 0;
  RC(ensure(m, T, g.H, std::max(std::max((g.heads + 2 * g.kv) * g.D, 2 * g.I), 3 * g.H),
            std::max(g.heads * g.D, g.H), std::max(g.I, ff)));
  RC(lfm2_backbone(m, g, d_ids, d_pos, d_rng, d_taps, T));
  return decision_head(m, g.H, d_rng, T, d_qtype, d_markers, M, d_out);
}

// Laya's configuration (scripts/export-laya.py:55-62).
struct LayaGeom {
  int H = 0, I = 0, heads = 0, L = 0, ff = 0;
  float eps = 1e-5f, theta_full = 160000.f, theta_slide = 10000.f;
};

int laya_geom(dc_model *m, LayaGeom &g) {
  double v;
  auto num = [&](const std::string &k, double dflt) { return cfg_num(m, k, v) ? v : dflt; };
  g.H = (int)num("hidden", 0), g.I = (int)num("intermediate", 0), g.heads = (int)num("heads", 0);
  g.eps = (float)num("eps", 1e-5), g.ff = (int)num("head_ff", 0);
  g.theta_full = (float)num("rope_theta.full_attention", 160000.0);
  g.theta_slide = (float)num("rope_theta.sliding_attention", 10000.0);
  DC_CHECK(g.H > 0 && g.I > 0 && g.heads > 0 && g.H == 64 * g.heads, DC_EFORMAT,
           "decision.js: Laya config needs hidden, intermediate and heads of 64 dims");
  const dcj::Value *lt = cfg(m, "layer_types");
  DC_CHECK(lt && lt->kind == dcj::Value::Arr && !lt->arr.empty(), DC_EFORMAT, "decision.js: Laya needs layer_types");
  g.L = (int)lt->arr.size();
  for (auto &t : lt->arr)
    DC_CHECK(t.kind == dcj::Value::Str && (t.str == "full_attention" || t.str == "sliding_attention"), DC_EFORMAT,
             "decision.js: Laya layer types are full_attention or sliding_attention");
  return DC_OK;
}

// LayaEngine.logits's GPU part (src/laya-engine.ts:86-131): the ModernBERT encoder (bias-free LayerNorms, RoPE
// attention over the whole sequence on full layers and a window on the others, GELU-gated MLP), then the head.
int laya_core(dc_model *m, const LayaGeom &g, const int32_t *d_ids, const int32_t *d_pos, const int32_t *d_rng,
              const int32_t *d_win, int T, const int32_t *d_qtype, const int32_t *d_markers, int M, float *d_out) {
  dc_ctx *ctx = m->ctx;
  const int H = g.H, I = g.I, heads = g.heads;
  Q emb;
  RC(qw(m, "embed", emb, H));
  RC(ensure(m, T, H, std::max(2 * I, 3 * H), H, std::max(I, g.ff)));
  const dcj::Value *lt = cfg(m, "layer_types");
  auto ln = [&](__half *X, bool add, const std::string &name, __half *O) -> int {
    const void *w;
    RC(fw(m, name, w, H));
    dc_prof_begin(ctx, DC_K_NORM, 0, (add ? 6.0 : 4.0) * T * H);
    RC(ops_add_layernorm(ctx, X, add ? m->o : nullptr, w, nullptr, O, T, H, add ? 1 : 0, g.eps));
    dc_prof_end(ctx);
    return DC_OK;
  };
  dc_prof_begin(ctx, DC_K_OTHER, 0, (double)T * H * 3);
  RC(ops_gather(ctx, d_ids, emb.codes, emb.scales, m->normed, T, H, emb.bits, emb.N));
  dc_prof_end(ctx);
  RC(ln(m->normed, false, "embed_norm", m->x));
  for (int i = 0; i < g.L; i++) {
    const std::string p = "layers." + std::to_string(i) + ".";
    const bool global = lt->arr[i].str == "full_attention";
    Q wqkv, wo, wi, wo2;
    RC(qw(m, p + "qkv", wqkv, H));
    RC(qw(m, p + "o", wo, H));
    RC(qw(m, p + "wi", wi, H));
    RC(qw(m, p + "wo", wo2, I));
    DC_CHECK(wqkv.N == 3 * H && wo.N == H && wi.N == 2 * I && wo2.N == H, DC_EFORMAT,
             "decision.js: Laya layer %d: shapes do not match the config", i);
    const __half *attn_in = m->x;
    if (m->tensors.count(p + "attn_norm")) {  // layer 0 has none; the others add the previous MLP output first
      RC(ln(m->x, true, p + "attn_norm", m->normed));
      attn_in = m->normed;
    }
    RC(matmul(m, attn_in, wqkv, m->z, T));
    dc_prof_begin(ctx, DC_K_NORM, 0, 8.0 * T * heads * 64);
    RC(ops_qk_rope(ctx, m->z, nullptr, nullptr, d_pos, T, heads, heads, 64, 3L * H, 64, 0, 0.f,
                   global ? g.theta_full : g.theta_slide));
    dc_prof_end(ctx);
    dc_prof_begin(ctx, DC_K_ATTN, m->attn_keys * 4.0 * heads * 64, 0);
    RC(attn_launch(ctx, m->z, global ? d_rng : d_win, m->y, T, heads, heads, 64, 0.125f));
    dc_prof_end(ctx);
    RC(matmul(m, m->y, wo, m->o, T));
    RC(ln(m->x, true, p + "mlp_norm", m->normed));
    RC(matmul(m, m->normed, wi, m->z, T));
    dc_prof_begin(ctx, DC_K_OTHER, 0, 6.0 * T * I);
    RC(ops_glu(ctx, m->z, m->h, T, I, DC_ACT_GELU_ERF, 0));
    dc_prof_end(ctx);
    RC(matmul(m, m->h, wo2, m->o, T));
  }
  RC(ln(m->x, true, "final_norm", m->normed));
  return decision_head(m, H, d_rng, T, d_qtype, d_markers, M, d_out);
}

}  // namespace

extern "C" int dc_forward_omni(dc_model *m, const int32_t *h_ids, const int32_t *h_pos, const int32_t *h_rng,
                               const int32_t *h_taps, int T, const int32_t *h_qtype, const int32_t *h_markers, int M,
                               float *h_out) {
  DC_CHECK(m && h_ids && h_pos && h_rng && h_taps && h_qtype && h_markers && h_out && T > 0 && M > 0 && M <= T,
           DC_EINVAL, "decision.js: d1-omni: bad arguments");
  RC(dc_use(m->ctx));
  DecGeom g;
  RC(decoder_geom(m, g));
  Q emb;
  RC(qw(m, "embed", emb, g.H));
  double keys = 0;
  for (int t = 0; t < T; t++) {
    DC_CHECK(h_ids[t] >= 0 && h_ids[t] < emb.N, DC_EINVAL, "decision.js: token id %d out of range", h_ids[t]);
    const int *r = h_rng + 4 * t;
    DC_CHECK(r[0] >= 0 && r[1] <= T && r[2] >= 0 && r[3] <= T && (r[1] > r[0] || r[3] > r[2]), DC_EINVAL,
             "decision.js: token %d has no keys or keys out of range", t);
    for (int j = 0; j < 3; j++)
      DC_CHECK(h_taps[4 * t + j] >= -1 && h_taps[4 * t + j] < T, DC_EINVAL, "decision.js: token %d: bad conv tap", t);
    keys += std::max(0, r[1] - r[0]) + std::max(0, r[3] - r[2]);
  }
  for (int k = 0; k < M; k++)
    DC_CHECK(h_markers[k] >= 0 && h_markers[k] < T, DC_EINVAL, "decision.js: d1-omni: marker %d out of range", k);
  m->attn_keys = keys;
  std::vector<int32_t *> d;
  RC(upload_meta(m, {{h_ids, 4 * (size_t)T}, {h_pos, 4 * (size_t)T}, {h_rng, 16 * (size_t)T},
                     {h_taps, 16 * (size_t)T}, {h_qtype, 4 * (size_t)T}, {h_markers, 4 * (size_t)M}},
                 d));
  RC(grow(m->out, m->out_cap, (size_t)M, 4));
  RC(run_graphed(m, m->gomni,
                 pass_key(m, 3, {(uintptr_t)T, (uintptr_t)M, (uintptr_t)d[0], (uintptr_t)d[1], (uintptr_t)d[2],
                                 (uintptr_t)d[3], (uintptr_t)d[4], (uintptr_t)d[5]}),
                 [&] { return omni_core(m, g, d[0], d[1], d[2], d[3], T, d[4], d[5], M, m->out); }));
  return download_out(m, h_out, (size_t)M);
}

extern "C" int dc_forward_laya(dc_model *m, const int32_t *h_ids, const int32_t *h_pos, const int32_t *h_rng,
                               const int32_t *h_win, int T, const int32_t *h_qtype, const int32_t *h_markers, int M,
                               float *h_out) {
  DC_CHECK(m && h_ids && h_pos && h_rng && h_win && h_qtype && h_markers && h_out && T > 0 && M > 0 && M <= T,
           DC_EINVAL, "decision.js: laya: bad arguments");
  RC(dc_use(m->ctx));
  LayaGeom g;
  RC(laya_geom(m, g));
  Q emb;
  RC(qw(m, "embed", emb, g.H));
  double keys = 0;
  for (int t = 0; t < T; t++) {
    DC_CHECK(h_ids[t] >= 0 && h_ids[t] < emb.N, DC_EINVAL, "decision.js: token id %d out of range", h_ids[t]);
    for (const int32_t *r : {h_rng + 4 * t, h_win + 4 * t})
      DC_CHECK(r[0] >= 0 && r[1] <= T && r[2] >= 0 && r[3] <= T && (r[1] > r[0] || r[3] > r[2]), DC_EINVAL,
               "decision.js: token %d has no keys or keys out of range", t);
    keys += std::max(0, h_rng[4 * t + 1] - h_rng[4 * t]);
  }
  for (int k = 0; k < M; k++)
    DC_CHECK(h_markers[k] >= 0 && h_markers[k] < T, DC_EINVAL, "decision.js: laya: marker %d out of range", k);
  m->attn_keys = keys;
  std::vector<int32_t *> d;
  RC(upload_meta(m, {{h_ids, 4 * (size_t)T}, {h_pos, 4 * (size_t)T}, {h_rng, 16 * (size_t)T},
                     {h_win, 16 * (size_t)T}, {h_qtype, 4 * (size_t)T}, {h_markers, 4 * (size_t)M}},
                 d));
  RC(grow(m->out, m->out_cap, (size_t)M, 4));
  RC(run_graphed(m, m->glaya,
                 pass_key(m, 4, {(uintptr_t)T, (uintptr_t)M, (uintptr_t)d[0], (uintptr_t)d[1], (uintptr_t)d[2],
                                 (uintptr_t)d[3], (uintptr_t)d[4], (uintptr_t)d[5]}),
                 [&] { return laya_core(m, g, d[0], d[1], d[2], d[3], T, d[4], d[5], M, m->out); }));
  return download_out(m, h_out, (size_t)M);
}

int ops_eg2_head(dc_ctx *, const Eg2HeadW &, const float *, const float *, const float *, const int *, int, int, int,
                 int, float *);

namespace {
// An f32 head tensor of exactly rows x cols values.
int head_t(dc_model *m, const char *name, int64_t rows, int64_t cols, const float *&p) {
  auto it = m->tensors.find(name);
  DC_CHECK(it != m->tensors.end(), DC_EFORMAT, "decision.js: the model has no head tensor %s", name);
  const dc_tensor &t = it->second;
  DC_CHECK(t.dtype == 32 && t.bytes == 4 * rows * cols && t.offset % 16 == 0, DC_EFORMAT,
           "decision.js: head tensor %s must be f32 with %lld x %lld values", name, (long long)rows, (long long)cols);
  p = reinterpret_cast<const float *>(m->base + t.offset);
  return DC_OK;
}
}  // namespace

extern "C" int dc_eg2_head(dc_model *m, const float *d_S, int nS, const float *d_Q, int nQ, const float *d_O, int nO,
                           const int32_t *d_items, int n_items, float *d_logits) {
  DC_CHECK(m && d_S && d_Q && d_O && d_items && d_logits && nS > 0 && nQ > 0 && nO >= 0 && n_items >= 0, DC_EINVAL,
           "decision.js: eg2 head: bad arguments");
  DC_CHECK(((uintptr_t)d_S | (uintptr_t)d_Q | (uintptr_t)d_O | (uintptr_t)d_items | (uintptr_t)d_logits) % 4 == 0,
           DC_EINVAL, "decision.js: eg2 head: pointers must be 4-byte aligned");
  RC(dc_use(m->ctx));
  if (n_items == 0) return DC_OK;
  double v;
  Eg2HeadW p;
  DC_CHECK(cfg_num(m, "head.width", v) && v > 0, DC_EFORMAT, "decision.js: the model has no decision head");
  p.W = (int)v;
  const dc_tensor *sp = nullptr;
  auto it = m->tensors.find("head.state_proj.weight");
  DC_CHECK(it != m->tensors.end(), DC_EFORMAT, "decision.js: the model has no decision head");
  sp = &it->second;
  p.E = (int)sp->cols;
  const int W = p.W, E = p.E;
  auto it2 = m->tensors.find("head.type_emb.weight");
  DC_CHECK(it2 != m->tensors.end() && it2->second.cols == W, DC_EFORMAT, "decision.js: head.type_emb.weight missing");
  p.ntypes = (int)it2->second.rows;
  RC(head_t(m, "head.state_proj.weight", W, E, p.state_w));
  RC(head_t(m, "head.state_proj.bias", 1, W, p.state_b));
  RC(head_t(m, "head.question_proj.weight", W, E, p.question_w));
  RC(head_t(m, "head.question_proj.bias", 1, W, p.question_b));
  RC(head_t(m, "head.option_proj.weight", W, E, p.option_w));
  RC(head_t(m, "head.option_proj.bias", 1, W, p.option_b));
  RC(head_t(m, "head.field.0.weight", W, 3 * W, p.field0_w));
  RC(head_t(m, "head.field.0.bias", 1, W, p.field0_b));
  RC(head_t(m, "head.field.3.weight", W, W, p.field3_w));
  RC(head_t(m, "head.field.3.bias", 1, W, p.field3_b));
  RC(head_t(m, "head.type_emb.weight", p.ntypes, W, p.type_emb));
  RC(head_t(m, "head.field_norm.weight", 1, W, p.field_norm_w));
  RC(head_t(m, "head.field_norm.bias", 1, W, p.field_norm_b));
  RC(head_t(m, "head.option_norm.weight", 1, W, p.option_norm_w));
  RC(head_t(m, "head.option_norm.bias", 1, W, p.option_norm_b));
  RC(head_t(m, "head.residual.0.weight", W, 4 * W, p.res0_w));
  RC(head_t(m, "head.residual.0.bias", 1, W, p.res0_b));
  RC(head_t(m, "head.residual.3.weight", 1, W, p.res3_w));
  auto scal = [&](const char *k, float &out) -> int {
    DC_CHECK(cfg_num(m, k, v), DC_EFORMAT, "decision.js: the model's config has no %s", k);
    out = (float)v;
    return DC_OK;
  };
  RC(scal("head.ln_eps", p.ln_eps));
  RC(scal("head.prior_scale", p.prior_scale));
  RC(scal("head.joint_scale", p.joint_scale));
  RC(scal("head.gate", p.gate));
  RC(scal("head.residual_bias", p.residual_bias));
  dc_prof_begin(m->ctx, DC_K_OTHER, 0, 0);
  int rc = ops_eg2_head(m->ctx, p, d_S, d_Q, d_O, d_items, n_items, nS, nQ, nO, d_logits);
  dc_prof_end(m->ctx);
  return rc;
}

extern "C" int dc_model_context(dc_model *m, dc_ctx **out) {
  DC_CHECK(m && out, DC_EINVAL, "decision.js: null argument");
  *out = m->ctx;
  return DC_OK;
}
