"""CPU oracle for the decision.js hot path (test infrastructure only).

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference legs may import this module. It
wraps liboracle.so (oracle.c, a C restatement of the reference's WGSL kernels) with numpy, and composes the
reference's engine graphs from those kernels:

  - encoder_embed:  Eg2Engine.embed (src/eg2-engine.ts:72-141), with or without per-layer embeddings;
  - decoder_logits: D13BEngine.run  (src/d1-3b-engine.ts:44-123), attention and LFM2 short-conv layers;
  - d3_logits:      D3Engine.logits (src/d3-engine.ts:67-139), Gated DeltaNet and gated attention layers;
  - omni_logits:    D1OmniEngine.logits (src/omni-engine.ts:56-141), the LFM2 backbone and the transformer head;
  - laya_logits:    LayaEngine.logits (src/laya-engine.ts:47-141), the ModernBERT encoder and the same head.

f16 tensors are numpy uint16 arrays holding IEEE binary16 bits (view them with .view(np.float16)).
"""
from __future__ import annotations

import ctypes
import json
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
SO = os.path.join(HERE, "liboracle.so")
SRC = os.path.join(HERE, "oracle.c")
CFLAGS = ["-O3", "-march=x86-64-v3", "-fopenmp", "-fno-math-errno", "-ffp-contract=off", "-shared", "-fPIC"]


def build(force: bool = False) -> str:
    """Compile oracle.c into liboracle.so beside it (gcc, OpenMP, AVX2/FMA baseline so it runs on any current
    x86-64 server)."""
    if force or not os.path.exists(SO) or os.path.getmtime(SO) < os.path.getmtime(SRC):
        subprocess.check_call(["gcc", *CFLAGS, SRC, "-o", SO + ".tmp", "-lm"])
        os.replace(SO + ".tmp", SO)
    return SO


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(SO):
            build()
        _lib = ctypes.CDLL(SO)
    return _lib


def _p(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def _f16(a):
    a = np.ascontiguousarray(a)
    if a.dtype == np.float16:
        return a.view(np.uint16)
    assert a.dtype == np.uint16, a.dtype
    return a


def threads(n: int | None = None) -> int:
    """OpenMP threads the oracle uses (default: all cores)."""
    n = n or os.cpu_count() or 1
    os.environ["OMP_NUM_THREADS"] = str(n)
    return n


# ---------------------------------------------------------------- kernels

def _limit(what, v, most):
    """The C restatement keeps a row (RoPE/attention: a head of D; pool/readout: H values) in a fixed stack array."""
    if v > most:
        raise ValueError(f"oracle {what}={v} exceeds {most}")


def dequant(Wq, S, N, K, bits):
    out = np.empty((N, K), np.uint16)
    lib().or_dequant(_p(np.ascontiguousarray(Wq)), _p(_f16(S)), _p(out), N, K, bits)
    return out


# The k order of every matmul the graphs below run: 0 = ascending (the reference's MATMUL_PORTABLE order), 1 =
# descending (a second valid f32 order, to measure a stack's sensitivity to summation order; see or_qmatmul_order).
MATMUL_ORDER = 0


def qmatmul(X, Wq, S, N, K, bits, order=None):
    X = _f16(X)
    M = X.size // K
    Y = np.empty((M, N), np.uint16)
    lib().or_qmatmul_order(_p(X), _p(np.ascontiguousarray(Wq)), _p(_f16(S)), _p(Y), M, N, K, bits,
                           MATMUL_ORDER if order is None else order)
    return Y


def add_rmsnorm(X, Yr, W, add, eps):
    """Returns (X after the optional residual add, O); X is not modified."""
    X = _f16(X).copy()
    T, H = X.shape
    O = np.empty_like(X)
    lib().or_add_rmsnorm(_p(X), _p(_f16(Yr) if add else X), _p(_f16(W)), _p(O), T, H, int(add),
                         ctypes.c_float(eps))
    return X, O


def sandwich(X, Y, W1, W2, eps, scale=1.0):
    """Returns (new residual X, O or None)."""
    X = _f16(X).copy()
    T, H = X.shape
    O = np.zeros_like(X)
    norm2 = W2 is not None
    lib().or_sandwich(_p(X), _p(_f16(Y)), _p(_f16(W1)), _p(_f16(W2) if norm2 else _f16(W1)), _p(O), T, H,
                      int(norm2), ctypes.c_float(eps), ctypes.c_float(scale))
    return X, (O if norm2 else None)


def qkv_norm_rope(Z, qn, kn, pos, heads, kv, D, eps, theta, vnorm):
    _limit("qkv_norm_rope: D", D, 1024)
    Z = _f16(Z).copy()
    T = Z.shape[0]
    pos = np.ascontiguousarray(pos, np.int32)
    lib().or_qkv_norm_rope(_p(Z), _p(_f16(qn)), _p(_f16(kn)), _p(pos), T, heads, kv, D, ctypes.c_float(eps),
                           ctypes.c_float(theta), int(vnorm))
    return Z


def attention(Z, rng, heads, kv, D, scale):
    _limit("attention: D", D, 1024)
    Z = _f16(Z)
    T = Z.shape[0]
    rng = np.ascontiguousarray(rng, np.int32).reshape(T, 4)
    Y = np.empty((T, heads * D), np.uint16)
    lib().or_attention(_p(Z), _p(rng), _p(Y), T, heads, kv, D, ctypes.c_float(scale))
    return Y


def attention_ex(Z, rng, heads, kv, D, scale, gate):
    """Attention over rows Z [T, stride] (q | k | v heads, then with `gate` the q heads' output gates)."""
    _limit("attention: D", D, 1024)
    Z = _f16(Z)
    T, stride = Z.shape
    rng = np.ascontiguousarray(rng, np.int32).reshape(T, 4)
    Y = np.empty((T, heads * D), np.uint16)
    lib().or_attention_ex(_p(Z), _p(rng), _p(Y), T, heads, kv, D, ctypes.c_float(scale), ctypes.c_long(stride),
                          int(gate))
    return Y


def glu(A, I, act):
    A = _f16(A)
    T = A.shape[0]
    Hh = np.empty((T, I), np.uint16)
    lib().or_glu(_p(A), _p(Hh), T, I, act)
    return Hh


def gather(ids, Eq, Es, H, bits):
    ids = np.ascontiguousarray(ids, np.int32)
    X = np.empty((ids.size, H), np.uint16)
    lib().or_gather(_p(ids), _p(np.ascontiguousarray(Eq)), _p(_f16(Es)), _p(X), ids.size, H, bits)
    return X


def pool(X, seqs, W=None):
    X = _f16(X)
    H = X.shape[1]
    _limit("pool: H", H, 8192)
    seqs = np.ascontiguousarray(seqs, np.int32).reshape(-1, 2)
    S = seqs.shape[0]
    N = H if W is None else W.shape[0]
    out = np.empty((S, N), np.float32)
    lib().or_pool(_p(X), _p(seqs), _p(None if W is None else _f16(W)), _p(out), S, H, N)
    return out


def leaf_logits(X, leaves, W, ids, Eq, Es, bits, eps):
    X = _f16(X)
    H = X.shape[1]
    _limit("leaf_logits: H", H, 8192)
    leaves = np.ascontiguousarray(leaves, np.int32)
    ids = np.ascontiguousarray(ids, np.int32).reshape(leaves.size, -1)
    L, nIds = ids.shape
    out = np.empty((L, nIds), np.float32)
    lib().or_leaf_logits(_p(X), _p(leaves), _p(_f16(W)), _p(ids), _p(np.ascontiguousarray(Eq)), _p(_f16(Es)),
                         _p(out), L, H, nIds, bits, ctypes.c_float(eps))
    return out


def short_conv(Z, Wc, taps):
    """SHORT_CONV over in-projection rows Z [T, 3H] with taps [T, 4] (-1: no token)."""
    Z = _f16(Z)
    T, H = Z.shape[0], Z.shape[1] // 3
    taps = np.ascontiguousarray(taps, np.int32).reshape(T, 4)
    Y = np.empty((T, H), np.uint16)
    lib().or_short_conv(_p(Z), _p(_f16(Wc)), _p(taps), _p(Y), T, H)
    return Y


def ple_mix(G, E, W, eps):
    G, E = _f16(G), _f16(E)
    T, P = E.shape
    O = np.empty((T, P), np.uint16)
    lib().or_ple_mix(_p(G), _p(E), _p(_f16(W)), _p(O), T, P, ctypes.c_float(eps))
    return O


def readout(X, R, pairs):
    X = _f16(X)
    H = X.shape[1]
    R = np.ascontiguousarray(R, np.float32)
    pairs = np.ascontiguousarray(pairs, np.int32).reshape(-1, 2)
    out = np.empty(pairs.shape[0], np.float32)
    lib().or_readout(_p(X), _p(R), _p(pairs), _p(out), pairs.shape[0], H)
    return out


# ---------------------------------------------------------------- weights (manifest.json + weights.bin)

class Weights:
    """A second, independent reader of the reference's export format (scripts/export_common.py:17-61): the
    manifest names each tensor's dtype, shape, byte offset and size in weights.bin (256-byte aligned), and for q4 /
    q8 the offset and size of its f16 scales."""

    def __init__(self, path: str):
        self.m = json.load(open(os.path.join(path, "manifest.json")))
        self.cfg = self.m["config"]
        self.blob = np.memmap(os.path.join(path, "weights.bin"), np.uint8, "r")

    def has(self, name):
        return name in self.m["tensors"]

    def info(self, name):
        return self.m["tensors"][name]

    def raw(self, name):
        t = self.info(name)
        return np.asarray(self.blob[t["offset"]:t["offset"] + t["bytes"]])

    def f16(self, name):
        t = self.info(name)
        return self.raw(name).view(np.uint16).reshape(t["shape"])

    def host_f32(self, name):
        """An f32 tensor of the manifest's "host" section (EmbeddingGemma 2's decision head)."""
        t = self.m["host"][name]
        return np.asarray(self.blob[t["offset"]:t["offset"] + t["bytes"]]).view(np.float32).reshape(t["shape"])

    def q(self, name):
        """(codes bytes, f16 scales, N, K, bits) of a q4 / q8 tensor."""
        t = self.info(name)
        N, K = t["shape"]
        bits = 8 if t["dtype"] == "q8" else 4
        sc = np.asarray(self.blob[t["scales"]:t["scales"] + t["scales_bytes"]]).view(np.uint16)
        return self.raw(name), sc, N, K, bits


def linear(w: Weights, X, name):
    codes, sc, N, K, bits = w.q(name)
    return qmatmul(X, codes, sc, N, K, bits)


# ---------------------------------------------------------------- graphs

def encoder_meta(seqs, window=None):
    """Per-token key ranges of packed bidirectional sequences (src/eg2-engine.ts:75-85): the whole sequence, or
    |query - key| <= window; plus each token's position and the sequences' [start, end)."""
    rng, pos, bounds = [], [], []
    start = 0
    for n in seqs:
        end = start + n
        for i in range(n):
            t = start + i
            if window is None:
                rng.append((start, end, 0, 0))
            else:
                rng.append((max(start, t - window), min(end, t + window + 1), 0, 0))
            pos.append(i)
        bounds.append((start, end))
        start = end
    return np.array(rng, np.int32), np.array(pos, np.int32), np.array(bounds, np.int32)


def encoder_embed(w: Weights, ids, seq_lens, layers=None):
    """Eg2Engine.embed (src/eg2-engine.ts:72-141): mean-pooled (optionally projected) embeddings [S, N] f32,
    before the host's L2 normalisation. With per-layer embeddings (config ple > 0) every layer ends with the PLE
    block (src/eg2-engine.ts:123-128): the MLP's post-norm alone, then x = (x + norm(proj(gelu(gate(x)) *
    norm(ple_in(xe))))) * layer scalar, xe the embedding rows; without them the layer scalar and the next
    layer's input norm go on the MLP's sandwich."""
    c = w.cfg
    H, eps, heads = c["hidden"], c["eps"], c["heads"]
    ple = int(c.get("ple", 0) or 0)
    ids = np.asarray(ids, np.int32)
    codes, sc, _, _, bits = w.q("embed")
    x = gather(ids, codes, sc, H, bits)
    xe = x.copy()
    zero = np.zeros(H, np.uint16)
    x, normed = sandwich(x, np.zeros_like(x), zero, w.f16("layers.0.input_layernorm"), eps)
    L = c["layers"] if layers is None else layers
    for i in range(L):
        p = f"layers.{i}."
        typ = c["layer_types"][i]
        D, kv = c["head_dim"][typ], c["kv_heads"][typ]
        win = c.get("window") if typ == "sliding_attention" else None
        rng, pos, bounds = encoder_meta(seq_lens, win)
        z = linear(w, normed, p + "qkv")
        z = qkv_norm_rope(z, w.f16(p + "q_norm"), w.f16(p + "k_norm"), pos, heads, kv, D, eps,
                          c["rope_theta"][typ], c.get("v_norm", True))
        y = attention(z, rng, heads, kv, D, c.get("attn_scale", 1.0))
        o = linear(w, y, p + "o")
        x, normed = sandwich(x, o, w.f16(p + "post_attention_layernorm"), w.f16(p + "pre_feedforward_layernorm"), eps)
        z = linear(w, normed, p + "gu")
        h = glu(z, c["intermediate"], 1)
        o = linear(w, h, p + "down")
        nxt = f"layers.{i + 1}.input_layernorm" if i + 1 < L else "final_norm"
        lscale = c.get("layer_scalars", [1.0] * c["layers"])[i]
        if ple:
            x, _ = sandwich(x, o, w.f16(p + "post_feedforward_layernorm"), None, eps)
            gate = linear(w, x, p + "ple_gate")
            e = linear(w, xe, p + "ple_in")
            mix = ple_mix(gate, e, w.f16("ple.norm"), eps)
            o = linear(w, mix, p + "ple_proj")
            x, normed = sandwich(x, o, w.f16(p + "ple_norm"), w.f16(nxt), eps, lscale)
        else:
            x, normed = sandwich(x, o, w.f16(p + "post_feedforward_layernorm"), w.f16(nxt), eps, lscale)
    _, _, bounds = encoder_meta(seq_lens)
    proj = w.f16("projection") if w.has("projection") else None
    return pool(normed, bounds, proj)


def decoder_meta(trees, with_taps=False):
    """The forest of D13BEngine.run (src/d1-3b-engine.ts:46-68) as per-token key ranges: a trunk token reads
    [start, t+1); a branch token reads the whole trunk and its own branch up to itself. Also positions, readout
    rows (the last token of each branch) and the flattened readout ids per leaf; with_taps adds the short
    convolution's taps [T, 4] built as the reference builds them (src/d1-3b-engine.ts:53-62): a trunk token reads
    its two predecessors in the trunk, a branch token its predecessors in the branch, then the trunk's last
    tokens."""
    ids, pos, rng, leaves, leaf_ids, taps = [], [], [], [], [], []
    for tr in trees:
        start = len(ids)
        p = len(tr["trunk"])
        for i, tok in enumerate(tr["trunk"]):
            ids.append(tok)
            pos.append(i)
            rng.append((start, start + i + 1, 0, 0))
            taps.append((start + i - 2 if i >= 2 else -1, start + i - 1 if i >= 1 else -1, start + i, 0))
        for b, br in enumerate(tr["branches"]):
            bstart = len(ids)
            for o, tok in enumerate(br):
                t = len(ids)
                ids.append(tok)
                pos.append(p + o)
                rng.append((start, start + p, bstart, t + 1))

                def back(j):
                    return t - j if o - j >= 0 else (start + p + (o - j) if p + (o - j) >= 0 else -1)

                taps.append((back(2), back(1), t, 0))
            leaves.append(len(ids) - 1)
            leaf_ids.append([i for g in tr["groups"][b] for i in g])
    n = max(len(x) for x in leaf_ids)
    flat = np.zeros((len(leaves), n), np.int32)
    for i, g in enumerate(leaf_ids):
        flat[i, :len(g)] = g
    out = (np.array(ids, np.int32), np.array(pos, np.int32), np.array(rng, np.int32), np.array(leaves, np.int32),
           flat)
    return out + (np.array(taps, np.int32).reshape(-1, 4),) if with_taps else out


def decoder_logits(w: Weights, ids, pos, rng, leaves, leaf_ids, layers=None, taps=None):
    """D13BEngine.run's GPU part (src/d1-3b-engine.ts:86-108): the option-token logits [L, nIds] f32 at each
    readout row. Conv layers (LFM2: in_proj, SHORT_CONV over `taps`, out_proj) need the taps of decoder_meta."""
    c = w.cfg
    H, I, heads, kv, D, eps = c["hidden"], c["intermediate"], c["heads"], c["kv_heads"], c["head_dim"], c["eps"]
    codes, sc, _, _, bits = w.q("embed")
    x = gather(ids, codes, sc, H, bits)
    x, normed = add_rmsnorm(x, None, w.f16("layers.0.operator_norm"), False, eps)
    L = len(c["layer_types"]) if layers is None else layers
    scale = c.get("attn_scale", 1.0 / np.sqrt(D))
    for i in range(L):
        p = f"layers.{i}."
        if c["layer_types"][i] == "conv":
            if taps is None:
                raise ValueError("oracle: a conv layer needs the taps (decoder_meta(trees, with_taps=True))")
            z = linear(w, normed, p + "in_proj")
            y = short_conv(z, w.f16(p + "conv"), taps)
            o = linear(w, y, p + "out_proj")
        else:
            z = linear(w, normed, p + "qkv")
            z = qkv_norm_rope(z, w.f16(p + "q_norm"), w.f16(p + "k_norm"), pos, heads, kv, D, eps, c["rope_theta"],
                              0)
            y = attention(z, rng, heads, kv, D, scale)
            o = linear(w, y, p + "o_proj")
        x, normed = add_rmsnorm(x, o, w.f16(p + "ffn_norm"), True, eps)
        z = linear(w, normed, p + "w13")
        h = glu(z, I, 0)
        o = linear(w, h, p + "w2")
        nxt = f"layers.{i + 1}.operator_norm" if i + 1 < L else "final_norm"
        x, normed = add_rmsnorm(x, o, w.f16(nxt), True, eps)
    return leaf_logits(x, leaves, w.f16("final_norm"), leaf_ids, codes, sc, bits, eps)


def _erf_as(x):
    """erf by Abramowitz & Stegun 7.1.26 (|error| < 1.5e-7), as src/eg2-head.ts:21-25 writes it."""
    t = 1.0 / (1.0 + 0.3275911 * np.abs(x))
    y = 1.0 - ((((1.061405429 * t - 1.453152027) * t + 1.421413741) * t - 0.284496736) * t + 0.254829592) * t * \
        np.exp(-x * x)
    return np.where(x >= 0, y, -y)


def _gelu_erf(x):
    return 0.5 * x * (1.0 + _erf_as(x / np.sqrt(2.0)))


def _layer_norm(x, w, b, eps):
    m = x.mean()
    v = ((x - m) ** 2).mean()
    return (x - m) / np.sqrt(v + eps) * w + b


def eg2_head_logits(w: Weights, qtype: str, s, q, opts):
    """Eg2Head.logits (src/eg2-head.ts:62-100) in float64: the raw logit of every option, from the normalised
    embeddings of the state `s`, the question `q` and the options `opts` [n, E]."""
    c = w.cfg
    h = c["head"]
    t = lambda n: w.host_f32("head." + n).astype(np.float64)
    s, q = np.asarray(s, np.float64), np.asarray(q, np.float64)
    S = t("state_proj.weight") @ s + t("state_proj.bias")
    Q = t("question_proj.weight") @ q + t("question_proj.bias")
    f1 = _gelu_erf(t("field.0.weight") @ np.concatenate([S, Q, S * Q]) + t("field.0.bias"))
    f2 = t("field.3.weight") @ f1 + t("field.3.bias") + t("type_emb.weight")[c["question_types"].index(qtype)]
    f = _layer_norm(f2, t("field_norm.weight"), t("field_norm.bias"), h["ln_eps"])
    W = f.size
    R0, rb, R3 = t("residual.0.weight"), t("residual.0.bias"), t("residual.3.weight").reshape(-1)
    rf = R0[:, :W] @ f + rb
    anchor = s + q
    an = max(np.linalg.norm(anchor), 1e-12)
    out = []
    for e in np.asarray(opts, np.float64):
        O = t("option_proj.weight") @ e + t("option_proj.bias")
        on = _layer_norm(O, t("option_norm.weight"), t("option_norm.bias"), h["ln_eps"])
        o = e / max(np.linalg.norm(e), 1e-12)
        r = R0[:, W:2 * W] @ on
        rm = R0[:, 2 * W:3 * W] @ (f * on)
        ra = R0[:, 3 * W:] @ np.abs(f - on)
        res = h["residual_bias"] + float(R3 @ _gelu_erf(rf + r + rm + ra))
        joint = h["joint_scale"] * float(f @ on) / max(np.linalg.norm(f) * np.linalg.norm(on), 1e-8)
        prior = h["prior_scale"] * float(o @ anchor) / an
        out.append(prior + h["gate"] * (joint + res))
    return np.array(out)


def softmax(z):
    """The host softmax of src/gpu.ts:294-297."""
    z = np.asarray(z, np.float64)
    e = np.exp(z - z.max())
    return e / e.sum()


def gdn(Z, stride, qkv, H, W, Alog, dtb, gw, spans, eps, T):
    """The Gated DeltaNet mixer (src/d3-kernels.ts:23-149) over in-projection rows Z [T, stride]; spans [nseq, 4]
    (a start, a length | write-a << 31, b start, b length). Returns Y [T, H*128] f16 bits (rows no span writes: 0)."""
    Z = _f16(Z).reshape(-1)
    spans = np.ascontiguousarray(spans, np.uint32).reshape(-1, 4)
    Y = np.zeros((T, H * 128), np.uint16)
    lib().or_gdn(_p(Z), ctypes.c_long(stride), ctypes.c_long(qkv), H, _p(_f16(W)), _p(_f16(Alog)), _p(_f16(dtb)),
                 _p(_f16(gw)), _p(spans), spans.shape[0], ctypes.c_float(eps), _p(Y))
    return Y


def add_rows(Xi, idx, E):
    Xi, E = _f16(Xi), _f16(E)
    T, H = Xi.shape
    Xo = np.empty_like(Xi)
    lib().or_add_rows(_p(Xi), _p(np.ascontiguousarray(idx, np.int32)), _p(E), _p(Xo), T, H)
    return Xo


def bias_act(Y, b, act):
    Y = _f16(Y).copy()
    T, N = Y.shape
    lib().or_bias_act(_p(Y), _p(_f16(b)), T, N, act)
    return Y


def add_layernorm(X, Yr, W, B, add, eps):
    """Returns (X after the optional residual add, O); X is not modified."""
    X = _f16(X).copy()
    T, H = X.shape
    O = np.empty_like(X)
    lib().or_add_layernorm(_p(X), _p(None if Yr is None else _f16(Yr)), _p(_f16(W)), _p(None if B is None else _f16(B)),
                           _p(O), T, H, int(add), ctypes.c_float(eps))
    return X, O


def gather_rows(X, rows):
    X = _f16(X)
    rows = np.ascontiguousarray(rows, np.int32)
    G = np.empty((rows.size, X.shape[1]), np.uint16)
    lib().or_gather_rows(_p(X), _p(rows), _p(G), rows.size, X.shape[1])
    return G


def score(Y, w, b):
    Y = _f16(Y)
    out = np.empty(Y.shape[0], np.float32)
    lib().or_score(_p(Y), _p(_f16(w)), _p(_f16(b)), _p(out), Y.shape[0], Y.shape[1])
    return out


def qk_rope(Z, qn, kn, pos, heads, kv, D, rot, norm, eps, theta):
    """Returns a rotated (and normed) copy of Z [T, stride]."""
    Z = _f16(Z).copy()
    T, stride = Z.shape
    lib().or_qk_rope(_p(Z), _p(None if qn is None else _f16(qn)), _p(None if kn is None else _f16(kn)),
                     _p(np.ascontiguousarray(pos, np.int32)), T, heads, kv, D, ctypes.c_long(stride), rot, int(norm),
                     ctypes.c_float(eps), ctypes.c_float(theta))
    return Z


def d3_meta(seqs, groups=None):
    """The per-token and per-sequence metadata D3Engine.logits builds (src/d3-engine.ts:71-92), restated: seqs are
    (ids, options); groups (sequences per request, consecutive) share their common token prefix as one trunk (at
    least one token left per sequence). Returns ids, pos, key ranges [T, 4], spans [nseq, 4] and readout pairs
    (last token, code) [P, 2]."""
    ids, pos, rng, spans, pairs = [], [], [], [], []
    sizes = groups or [1] * len(seqs)
    si = 0
    for n in sizes:
        group = seqs[si:si + n]
        si += n
        P = 0
        if n > 1:
            lim = min(len(s[0]) for s in group) - 1
            while P < lim and all(s[0][P] == group[0][0][P] for s in group):
                P += 1
        ts = len(ids)
        for i in range(P):
            ids.append(group[0][0][i]), pos.append(i), rng.append((ts, ts + P, 0, 0))
        for b, (sids, opts) in enumerate(group):
            bs = len(ids)
            be = bs + len(sids) - P
            for i in range(P, len(sids)):
                ids.append(sids[i]), pos.append(i)
                rng.append((ts, ts + P, bs, be) if P else (bs, be, 0, 0))
            flag = 0x80000000 if (b == 0 or not P) else 0
            spans.append((ts if P else bs, (P if P else be - bs) | flag, bs if P else 0, be - bs if P else 0))
            pairs += [(be - 1, k) for k in range(opts)]
    return (np.array(ids, np.int32), np.array(pos, np.int32), np.array(rng, np.int32).reshape(-1, 4),
            np.array(spans, np.uint32).reshape(-1, 4), np.array(pairs, np.int32).reshape(-1, 2))


def d3_logits(w: Weights, ids, pos, rng, spans, pairs, layers=None):
    """D3Engine.logits's GPU part (src/d3-engine.ts:103-131): the code logits [P] f32 at the readout pairs."""
    c = w.cfg
    H, I, heads, kv, D, eps = c["hidden"], c["intermediate"], c["heads"], c["kv_heads"], c["head_dim"], c["eps"]
    LH, rows = c.get("linear_heads", 0), c.get("linear_rows", 0)
    T = len(ids)
    codes, sc, _, _, bits = w.q("embed")
    x = gather(ids, codes, sc, H, bits)
    o = None
    L = len(c["layer_types"]) if layers is None else layers
    for i in range(L):
        p = f"layers.{i}."
        x, normed = add_rmsnorm(x, o if i > 0 else None, w.f16(p + "input_norm"), i > 0, eps)
        if c["layer_types"][i] == "linear_attention":
            z = linear(w, normed, p + "in")
            y = gdn(z, rows, 3 * LH * 128, LH, w.f16(p + "conv"), w.f16(p + "A_log"), w.f16(p + "dt_bias"),
                    w.f16(p + "gnorm"), spans, eps, T)
            o = linear(w, y, p + "out")
        else:
            z = linear(w, normed, p + "qkvg")
            z = qk_rope(z, w.f16(p + "q_norm"), w.f16(p + "k_norm"), pos, heads, kv, D, c.get("rotary_dim", D), True,
                        eps, c["rope_theta"])
            y = attention_ex(z, rng, heads, kv, D, 1.0 / np.sqrt(D), True)
            o = linear(w, y, p + "o")
        x, normed = add_rmsnorm(x, o, w.f16(p + "post_norm"), True, eps)
        h = glu(linear(w, normed, p + "w13"), I, 0)
        o = linear(w, h, p + "w2")
    x, normed = add_rmsnorm(x, o, w.f16("final_norm"), True, eps)
    t = w.info("readout")
    R = w.raw("readout").view(np.float32).reshape(t["shape"])
    return readout(normed, R, pairs)


def omni_meta(seqs):
    """The per-token metadata D1OmniEngine.logits builds (src/omni-engine.ts:58-69), restated: seqs are (ids,
    markers relative to the sequence, question type 0 choice / 1 score / 2 noul). Returns ids, positions, key ranges
    (the sequence, bidirectional), conv taps (t-1, t, t+1 inside the sequence), types per token, absolute markers."""
    ids, pos, rng, taps, qt, marks = [], [], [], [], [], []
    for sids, mk, typ in seqs:
        start, end = len(ids), len(ids) + len(sids)
        for i, tok in enumerate(sids):
            t = start + i
            ids.append(tok), pos.append(i), qt.append(typ), rng.append((start, end, 0, 0))
            taps.append((t - 1 if t > start else -1, t, t + 1 if t + 1 < end else -1, 0))
        marks += [start + m for m in mk]
    a = lambda x, s=None: np.asarray(x, np.int32) if s is None else np.asarray(x, np.int32).reshape(s)  # noqa: E731
    return a(ids), a(pos), a(rng, (-1, 4)), a(taps, (-1, 4)), a(qt), a(marks)


def _lfm2_backbone(w: Weights, ids, pos, rng, taps):
    """The backbone loop of D13BEngine.run / D1OmniEngine.logits: returns (x, the final-normed rows)."""
    c = w.cfg
    H, I, heads, kv, D, eps = c["hidden"], c["intermediate"], c["heads"], c["kv_heads"], c["head_dim"], c["eps"]
    codes, sc, _, _, bits = w.q("embed")
    x = gather(ids, codes, sc, H, bits)
    x, normed = add_rmsnorm(x, None, w.f16("layers.0.operator_norm"), False, eps)
    L = len(c["layer_types"])
    scale = c.get("attn_scale", 1.0 / np.sqrt(D))
    for i in range(L):
        p = f"layers.{i}."
        if c["layer_types"][i] == "conv":
            y = short_conv(linear(w, normed, p + "in_proj"), w.f16(p + "conv"), taps)
            o = linear(w, y, p + "out_proj")
        else:
            z = qkv_norm_rope(linear(w, normed, p + "qkv"), w.f16(p + "q_norm"), w.f16(p + "k_norm"), pos, heads, kv,
                              D, eps, c["rope_theta"], 0)
            o = linear(w, attention(z, rng, heads, kv, D, scale), p + "o_proj")
        x, normed = add_rmsnorm(x, o, w.f16(p + "ffn_norm"), True, eps)
        o = linear(w, glu(linear(w, normed, p + "w13"), I, 0), p + "w2")
        nxt = f"layers.{i + 1}.operator_norm" if i + 1 < L else "final_norm"
        x, normed = add_rmsnorm(x, o, w.f16(nxt), True, eps)
    return x, normed


def omni_logits(w: Weights, ids, pos, rng, taps, qtype, markers):
    """D1OmniEngine.logits's GPU part (src/omni-engine.ts:98-131): the raw logit at every option marker."""
    _, normed = _lfm2_backbone(w, ids, pos, rng, taps)
    return _decision_head(w, normed, rng, qtype, markers)


def laya_meta(seqs, window):
    """The per-token metadata LayaEngine.logits builds (src/laya-engine.ts:52-63), restated: omni_meta's ids,
    positions, ranges, types and markers, and each token's window [max(start, t - window), min(end, t + window + 1))."""
    ids, pos, rng, taps, qt, marks = omni_meta(seqs)
    t = np.arange(len(ids))
    win = np.zeros_like(rng)
    win[:, 0] = np.maximum(rng[:, 0], t - window)
    win[:, 1] = np.minimum(rng[:, 1], t + window + 1)
    return ids, pos, rng, win, qt, marks


def _decision_head(w: Weights, normed, rng, qtype, markers):
    """The d1-omni / Laya head (src/omni-engine.ts:115-131, src/laya-engine.ts:112-130)."""
    c = w.cfg
    ln_eps, hh = c["ln_eps"], c["head_heads"]
    x = add_rows(normed, qtype, w.f16("head.type_emb"))
    o = None
    for i in range(c["head_layers"]):
        p = f"head.{i}."
        x, n = add_layernorm(x, o, w.f16(p + "norm1"), w.f16(p + "norm1_bias"), i > 0, ln_eps)
        z = bias_act(linear(w, n, p + "in_proj"), w.f16(p + "in_proj_bias"), 0)
        o = bias_act(linear(w, attention(z, rng, hh, hh, 64, 0.125), p + "out_proj"), w.f16(p + "out_proj_bias"), 0)
        x, n = add_layernorm(x, o, w.f16(p + "norm2"), w.f16(p + "norm2_bias"), True, ln_eps)
        h = bias_act(linear(w, n, p + "linear1"), w.f16(p + "linear1_bias"), 1)
        o = bias_act(linear(w, h, p + "linear2"), w.f16(p + "linear2_bias"), 0)
    x, n = add_layernorm(x, o, w.f16("scorer.norm"), w.f16("scorer.norm_bias"), True, ln_eps)
    g = bias_act(linear(w, gather_rows(n, markers), "scorer.fc"), w.f16("scorer.fc_bias"), 2)
    return score(g, w.f16("scorer.out"), w.f16("scorer.out_bias"))


def laya_logits(w: Weights, ids, pos, rng, win, qtype, markers):
    """LayaEngine.logits's GPU part (src/laya-engine.ts:86-131): the raw logit at every option marker."""
    c = w.cfg
    H, I, heads, eps = c["hidden"], c["intermediate"], c["heads"], c["eps"]
    codes, sc, _, _, bits = w.q("embed")
    e = gather(ids, codes, sc, H, bits)
    _, x = add_layernorm(e, None, w.f16("embed_norm"), None, False, eps)
    o = None
    for i in range(len(c["layer_types"])):
        p = f"layers.{i}."
        glob = c["layer_types"][i] == "full_attention"
        attn_in = x
        if w.has(p + "attn_norm"):
            x, attn_in = add_layernorm(x, o, w.f16(p + "attn_norm"), None, True, eps)
        z = qk_rope(linear(w, attn_in, p + "qkv"), None, None, pos, heads, heads, 64, 64, False, eps,
                    c["rope_theta"]["full_attention" if glob else "sliding_attention"])
        o = linear(w, attention(z, rng if glob else win, heads, heads, 64, 0.125), p + "o")
        x, n = add_layernorm(x, o, w.f16(p + "mlp_norm"), None, True, eps)
        o = linear(w, glu(linear(w, n, p + "wi"), I, 2), p + "wo")
    x, normed = add_layernorm(x, o, w.f16("final_norm"), None, True, eps)
    return _decision_head(w, normed, rng, qtype, markers)
