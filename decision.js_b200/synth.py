"""Synthetic, seeded models and inputs in the reference's export format.

The reference's exporters (scripts/export_common.py:17-97) write weights.bin (every tensor 256-byte aligned) and
manifest.json ({"format": "d1.js/1", config, tensors: {name: {dtype, shape, offset, bytes[, scales,
scales_bytes]}}, bytes}). The quantizers here follow the same published rules, so files written here are
indistinguishable in format from the reference's own exports:
  q8: scale = f16(absmax / 127) per 32 values along K (1 for an all-zero block), code = clamp(round(w / scale),
      -127, 127) stored + 128;
  q4: the best (least squared error) of 46 candidate scales f16(absmax * f / d), f in linspace(0.6, 1.15, 23),
      d in {7, 8}; code = clamp(round(w / scale), -8, 7) stored + 8, two codes per byte, low nibble first.

Model presets mirror the BASELINE configs: EmbeddingGemma-300M-architecture encoder (q8), a 0.6B dense decoder
(q8) and a 3B dense decoder (q4), with random weights (linears ~N(0, 0.02) then quantized; norms 1 + 0.1 N(0, 1)).
"""
from __future__ import annotations

import json
import math
import os

import numpy as np
import torch

BLOCK = 32


def quantize8(w: torch.Tensor):
    """q8 codes [N, K] uint8 and f16 scales [N, K/32] of a float [N, K] weight."""
    n, k = w.shape
    blocks = w.float().reshape(n, k // BLOCK, BLOCK)
    scale = (blocks.abs().amax(-1) / 127).half().float()
    scale = torch.where(scale == 0, torch.ones_like(scale), scale)
    codes = torch.clamp(torch.round(blocks / scale[..., None]), -127, 127)
    return (codes + 128).to(torch.uint8).reshape(n, k).cpu().numpy(), scale.half().cpu().numpy()


def quantize4(w: torch.Tensor, rows: int = 8192):
    """q4 codes [N, K/2] uint8 (low nibble first) and f16 scales [N, K/32] of a float [N, K] weight."""
    if w.shape[0] > rows:
        parts = [quantize4(w[i:i + rows]) for i in range(0, w.shape[0], rows)]
        return np.concatenate([p[0] for p in parts]), np.concatenate([p[1] for p in parts])
    n, k = w.shape
    blocks = w.float().reshape(n, k // BLOCK, BLOCK)
    amax = blocks.abs().amax(-1).clamp(min=1e-12)
    best_codes = best_scale = err = None
    for f in torch.linspace(0.6, 1.15, 23):
        for d in (7.0, 8.0):
            scale = (amax * f.to(amax.device) / d).half().float()
            scale = torch.where(scale == 0, torch.ones_like(scale), scale)
            codes = torch.clamp(torch.round(blocks / scale[..., None]), -8, 7)
            e = ((codes * scale[..., None] - blocks) ** 2).sum(-1)
            if err is None:
                best_codes, best_scale, err = codes, scale, e
            else:
                better = e < err
                best_codes = torch.where(better[..., None], codes, best_codes)
                best_scale = torch.where(better, scale, best_scale)
                err = torch.minimum(e, err)
    codes = (best_codes + 8).to(torch.uint8).reshape(n, k)
    packed = codes[:, 0::2] | (codes[:, 1::2] << 4)
    return packed.contiguous().cpu().numpy(), best_scale.half().cpu().numpy()


def dequantize(codes: np.ndarray, scales: np.ndarray, N: int, K: int, bits: int) -> np.ndarray:
    """f16 [N, K] = f16((code - Z) * scale), one rounding (numpy; for tests and tools)."""
    if bits == 8:
        c = codes.reshape(N, K).astype(np.int32) - 128
    else:
        b = codes.reshape(N, K // 2)
        c = np.empty((N, K), np.int32)
        c[:, 0::2] = b & 15
        c[:, 1::2] = b >> 4
        c -= 8
    s = np.repeat(scales.reshape(N, K // BLOCK).astype(np.float32), BLOCK, axis=1)
    return (c.astype(np.float32) * s).astype(np.float16)


class Writer:
    """weights.bin + manifest.json in the reference's layout (scripts/export_common.py:17-61)."""

    def __init__(self, out: str, config: dict):
        os.makedirs(out, exist_ok=True)
        self.out = out
        self.f = open(os.path.join(out, "weights.bin"), "wb")
        self.offset = 0
        self.manifest = {"format": "d1.js/1", "config": config, "tensors": {}}

    def put(self, raw: bytes) -> int:
        pad = (-self.offset) % 256
        self.f.write(b"\0" * pad)
        self.offset += pad
        start = self.offset
        self.f.write(raw)
        self.offset += len(raw)
        return start

    def quant(self, name: str, w: torch.Tensor, bits: int):
        codes, scales = (quantize8 if bits == 8 else quantize4)(w)
        self.manifest["tensors"][name] = {"dtype": f"q{bits}", "shape": list(w.shape),
                                          "offset": self.put(codes.tobytes()), "bytes": int(codes.nbytes),
                                          "scales": self.put(scales.tobytes()), "scales_bytes": int(scales.nbytes)}

    def raw_quant(self, name: str, codes: np.ndarray, scales: np.ndarray, shape, bits: int):
        self.manifest["tensors"][name] = {"dtype": f"q{bits}", "shape": list(shape),
                                          "offset": self.put(codes.tobytes()), "bytes": int(codes.nbytes),
                                          "scales": self.put(scales.tobytes()), "scales_bytes": int(scales.nbytes)}

    def f32_host(self, name: str, t):
        """An f32 tensor listed under the manifest's "host" section (scripts/export-eg2.py:119-123)."""
        a = np.ascontiguousarray(np.asarray(t.detach().float().cpu().numpy() if isinstance(t, torch.Tensor) else t,
                                            np.float32))
        self.manifest.setdefault("host", {})[name] = {"dtype": "f32", "shape": list(a.shape),
                                                      "offset": self.put(a.tobytes()), "bytes": int(a.nbytes)}

    def f16(self, name: str, t):
        a = np.asarray(t.detach().float().cpu().numpy() if isinstance(t, torch.Tensor) else t).astype(np.float16)
        self.manifest["tensors"][name] = {"dtype": "f16", "shape": list(a.shape), "offset": self.put(a.tobytes()),
                                          "bytes": int(a.nbytes)}

    def close(self):
        self.f.close()
        self.manifest["bytes"] = self.offset
        with open(os.path.join(self.out, "manifest.json"), "w") as f:
            json.dump(self.manifest, f)


# ---------------------------------------------------------------- presets

ENCODER_EG300M = dict(model="eg2", hidden=768, intermediate=1152, layers=24, heads=3, vocab=262144,
                      layer_types=(["sliding_attention"] * 5 + ["full_attention"]) * 4, window=512, eps=1e-6,
                      head_dim={"sliding_attention": 256, "full_attention": 256},
                      kv_heads={"sliding_attention": 1, "full_attention": 1},
                      rope_theta={"sliding_attention": 10000.0, "full_attention": 1000000.0}, ple=0,
                      attn_scale=1.0 / 16.0, v_norm=True, embedding_dim=768, embed_dim=768, bits=8)
DECODER_0P6B = dict(model="d1-3b", hidden=1024, intermediate=3072, heads=16, kv_heads=8, head_dim=128, vocab=151936,
                    eps=1e-6, rope_theta=1000000.0, layers=28, bits=8)
DECODER_3B = dict(model="d1-3b", hidden=3072, intermediate=8192, heads=24, kv_heads=8, head_dim=128, vocab=65536,
                  eps=1e-5, rope_theta=1000000.0, layers=32, bits=4)
# The reference's own engines, at their architectures (scripts/export-3b.py, scripts/export-eg2.py): d1-3B is an LFM2
# hybrid (short-conv layers between grouped-query attention layers with 64-wide heads, q4); EmbeddingGemma 2 has
# per-layer embeddings, 256-wide heads on its sliding layers and 512-wide heads on every sixth (full) layer. The
# reference's EG2 attends with scale 1 (src/eg2-engine.ts:117) and trained q/k norm weights; with random norm weights
# near 1, 512-wide scores would spread +-20 and the softmax would be nearly one-hot, so the synthetic preset scales
# the scores by 1/16 (config attn_scale), as the EmbeddingGemma-300M preset does.
DECODER_LFM2 = dict(model="d1-3b", hidden=2048, intermediate=8192, heads=32, kv_heads=8, head_dim=64, vocab=65536,
                    eps=1e-5, rope_theta=1000000.0, layers=30, bits=4,
                    layer_types=["conv", "conv", "full_attention"] * 10)
ENCODER_EG2 = dict(model="eg2", hidden=512, intermediate=2048, layers=24, heads=4, vocab=262144,
                   layer_types=(["sliding_attention"] * 5 + ["full_attention"]) * 4, window=512, eps=1e-6,
                   head_dim={"sliding_attention": 256, "full_attention": 512},
                   kv_heads={"sliding_attention": 1, "full_attention": 1},
                   rope_theta={"sliding_attention": 10000.0, "full_attention": 1000000.0}, ple=512,
                   attn_scale=1.0 / 16.0, embedding_dim=768, embed_dim=768, bits=8, prompt="task: classification | query: ", max_len=2048,
                   question_types=["choice", "score", "noul"],
                   temperatures={"choice": 1.0, "score": 0.8, "noul": 1.2},
                   head={"width": 256, "ln_eps": 1e-5, "prior_scale": 4.0, "joint_scale": 6.0, "gate": 0.6,
                         "residual_bias": 0.1})


def _gen(seed: int, device: str):
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return g


def _normal(shape, std, g, device):
    return torch.randn(*shape, generator=g, device=device) * std


def _norm_w(n, g, device):
    return 1.0 + 0.1 * torch.randn(n, generator=g, device=device)


def write_encoder(out: str, seed: int = 0, device: str = "cpu", preset: dict | None = None, **over) -> dict:
    """An Eg2Engine-format encoder (src/eg2-engine.ts); with config ple > 0 it has per-layer embeddings
    (scripts/export-eg2.py:103-125: ple.norm, and per layer ple_gate, ple_in, ple_proj, ple_norm) and, when its
    config names an embedding_dim other than hidden, a pooled projection. Returns the config."""
    c = {**(preset or ENCODER_EG300M), **over}
    bits = c.pop("bits")
    H, I, L, heads = c["hidden"], c["intermediate"], c["layers"], c["heads"]
    P = int(c.get("ple", 0) or 0)
    c["layer_types"] = list(c["layer_types"])[:L]
    # layer scalars near the trained model's (< 1 with PLE, which adds a third residual branch per layer)
    c["layer_scalars"] = [1.0] * L if not P else [0.6 + 0.02 * (i % 5) for i in range(L)]
    g = _gen(seed, device)
    w = Writer(out, c)
    # the embedding with its sqrt(hidden) scale folded in (scripts/export-eg2.py:69,100)
    V = c["vocab"]
    emb_rows = []
    for i in range(0, V, 65536):
        emb_rows.append(_normal((min(65536, V - i), H), 0.02 * math.sqrt(H), g, device))
    w.quant("embed", torch.cat(emb_rows), bits)
    for i in range(L):
        p = f"layers.{i}."
        t = c["layer_types"][i]
        D, kv = c["head_dim"][t], c["kv_heads"][t]
        w.quant(p + "qkv", _normal(((heads + 2 * kv) * D, H), 0.02, g, device), bits)
        w.f16(p + "q_norm", _norm_w(D, g, device))
        w.f16(p + "k_norm", _norm_w(D, g, device))
        w.quant(p + "o", _normal((H, heads * D), 0.02, g, device), bits)
        w.quant(p + "gu", _normal((2 * I, H), 0.02, g, device), bits)
        w.quant(p + "down", _normal((H, I), 0.02, g, device), bits)
        for n in ("input_layernorm", "post_attention_layernorm", "pre_feedforward_layernorm",
                  "post_feedforward_layernorm"):
            w.f16(p + n, _norm_w(H, g, device))
        if P:
            w.quant(p + "ple_gate", _normal((P, H), 0.02, g, device), bits)
            w.quant(p + "ple_in", _normal((P, H), 0.02, g, device), bits)
            w.quant(p + "ple_proj", _normal((H, P), 0.02, g, device), bits)
            w.f16(p + "ple_norm", _norm_w(H, g, device))
    if P:
        w.f16("ple.norm", _norm_w(P, g, device))
    w.f16("final_norm", _norm_w(H, g, device))
    if c.get("embedding_dim", H) != H:  # the pooled embedding's projection [embedding_dim, H] f16
        w.f16("projection", _normal((c["embedding_dim"], H), 1.0 / math.sqrt(H), g, device))
    if c.get("head"):  # the typed-decision head, f32 on the host side of the manifest (src/eg2-head.ts)
        Wd, E, nt = c["head"]["width"], c["embed_dim"], len(c["question_types"])
        for n, shape, std in (("state_proj", (Wd, E), 1 / math.sqrt(E)), ("question_proj", (Wd, E), 1 / math.sqrt(E)),
                              ("option_proj", (Wd, E), 1 / math.sqrt(E)), ("field.0", (Wd, 3 * Wd), 1 / math.sqrt(3 * Wd)),
                              ("field.3", (Wd, Wd), 1 / math.sqrt(Wd)), ("residual.0", (Wd, 4 * Wd), 1 / math.sqrt(4 * Wd))):
            w.f32_host(f"head.{n}.weight", _normal(shape, std, g, device))
            w.f32_host(f"head.{n}.bias", _normal((Wd,), 0.02, g, device))
        w.f32_host("head.residual.3.weight", _normal((1, Wd), 1 / math.sqrt(Wd), g, device))
        w.f32_host("head.type_emb.weight", _normal((nt, Wd), 0.5, g, device))
        for n in ("field_norm", "option_norm"):
            w.f32_host(f"head.{n}.weight", _norm_w(Wd, g, device))
            w.f32_host(f"head.{n}.bias", _normal((Wd,), 0.02, g, device))
    w.close()
    return c


def write_decoder(out: str, seed: int = 0, device: str = "cpu", preset: dict | None = None, **over) -> dict:
    """A D13BEngine-format decoder (src/d1-3b-engine.ts): attention layers, and LFM2 short-conv layers where the
    config's layer_types say "conv" (scripts/export-3b.py:43-47: in_proj [3H, H], out_proj [H, H], conv taps
    [H, 3] f16). Returns the config."""
    c = {**(preset or DECODER_0P6B), **over}
    bits = c.pop("bits")
    L = c.pop("layers")
    c["layer_types"] = list(c.get("layer_types") or ["full_attention"] * L)[:L]
    assert len(c["layer_types"]) == L, "layer_types shorter than layers"
    H, I, heads, kv, D = c["hidden"], c["intermediate"], c["heads"], c["kv_heads"], c["head_dim"]
    g = _gen(seed, device)
    w = Writer(out, c)
    V = c["vocab"]
    emb_rows = []
    for i in range(0, V, 65536):
        emb_rows.append(_normal((min(65536, V - i), H), 0.02, g, device))
    w.quant("embed", torch.cat(emb_rows), bits)
    w.f16("final_norm", _norm_w(H, g, device))
    for i in range(L):
        p = f"layers.{i}."
        w.f16(p + "operator_norm", _norm_w(H, g, device))
        w.f16(p + "ffn_norm", _norm_w(H, g, device))
        if c["layer_types"][i] == "conv":
            w.quant(p + "in_proj", _normal((3 * H, H), 0.02, g, device), bits)
            w.quant(p + "out_proj", _normal((H, H), 0.02, g, device), bits)
            w.f16(p + "conv", _normal((H, 3), 0.5, g, device))
            w.quant(p + "w13", _normal((2 * I, H), 0.02, g, device), bits)
            w.quant(p + "w2", _normal((H, I), 0.02, g, device), bits)
            continue
        w.quant(p + "qkv", _normal(((heads + 2 * kv) * D, H), 0.02, g, device), bits)
        w.quant(p + "o_proj", _normal((H, heads * D), 0.02, g, device), bits)
        w.f16(p + "q_norm", _norm_w(D, g, device))
        w.f16(p + "k_norm", _norm_w(D, g, device))
        w.quant(p + "w13", _normal((2 * I, H), 0.02, g, device), bits)
        w.quant(p + "w2", _normal((H, I), 0.02, g, device), bits)
    w.close()
    return c


# d3-lite (scripts/export-d3.py) at a small width: Gated DeltaNet layers with a gated attention layer every
# fourth, 256-wide attention heads with RoPE on their first 64 dims, 128-wide linear heads, a code readout.
D3_LITE = dict(model="d3", hidden=1024, intermediate=3072, layers=8, heads=8, kv_heads=2, head_dim=256,
               rotary_dim=64, rope_theta=10000000.0, eps=1e-6, linear_heads=8, linear_key_dim=128,
               linear_value_dim=128, conv_kernel=4, linear_rows=4160, vocab=32768, bits=8,
               layer_types=["linear_attention"] * 3 + ["full_attention"],
               codes=[chr(65 + i) for i in range(16)], temperature=1.0)


def write_d3(out: str, seed: int = 0, device: str = "cpu", preset: dict | None = None, **over) -> dict:
    """A D3Engine-format model (src/d3-engine.ts, scripts/export-d3.py:55-101): per layer input / post norms, a
    Gated DeltaNet mixer (in [linear_rows, H] = q|k|v|z|b|a then zero rows, conv [3*LH*128, 4], A_log, dt_bias
    [LH], gnorm [128], out) or a gated attention (qkvg = q|k|v|gate heads, q / k norms [head_dim], o), a SwiGLU MLP
    (w13, w2), the final norm and an f32 readout [codes, H]. Returns the config."""
    c = {**(preset or D3_LITE), **over}
    bits = c.pop("bits")
    L = c.pop("layers")
    V = c.pop("vocab")
    c["layer_types"] = [c["layer_types"][i % len(c["layer_types"])] for i in range(L)]
    H, I, heads, kv, D, LH = c["hidden"], c["intermediate"], c["heads"], c["kv_heads"], c["head_dim"], c["linear_heads"]
    rows, QK = c["linear_rows"], LH * 128
    assert rows >= 4 * QK + 2 * LH
    g = _gen(seed, device)
    w = Writer(out, c)
    w.quant("embed", _normal((V, H), 0.02, g, device), bits)
    for i in range(L):
        p = f"layers.{i}."
        w.f16(p + "input_norm", _norm_w(H, g, device))
        w.f16(p + "post_norm", _norm_w(H, g, device))
        if c["layer_types"][i] == "linear_attention":
            win = _normal((4 * QK + 2 * LH, H), 0.02, g, device)
            w.quant(p + "in", torch.cat([win, torch.zeros(rows - win.shape[0], H, device=device)]), bits)
            w.f16(p + "conv", _normal((3 * QK, 4), 0.5, g, device))
            w.f16(p + "A_log", torch.rand(LH, generator=g, device=device) * 2 - 1.5)
            w.f16(p + "dt_bias", torch.rand(LH, generator=g, device=device) * 2 - 1)
            w.f16(p + "gnorm", _norm_w(128, g, device))
            w.quant(p + "out", _normal((H, QK), 0.02, g, device), bits)
        else:
            w.quant(p + "qkvg", _normal(((2 * heads + 2 * kv) * D, H), 0.02, g, device), bits)
            w.f16(p + "q_norm", _norm_w(D, g, device))
            w.f16(p + "k_norm", _norm_w(D, g, device))
            w.quant(p + "o", _normal((H, heads * D), 0.02, g, device), bits)
        w.quant(p + "w13", _normal((2 * I, H), 0.02, g, device), bits)
        w.quant(p + "w2", _normal((H, I), 0.02, g, device), bits)
    w.f16("final_norm", _norm_w(H, g, device))
    R = _normal((len(c["codes"]), H), 0.05, g, device).float().cpu().numpy()
    w.manifest["tensors"]["readout"] = {"dtype": "f32", "shape": list(R.shape), "offset": w.put(R.tobytes()),
                                        "bytes": int(R.nbytes)}
    w.close()
    return c


# d1-omni (scripts/export-omni.py) at a small width: an LFM2 backbone (short-conv and 64-wide attention layers) and
# a pre-norm transformer head of 64-wide heads with biases, then the marker scorer.
OMNI = dict(model="d1-omni", hidden=512, intermediate=1536, heads=8, kv_heads=2, head_dim=64, vocab=16384, eps=1e-5,
            rope_theta=1000000.0, layers=6, bits=8, layer_types=["conv", "conv", "full_attention"],
            head_layers=2, head_heads=8, head_ff=1024, ln_eps=1e-5, max_length=16384,
            temperatures={"choice:2": 1.0, "choice:3-5": 1.1, "score:3-5": 0.9, "noul:2": 1.2, "choice": 1.05})


def write_omni(out: str, seed: int = 0, device: str = "cpu", preset: dict | None = None, **over) -> dict:
    """A D1OmniEngine-format model (src/omni-engine.ts, scripts/export-omni.py:28-90): the backbone as
    write_decoder writes it, then head.type_emb [3, H], per head layer norm1 / norm2 (+ biases), in_proj [3H, H],
    out_proj, linear1 [ff, H], linear2 [H, ff] quantized with their f16 biases, and the scorer (norm + bias, fc
    [H, H] + bias, out [H], out_bias as two halves). Returns the config."""
    c = {**(preset or OMNI), **over}
    bits = c.pop("bits")
    L = c.pop("layers")
    c["layer_types"] = [c["layer_types"][i % len(c["layer_types"])] for i in range(L)]
    H, I, heads, kv, D, ff = c["hidden"], c["intermediate"], c["heads"], c["kv_heads"], c["head_dim"], c["head_ff"]
    g = _gen(seed, device)
    w = Writer(out, c)
    w.quant("embed", _normal((c["vocab"], H), 0.02, g, device), bits)
    w.f16("final_norm", _norm_w(H, g, device))
    for i in range(L):
        p = f"layers.{i}."
        w.f16(p + "operator_norm", _norm_w(H, g, device))
        w.f16(p + "ffn_norm", _norm_w(H, g, device))
        if c["layer_types"][i] == "conv":
            w.quant(p + "in_proj", _normal((3 * H, H), 0.02, g, device), bits)
            w.quant(p + "out_proj", _normal((H, H), 0.02, g, device), bits)
            w.f16(p + "conv", _normal((H, 3), 0.5, g, device))
        else:
            w.quant(p + "qkv", _normal(((heads + 2 * kv) * D, H), 0.02, g, device), bits)
            w.quant(p + "o_proj", _normal((H, heads * D), 0.02, g, device), bits)
            w.f16(p + "q_norm", _norm_w(D, g, device))
            w.f16(p + "k_norm", _norm_w(D, g, device))
        w.quant(p + "w13", _normal((2 * I, H), 0.02, g, device), bits)
        w.quant(p + "w2", _normal((H, I), 0.02, g, device), bits)
    _write_head(w, c, g, device, bits)
    w.close()
    return c


# Laya (scripts/export-laya.py) at a small width: a ModernBERT encoder (bias-free LayerNorms, every third layer
# global, the others a +-64-token window) and d1-omni's head.
LAYA = dict(model="laya", hidden=512, intermediate=1024, heads=8, layers=6, vocab=16384, bits=8,
            layer_types=["full_attention", "sliding_attention", "sliding_attention"], window=64,
            rope_theta={"full_attention": 160000.0, "sliding_attention": 10000.0}, eps=1e-5, head_layers=2,
            head_heads=8, head_ff=1024, ln_eps=1e-5, max_len=512, head_max_len=192,
            temperatures={"choice:3-5": 1.1, "noul:2": 0.9, "choice": 1.0})


def _write_head(w, c, g, device, bits):
    """d1-omni's decision head tensors (scripts/export-omni.py:68-89, scripts/export-laya.py:84-103)."""
    H, ff = c["hidden"], c["head_ff"]
    w.f16("head.type_emb", _normal((3, H), 0.5, g, device))
    for i in range(c["head_layers"]):
        p = f"head.{i}."
        w.quant(p + "in_proj", _normal((3 * H, H), 0.03, g, device), bits)
        w.f16(p + "in_proj_bias", _normal((3 * H,), 0.05, g, device))
        w.quant(p + "out_proj", _normal((H, H), 0.03, g, device), bits)
        w.f16(p + "out_proj_bias", _normal((H,), 0.05, g, device))
        w.quant(p + "linear1", _normal((ff, H), 0.03, g, device), bits)
        w.f16(p + "linear1_bias", _normal((ff,), 0.05, g, device))
        w.quant(p + "linear2", _normal((H, ff), 0.03, g, device), bits)
        w.f16(p + "linear2_bias", _normal((H,), 0.05, g, device))
        for nm in ("norm1", "norm2"):
            w.f16(p + nm, _norm_w(H, g, device))
            w.f16(p + nm + "_bias", _normal((H,), 0.05, g, device))
    w.f16("scorer.norm", _norm_w(H, g, device))
    w.f16("scorer.norm_bias", _normal((H,), 0.05, g, device))
    w.quant("scorer.fc", _normal((H, H), 0.04, g, device), bits)
    w.f16("scorer.fc_bias", _normal((H,), 0.05, g, device))
    w.f16("scorer.out", _normal((H,), 0.1, g, device))
    w.f16("scorer.out_bias", torch.tensor([0.1, 0.0]))


def write_laya(out: str, seed: int = 0, device: str = "cpu", preset: dict | None = None, **over) -> dict:
    """A LayaEngine-format model (src/laya-engine.ts, scripts/export-laya.py:54-104): embed, embed_norm, per layer
    attn_norm (not layer 0), mlp_norm, qkv [3H, H], o, wi [2I, H] (gate | up), wo, final_norm, then the head.
    Returns the config."""
    c = {**(preset or LAYA), **over}
    bits = c.pop("bits")
    V = c.pop("vocab")
    L = c["layers"]
    c["layer_types"] = [c["layer_types"][i % len(c["layer_types"])] for i in range(L)]
    H, I = c["hidden"], c["intermediate"]
    g = _gen(seed, device)
    w = Writer(out, c)
    w.quant("embed", _normal((V, H), 0.5, g, device), bits)
    w.f16("embed_norm", _norm_w(H, g, device))
    for i in range(L):
        p = f"layers.{i}."
        if i > 0:
            w.f16(p + "attn_norm", _norm_w(H, g, device))
        w.f16(p + "mlp_norm", _norm_w(H, g, device))
        w.quant(p + "qkv", _normal((3 * H, H), 0.03, g, device), bits)
        w.quant(p + "o", _normal((H, H), 0.03, g, device), bits)
        w.quant(p + "wi", _normal((2 * I, H), 0.03, g, device), bits)
        w.quant(p + "wo", _normal((H, I), 0.03, g, device), bits)
    w.f16("final_norm", _norm_w(H, g, device))
    _write_head(w, c, g, device, bits)
    w.close()
    return c


PRESETS = {"encoder": ENCODER_EG300M, "decoder": DECODER_0P6B, "encoder-eg2": ENCODER_EG2,
           "decoder-lfm2": DECODER_LFM2, "d3": D3_LITE, "omni": OMNI, "laya": LAYA}


def cached_model(kind: str, root: str | None = None, device: str = "cpu", **over) -> str:
    """Writes (once) and returns the directory of a synthetic model: kind "encoder" / "decoder" (the BASELINE
    architectures) or "encoder-eg2" / "decoder-lfm2" / "d3" / "omni" / "laya" (the reference's own engines')."""
    root = root or os.environ.get("DECISION_B200_MODELS") or os.path.join(
        os.environ.get("TMPDIR", "/tmp"), "decision_b200_models")
    key = kind + "-" + "-".join(f"{k}={over[k]}" for k in sorted(over))
    out = os.path.join(root, key.replace("/", "_"))
    if not os.path.exists(os.path.join(out, "manifest.json")):
        tmp = out + f".tmp{os.getpid()}"
        writer = (write_encoder if kind.startswith("encoder") else write_d3 if kind == "d3" else
                  write_omni if kind == "omni" else write_laya if kind == "laya" else write_decoder)
        writer(tmp, device=device, preset=PRESETS[kind], **over)
        os.makedirs(root, exist_ok=True)
        try:
            os.rename(tmp, out)
        except OSError:
            pass  # another process finished first
    return out


def write_tokenizer(out: str, texts, vocab_size: int, bos: str = "<bos>", eos: str = "<eos>",
                    extra=("<|im_start|>", "<|im_end|>")) -> dict:
    """A word-level tokenizer.json + tokenizer_config.json (Hugging Face's format, as the reference's exports ship
    them) whose vocabulary holds every word and punctuation run of `texts`, single letters, digits, yes/no and the
    special tokens, with ids below vocab_size. For tests of the text path: the ids are arbitrary, the interfaces
    (encode without special tokens, special tokens that match inside text, ids by token) are the real ones."""
    import re

    from tokenizers import Tokenizer, models, pre_tokenizers
    words = ["<pad>", bos, eos, "<unk>", *extra]
    seen = set(words)
    base = [chr(c) for c in range(65, 91)] + [chr(c) for c in range(97, 123)] + [str(i) for i in range(100)] + \
        ["yes", "Yes", "YES", "no", "No", "NO"]
    for t in list(base) + [w for t in texts for w in re.findall(r"\w+|[^\w\s]+", t)]:
        if t not in seen:
            seen.add(t)
            words.append(t)
    if len(words) > vocab_size:
        raise ValueError(f"tokenizer: {len(words)} words exceed the vocabulary of {vocab_size}")
    tok = Tokenizer(models.WordLevel({w: i for i, w in enumerate(words)}, unk_token="<unk>"))
    tok.pre_tokenizer = pre_tokenizers.Whitespace()
    tok.add_special_tokens([bos, eos, *extra])
    os.makedirs(out, exist_ok=True)
    tok.save(os.path.join(out, "tokenizer.json"))
    cfg = {"bos_token": bos, "eos_token": eos, "pad_token": "<pad>", "unk_token": "<unk>"}
    with open(os.path.join(out, "tokenizer_config.json"), "w") as f:
        json.dump(cfg, f)
    return cfg


# ---------------------------------------------------------------- inputs

def config1_inputs(seed: int = 0, M: int = 256, N: int = 1152, K: int = 768, bits: int = 8):
    """BASELINE config 1 (and the sweep): X [M, K] f16 ~N(0,1); codes uniform over what the reference's quantizers
    emit, stored + Z: int8 in [-127, 127] for q8 (quantize8 clamps to +-127), [-8, 7] for q4 (quantize4 clamps to
    [-8, 7], scripts/export_common.py:76, so nibble 0 occurs); f16 scales ~U(0.001, 0.02) per 32 along K."""
    rng = np.random.default_rng(seed)
    X = rng.standard_normal((M, K)).astype(np.float16)
    if bits == 8:
        codes = (rng.integers(-127, 128, (N, K)) + 128).astype(np.uint8)
    else:
        c = (rng.integers(-8, 8, (N, K)) + 8).astype(np.uint8)
        codes = (c[:, 0::2] | (c[:, 1::2] << 4)).astype(np.uint8)
    S = rng.uniform(0.001, 0.02, (N, K // BLOCK)).astype(np.float16)
    return X, codes, S


def encoder_requests(n: int, tokens: int, vocab: int, seed: int = 0):
    """n texts of `tokens` ids uniform over the vocabulary."""
    rng = np.random.default_rng(seed)
    return [rng.integers(0, vocab, tokens).astype(np.int32).tolist() for _ in range(n)]


def decoder_trees(n: int, tokens: int, vocab: int, questions: int = 3, answers: int = 10, seed: int = 0):
    """n D13BEngine trees of `tokens` tokens each: a trunk plus `questions` branches of 4 tokens, each read out
    over a fixed answer subset of `answers` ids split into options of 2 forms."""
    rng = np.random.default_rng(seed)
    answer_ids = rng.integers(0, vocab, answers).astype(int).tolist()
    groups = [answer_ids[i:i + 2] for i in range(0, answers, 2)]
    trees = []
    for _ in range(n):
        trunk = rng.integers(0, vocab, tokens - 4 * questions).astype(int).tolist()
        branches = [rng.integers(0, vocab, 4).astype(int).tolist() for _ in range(questions)]
        trees.append({"trunk": trunk, "branches": branches, "groups": [groups] * questions})
    return trees
