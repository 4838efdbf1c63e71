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


def _gen(seed: int, device: str):
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return g


def _normal(shape, std, g, device):
    return torch.randn(*shape, generator=g, device=device) * std


def _norm_w(n, g, device):
    return 1.0 + 0.1 * torch.randn(n, generator=g, device=device)


def write_encoder(out: str, seed: int = 0, device: str = "cpu", **over) -> dict:
    """An Eg2Engine-format encoder (src/eg2-engine.ts) without per-layer embeddings. Returns the config."""
    c = {**ENCODER_EG300M, **over}
    bits = c.pop("bits")
    H, I, L, heads = c["hidden"], c["intermediate"], c["layers"], c["heads"]
    c["layer_types"] = list(c["layer_types"])[:L]
    c["layer_scalars"] = [1.0] * L
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
    w.f16("final_norm", _norm_w(H, g, device))
    w.close()
    return c


def write_decoder(out: str, seed: int = 0, device: str = "cpu", **over) -> dict:
    """A D13BEngine-format decoder (src/d1-3b-engine.ts) with attention layers only. Returns the config."""
    c = {**DECODER_0P6B, **over}
    bits = c.pop("bits")
    L = c.pop("layers")
    c["layer_types"] = ["full_attention"] * L
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
        w.quant(p + "qkv", _normal(((heads + 2 * kv) * D, H), 0.02, g, device), bits)
        w.quant(p + "o_proj", _normal((H, heads * D), 0.02, g, device), bits)
        w.f16(p + "q_norm", _norm_w(D, g, device))
        w.f16(p + "k_norm", _norm_w(D, g, device))
        w.quant(p + "w13", _normal((2 * I, H), 0.02, g, device), bits)
        w.quant(p + "w2", _normal((H, I), 0.02, g, device), bits)
    w.close()
    return c


def cached_model(kind: str, root: str | None = None, device: str = "cpu", **over) -> str:
    """Writes (once) and returns the directory of a synthetic model: kind "encoder" or "decoder"."""
    root = root or os.environ.get("DECISION_B200_MODELS") or os.path.join(
        os.environ.get("TMPDIR", "/tmp"), "decision_b200_models")
    key = kind + "-" + "-".join(f"{k}={over[k]}" for k in sorted(over))
    out = os.path.join(root, key.replace("/", "_"))
    if not os.path.exists(os.path.join(out, "manifest.json")):
        tmp = out + f".tmp{os.getpid()}"
        (write_encoder if kind == "encoder" else write_decoder)(tmp, device=device, **over)
        os.makedirs(root, exist_ok=True)
        try:
            os.rename(tmp, out)
        except OSError:
            pass  # another process finished first
    return out


# ---------------------------------------------------------------- inputs

def config1_inputs(seed: int = 0, M: int = 256, N: int = 1152, K: int = 768, bits: int = 8):
    """BASELINE config 1 (and the sweep): X [M, K] f16 ~N(0,1); codes uniform in [-Z+1, Z-1] stored + Z (int8 in
    [-127, 127] for q8, [-7, 7] for q4); f16 scales ~U(0.001, 0.02) per 32 along K."""
    rng = np.random.default_rng(seed)
    X = rng.standard_normal((M, K)).astype(np.float16)
    if bits == 8:
        codes = (rng.integers(-127, 128, (N, K)) + 128).astype(np.uint8)
    else:
        c = (rng.integers(-7, 8, (N, K)) + 8).astype(np.uint8)
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
