"""Host logic without a GPU: pass packing, request sharding, the forest, questions and answers, the weights
format round trip, and the oracle against plain numpy definitions."""
import json
import math
import os

import numpy as np
import pytest


def test_passes_pack_whole_requests(pkg):
    # src/d1.ts:130-133: at least one request per pass, then add while the budget holds
    assert pkg.passes([3, 3, 3, 9, 1], 6) == [(0, 2), (2, 3), (3, 4), (4, 5)]
    assert pkg.passes([10], 4) == [(0, 1)]
    assert pkg.passes([], 4) == []
    assert pkg.passes([256] * 64, 16384) == [(0, 64)]
    assert pkg.passes([256] * 64, 8192) == [(0, 32), (32, 64)]


@pytest.mark.parametrize("n", [1, 2, 3, 4, 8])
def test_shard_is_contiguous_and_balanced(pkg, n):
    rng = np.random.default_rng(n)
    sizes = rng.integers(1, 500, 97).tolist()
    sh = pkg.shard(sizes, n)
    assert len(sh) == n and sh[0][0] == 0 and sh[-1][1] == len(sizes)
    assert all(a[1] == b[0] for a, b in zip(sh, sh[1:]))
    loads = [sum(sizes[a:b]) for a, b in sh]
    assert max(loads) <= sum(sizes) / n + max(sizes)


def test_shard_more_workers_than_requests(pkg):
    sh = pkg.shard([5, 5], 4)
    assert sh[-1][1] == 2 and sum(b - a for a, b in sh) == 2


def test_forest_matches_reference_mask(pkg):
    """The key ranges encode the reference's tree mask (src/kernels.ts:135): a trunk token sees earlier trunk
    tokens; a branch token sees the whole trunk and its own branch up to itself."""
    trees = [{"trunk": [1, 2, 3], "branches": [[4, 5], [6]], "groups": [[[7], [8]], [[9, 10]]]},
             {"trunk": [11], "branches": [[12, 13, 14]], "groups": [[[15]]]}]
    ids, pos, rng, leaves, leaf_ids = pkg.forest(trees)
    assert ids.tolist() == [1, 2, 3, 4, 5, 6, 11, 12, 13, 14]
    assert pos.tolist() == [0, 1, 2, 3, 4, 3, 0, 1, 2, 3]
    assert leaves.tolist() == [4, 5, 9]
    assert leaf_ids == [[7, 8], [9, 10], [15]]
    # brute-force mask from the reference's meta (start, end, branch, offset)
    meta = [(0, 6, -1, 0), (0, 6, -1, 1), (0, 6, -1, 2), (0, 6, 0, 3), (0, 6, 0, 4), (0, 6, 1, 3),
            (6, 10, -1, 0), (6, 10, 0, 1), (6, 10, 0, 2), (6, 10, 0, 3)]
    for t, mt in enumerate(meta):
        for k in range(mt[0], mt[1]):
            mk = meta[k]
            ok = (mk[2] == -1 and (mt[2] != -1 or mk[3] <= mt[3])) or (mk[2] == mt[2] and mt[2] != -1 and mk[3] <= mt[3])
            r = rng[t]
            vis = r[0] <= k < r[1] or r[2] <= k < r[3]
            assert ok == vis, (t, k)


def _forest_loops(trees):
    """A per-token restatement of the packed forest (the reference's loops, src/d1-3b-engine.ts:46-68)."""
    ids, pos, rng, leaves, leaf_ids = [], [], [], [], []
    for tr in trees:
        start, p = len(ids), len(tr["trunk"])
        for i, tok in enumerate(tr["trunk"]):
            ids.append(tok), pos.append(i), rng.append((start, start + i + 1, 0, 0))
        for b, br in enumerate(tr["branches"]):
            bs = len(ids)
            for o, tok in enumerate(br):
                ids.append(tok), pos.append(p + o), rng.append((start, start + p, bs, len(ids)))
            leaves.append(len(ids) - 1)
            leaf_ids.append([i for g in tr["groups"][b] for i in g])
    return ids, pos, rng, leaves, leaf_ids


def test_forest_vectorised_matches_loops(pkg):
    rng_ = np.random.default_rng(5)
    trees = []
    for n in range(40):
        p = int(rng_.integers(0, 40)) if n else 0  # the first tree has an empty trunk
        nb = int(rng_.integers(1, 4))
        trees.append({"trunk": rng_.integers(0, 1000, p).tolist(),
                      "branches": [rng_.integers(0, 1000, int(rng_.integers(1, 6))).tolist() for _ in range(nb)],
                      "groups": [[[int(x) for x in rng_.integers(0, 1000, int(rng_.integers(1, 3)))]
                                  for _ in range(int(rng_.integers(2, 5)))] for _ in range(nb)]})
    ids, pos, rng, leaves, leaf_ids = pkg.forest(trees)
    # the C ABI reads these as int32 arrays
    assert all(a.dtype == np.int32 and a.flags.c_contiguous for a in (ids, pos, rng, leaves))
    ref = _forest_loops(trees)
    assert ids.tolist() == ref[0] and pos.tolist() == ref[1] and [tuple(r) for r in rng.tolist()] == ref[2]
    assert leaves.tolist() == ref[3] and leaf_ids == ref[4]
    # readout: each option's best form, per tree and question, as a loop over the logits would find it
    from decision_js_b200.decision import readout_scores
    n = max(len(g) for g in leaf_ids)
    out = rng_.standard_normal((len(leaves), n)).astype(np.float32)
    got = readout_scores(trees, out)
    leaf = 0
    for tr, per_q in zip(trees, got):
        assert len(per_q) == len(tr["groups"])
        for groups, s in zip(tr["groups"], per_q):
            j, want = 0, []
            for g in groups:
                want.append(float(out[leaf, j:j + len(g)].max()))
                j += len(g)
            assert s == want
            leaf += 1


def test_questions(pkg):
    from decision_js_b200.questions import QuestionError
    with pytest.raises(QuestionError, match="decision.js: a question is an object"):
        pkg.check_question({"type": "noul"})
    with pytest.raises(QuestionError) as e:
        pkg.check_question({"type": "x", "instructions": ""})
    assert str(e.value) == 'decision.js: question type must be noul, choice or score, got "x"'  # JSON.stringify
    with pytest.raises(QuestionError, match="at least two options"):
        pkg.check_question({"type": "choice", "instructions": "", "criteria": ["a", "b"]})  # a list is not a map
    with pytest.raises(QuestionError, match="noul criteria are optional"):
        pkg.check_question({"type": "noul", "instructions": "", "criteria": ["yes"]})
    with pytest.raises(QuestionError, match="at least two options"):
        pkg.check_question({"type": "choice", "instructions": "", "criteria": {"a": 1}})
    with pytest.raises(QuestionError, match="2 to 10 level"):
        pkg.check_question({"type": "score", "instructions": "", "criteria": [1]})
    a = pkg.answer({"type": "choice", "instructions": "", "criteria": {"x": 1, "y": 2}}, [0.2, 0.8])
    assert a["choice"] == "y" and a["confidence"] == 0.8
    s = pkg.answer({"type": "score", "instructions": "", "criteria": ["lo", "mid", "hi"]}, [0.25, 0.25, 0.5])
    assert math.isclose(s["score"], 1.25) and s["legend"] == {"0": "lo", "1": "mid", "2": "hi"}
    assert pkg.answer({"type": "noul", "instructions": ""}, [0.9, 0.1]) == {"type": "noul", "noul": 0.9}
    p = pkg.softmax([1.0, 2.0, 3.0])
    assert math.isclose(sum(p), 1.0) and p[2] > p[1] > p[0]


def test_weights_round_trip(pkg, oracle, tmp_path):
    """A synthetic model in the reference's layout: 256-byte aligned tensors, scales after codes, a manifest the
    oracle's independent reader understands, codes that dequantize back near the weights."""
    from decision_js_b200 import synth
    c = synth.write_decoder(str(tmp_path), layers=1, vocab=512, hidden=256, intermediate=512, heads=4, kv_heads=2,
                            head_dim=64)
    m = json.load(open(tmp_path / "manifest.json"))
    assert m["format"] == "d1.js/1" and m["bytes"] == os.path.getsize(tmp_path / "weights.bin")
    for t in m["tensors"].values():
        assert t["offset"] % 256 == 0
        if t["dtype"] in ("q4", "q8"):
            assert t["scales"] % 256 == 0 and t["scales_bytes"] == t["shape"][0] * t["shape"][1] // 32 * 2
    w = oracle.Weights(str(tmp_path))
    codes, sc, N, K, bits = w.q("layers.0.qkv")
    assert (N, K, bits) == ((4 + 4) * 64, 256, 8)
    deq = synth.dequantize(codes, sc.view(np.float16), N, K, bits).astype(np.float32)
    assert np.abs(deq).max() < 0.2 and np.abs(deq).mean() > 0.005


def test_oracle_attention_against_numpy(oracle):
    rng = np.random.default_rng(0)
    T, heads, kv, D = 12, 4, 2, 64
    Z = rng.standard_normal((T, (heads + 2 * kv) * D)).astype(np.float16)
    r = np.array([(0, t + 1, 0, 0) for t in range(T)], np.int32)
    got = oracle.attention(Z, r, heads, kv, D, 0.125).view(np.float16).astype(np.float32)
    Zf = Z.astype(np.float32)
    for h in range(heads):
        g = h // (heads // kv)
        q = Zf[:, h * D:(h + 1) * D] * 0.125
        k = Zf[:, (heads + g) * D:(heads + g + 1) * D]
        v = Zf[:, (heads + kv + g) * D:(heads + kv + g + 1) * D]
        s = q @ k.T
        s[np.triu_indices(T, 1)] = -np.inf
        p = np.exp(s - s.max(1, keepdims=True))
        p /= p.sum(1, keepdims=True)
        assert np.abs(got[:, h * D:(h + 1) * D] - p @ v).max() < 2e-3


def test_oracle_matmul_against_numpy(oracle, pkg):
    from decision_js_b200 import synth
    X, codes, S = synth.config1_inputs(seed=0, M=64, N=96, K=128, bits=4)
    got = oracle.qmatmul(X, codes, S, 96, 128, 4).view(np.float16).astype(np.float32)
    W = synth.dequantize(codes, S, 96, 128, 4).astype(np.float32)
    ref = X.astype(np.float32) @ W.T
    assert np.abs(got - ref).max() <= 1e-3 * np.abs(ref).max()


def test_oracle_rmsnorm_against_numpy(oracle):
    rng = np.random.default_rng(1)
    X = rng.standard_normal((5, 64)).astype(np.float16)
    W = (1 + 0.1 * rng.standard_normal(64)).astype(np.float16)
    _, O = oracle.add_rmsnorm(X, None, W, False, 1e-6)
    x = X.astype(np.float32)
    ref = x / np.sqrt((x * x).mean(1, keepdims=True) + 1e-6) * W.astype(np.float32)
    assert np.abs(O.view(np.float16).astype(np.float32) - ref).max() < 4e-3


# Numpy restatements of the remaining oracle kernels, written from the WGSL the oracle cites, in float64 with f16
# rounding exactly where the WGSL stores f16. Tolerances: one f16 rounding of the output (the oracle computes in f32).
def _f16_close(got, ref, what, rtol=2e-3, afrac=1e-3, atol=0.0):
    """rtol of each value, plus afrac of the largest (outputs that cancel, as RoPE's a·c − b·s), plus atol."""
    got = np.asarray(got, np.float32)
    ref = np.asarray(ref, np.float64)
    err = np.abs(got - ref)
    tol = rtol * np.abs(ref) + afrac * max(np.abs(ref).max(), 1e-6) + atol
    assert (err <= tol).all(), (what, float(err.max()))


def _h(a):
    return np.asarray(a).view(np.float16).astype(np.float64)


@pytest.mark.parametrize("norm2", [False, True])
def test_oracle_sandwich_against_numpy(oracle, norm2):
    """SANDWICH (src/eg2-kernels.ts:18-48): x = f16((x + rms(y)·w1)·scale); O = f16(rms(x)·w2) over the stored x."""
    rng = np.random.default_rng(2)
    T, H, eps, scale = 7, 768, 1e-6, 0.75
    X = rng.standard_normal((T, H)).astype(np.float16)
    Y = (3 * rng.standard_normal((T, H))).astype(np.float16)
    W1 = (1 + 0.1 * rng.standard_normal(H)).astype(np.float16)
    W2 = (1 + 0.1 * rng.standard_normal(H)).astype(np.float16)
    Xn, O = oracle.sandwich(X, Y, W1, W2 if norm2 else None, eps, scale)
    x, y = X.astype(np.float64), Y.astype(np.float64)
    iy = 1 / np.sqrt((y * y).mean(1, keepdims=True) + eps)
    xr = ((x + y * iy * W1.astype(np.float64)) * scale).astype(np.float16)
    _f16_close(_h(Xn), xr, "residual")
    if norm2:
        a = xr.astype(np.float64)
        ix = 1 / np.sqrt((a * a).mean(1, keepdims=True) + eps)
        _f16_close(_h(O), a * ix * W2.astype(np.float64), "O")
    else:
        assert O is None


@pytest.mark.parametrize("D,heads,kv,vnorm", [(64, 4, 2, 0), (128, 3, 1, 0), (256, 3, 1, 1)])
def test_oracle_qkv_norm_rope_against_numpy(oracle, D, heads, kv, vnorm):
    """QK_NORM_ROPE (src/kernels.ts:87-112) / QKV_NORM_ROPE (src/eg2-kernels.ts:53-96): per-head RMSNorm (q by qn,
    k by kn, v plainly when vnorm, else untouched), then rotate-half RoPE on q and k at the token's position."""
    rng = np.random.default_rng(3 + D)
    T, eps, theta = 6, 1e-6, 10000.0
    per = heads + 2 * kv
    Z = (2 * rng.standard_normal((T, per * D))).astype(np.float16)
    qn = (1 + 0.1 * rng.standard_normal(D)).astype(np.float16)
    kn = (1 + 0.1 * rng.standard_normal(D)).astype(np.float16)
    pos = np.array([0, 1, 5, 17, 100, 511], np.int32)
    got = oracle.qkv_norm_rope(Z, qn, kn, pos, heads, kv, D, eps, theta, vnorm)
    z = Z.astype(np.float64).reshape(T, per, D)
    ref = z.copy()
    inv_freq = theta ** (-np.arange(0, D, 2, dtype=np.float64) / D)  # theta^(-2d/D), d < D/2
    for h in range(per):
        isq, isk = h < heads, heads <= h < heads + kv
        if not (isq or isk or vnorm):
            continue
        v = z[:, h] / np.sqrt((z[:, h] ** 2).mean(1, keepdims=True) + eps)
        if isq:
            v = v * qn.astype(np.float64)
        elif isk:
            v = v * kn.astype(np.float64)
        if isq or isk:
            ang = pos[:, None].astype(np.float64) * inv_freq[None, :]
            a, b = v[:, :D // 2], v[:, D // 2:]
            v = np.concatenate([a * np.cos(ang) - b * np.sin(ang), b * np.cos(ang) + a * np.sin(ang)], 1)
        ref[:, h] = v
    g = _h(got).reshape(T, per, D)
    _f16_close(g, ref, "qkv")
    if not vnorm:  # v heads untouched, bit for bit
        assert np.array_equal(got.reshape(T, per, D)[:, heads + kv:].view(np.uint16),
                              Z.reshape(T, per, D)[:, heads + kv:].view(np.uint16))


@pytest.mark.parametrize("act", [0, 1])
def test_oracle_glu_against_numpy(oracle, act):
    """SILU_MUL (src/kernels.ts:49-60), GELU_MUL (src/eg2-kernels.ts:166-177): h = f16(act(gate) · up) over a fused
    gate|up row; GELU is the tanh approximation (tanh written through exp with the argument clamped to ±15)."""
    rng = np.random.default_rng(4)
    T, I = 5, 384
    A = (3 * rng.standard_normal((T, 2 * I))).astype(np.float16)
    A[0, :4] = np.array([0, -20, 20, 1e-3], np.float16)  # zero, both saturation ends, a tiny gate
    got = oracle.glu(A, I, act)
    a, b = A[:, :I].astype(np.float64), A[:, I:].astype(np.float64)
    if act == 0:
        g = a / (1 + np.exp(-a))
    else:
        g = 0.5 * a * (1 + np.tanh(np.sqrt(2 / np.pi) * (a + 0.044715 * a ** 3)))
    # a product of two terms, nothing cancels: one f16 rounding of each value (f32 keeps 1 + tanh to ~1e-7 absolute)
    _f16_close(_h(got), g * b, "glu", rtol=1e-3, afrac=0.0, atol=1e-5)


@pytest.mark.parametrize("bits", [8, 4])
def test_oracle_gather_against_numpy(oracle, pkg, bits):
    """GATHER_Q8 / GATHER_Q4 (src/kernels.ts:7-21, 293-296): rows of the dequantized embedding, bit for bit."""
    from decision_js_b200 import synth
    V, H = 50, 256
    _, codes, S = synth.config1_inputs(seed=5, M=1, N=V, K=H, bits=bits)
    ids = np.array([0, 49, 7, 7, 23], np.int32)
    got = oracle.gather(ids, codes, S, H, bits)
    ref = synth.dequantize(codes, S, V, H, bits)[ids]
    assert np.array_equal(got.view(np.uint16), ref.view(np.uint16))


@pytest.mark.parametrize("proj", [False, True])
def test_oracle_pool_against_numpy(oracle, proj):
    """POOL_PROJECT (src/eg2-kernels.ts:204-228): the f32 mean of each sequence's rows, then the optional
    projection by W [N, H]."""
    rng = np.random.default_rng(6)
    T, H, N = 13, 256, 96
    X = rng.standard_normal((T, H)).astype(np.float16)
    seqs = np.array([[0, 1], [1, 9], [9, 13]], np.int32)
    W = (0.05 * rng.standard_normal((N, H))).astype(np.float16) if proj else None
    got = oracle.pool(X, seqs, W)
    x = X.astype(np.float64)
    mean = np.stack([x[a:b].mean(0) for a, b in seqs])
    ref = mean @ W.astype(np.float64).T if proj else mean
    assert np.abs(got - ref).max() <= 1e-5 * max(np.abs(ref).max(), 1.0)


@pytest.mark.parametrize("bits", [8, 4])
def test_oracle_leaf_logits_against_numpy(oracle, pkg, bits):
    """LEAF_LOGITS (src/kernels.ts:150-185): the final RMSNorm at each readout row (f32, not rounded), then the
    dot with the tied embedding rows of the row's ids, dequantized in f32 ((code − Z)·scale, no f16 rounding)."""
    from decision_js_b200 import synth
    rng = np.random.default_rng(7)
    V, H, T, eps = 40, 512, 9, 1e-6
    _, codes, S = synth.config1_inputs(seed=8, M=1, N=V, K=H, bits=bits)
    X = (2 * rng.standard_normal((T, H))).astype(np.float16)
    W = (1 + 0.1 * rng.standard_normal(H)).astype(np.float16)
    leaves = np.array([8, 3, 0], np.int32)
    ids = rng.integers(0, V, (3, 10)).astype(np.int32)
    got = oracle.leaf_logits(X, leaves, W, ids, codes, S, bits, eps)
    if bits == 8:
        c = codes.reshape(V, H).astype(np.float64) - 128
    else:
        b = codes.reshape(V, H // 2)
        c = np.empty((V, H))
        c[:, 0::2], c[:, 1::2] = b & 15, b >> 4
        c -= 8
    E = c * np.repeat(S.astype(np.float64), 32, axis=1)  # exact in f64: no f16 rounding of the weight
    x = X.astype(np.float64)[leaves]
    normed = x / np.sqrt((x * x).mean(1, keepdims=True) + eps) * W.astype(np.float64)
    ref = np.einsum("lh,lih->li", normed, E[ids])
    assert np.abs(got - ref).max() <= 1e-4 * np.abs(ref).max()


class _FakeModel:
    """Stands in for one device's context + weights (no GPU): records close() calls."""
    closed = []

    def __init__(self, base, device):
        if device == 1:
            from decision_js_b200._lib import DC_ENOMEM, DecisionError
            raise DecisionError(DC_ENOMEM, "decision.js: cannot allocate (fake)")
        self.device, self.kind = device, "eg2"
        self.embed_dim = 3

    def encoder_pass(self, seqs):
        return np.full((len(seqs), 4), float(self.device), np.float32)

    def cfg(self, key, default=None):
        return {"embed_dim": 3.0}.get(key, default)

    def close(self):
        _FakeModel.closed.append(self.device)


def test_load_failure_frees_the_replicas_that_loaded(pkg, tmp_path, monkeypatch):
    """A multi-device load where one device fails frees the weights already uploaded to the others and raises the
    failure (host-side injection: the fake model of device 1 raises DC_ENOMEM)."""
    from decision_js_b200 import decision as dmod
    from decision_js_b200._lib import DC_ENOMEM, DecisionError
    (tmp_path / "manifest.json").write_text("{}")
    monkeypatch.setattr(dmod, "_Model", _FakeModel)
    _FakeModel.closed = []
    with pytest.raises(DecisionError) as e:
        dmod.Decision.load(str(tmp_path), devices=[0, 1, 2])
    assert e.value.code == DC_ENOMEM
    assert sorted(_FakeModel.closed) == [0, 2]


def test_destroy_then_call_raises(pkg, tmp_path, monkeypatch):
    from decision_js_b200 import decision as dmod
    from decision_js_b200._lib import DC_EINVAL, DecisionError
    (tmp_path / "manifest.json").write_text("{}")
    monkeypatch.setattr(dmod, "_Model", _FakeModel)
    _FakeModel.closed = []
    d = dmod.Decision.load(str(tmp_path), devices=[0, 2])
    assert len(d.embed_raw([[1, 2, 3]] * 5)) == 5
    assert d.embed_raw([]) == [] and d.embed([]) == []  # no pass, no device work
    d.destroy()
    d.destroy()  # idempotent
    assert sorted(_FakeModel.closed) == [0, 2]
    with pytest.raises(DecisionError) as e:
        d.embed_raw([[1, 2, 3]])
    assert e.value.code == DC_EINVAL and "destroyed" in str(e.value)


def test_model_without_a_device_fails_cleanly(pkg, tmp_path):
    """On a machine without a GPU the per-device model raises DC_ECUDA from dc_init and leaves nothing to free."""
    from decision_js_b200 import decision as dmod
    from decision_js_b200._lib import DC_ECUDA, DecisionError, device_count
    if device_count() > 0:
        pytest.skip("a device is present")
    with pytest.raises(DecisionError) as e:
        dmod._Model(str(tmp_path), 0)
    assert e.value.code == DC_ECUDA


def test_decoder_pass_host_path_with_a_fake_library(pkg, monkeypatch):
    """The decoder pass's host side through a stand-in for dc_forward_decoder that reads the arrays through the raw
    pointers, as the C side does: int32 ids / positions / ranges / readout rows, padded readout ids [L, n], and
    logits written back into `out`. Each logit is its id + 0.001 x its readout row, so the option scores show that
    every option took the max over its own group's ids of its own readout."""
    import ctypes
    from decision_js_b200 import decision as dmod

    class FakeLib:
        def dc_forward_decoder(self, h, ids, pos, rng, T, leaves, flat, L, n, out):
            i32 = lambda p, k: np.ctypeslib.as_array((ctypes.c_int32 * k).from_address(p))
            f = i32(flat, L * n).reshape(L, n)
            r = i32(rng, 4 * T).reshape(T, 4)
            lv = i32(leaves, L)
            assert (r[:, 1] > r[:, 0]).all() and (lv < T).all() and len(i32(ids, T)) == T and len(i32(pos, T)) == T
            o = np.ctypeslib.as_array((ctypes.c_float * (L * n)).from_address(out)).reshape(L, n)
            o[:] = f + 0.001 * np.arange(L)[:, None]
            return 0

    monkeypatch.setattr(dmod, "lib", lambda: FakeLib())
    m = object.__new__(dmod._Model)
    m.h = None
    rs = np.random.default_rng(11)
    trees = []
    for _ in range(5):
        nb = int(rs.integers(1, 4))
        trees.append({"trunk": rs.integers(0, 500, int(rs.integers(1, 30))).tolist(),
                      "branches": [rs.integers(0, 500, int(rs.integers(1, 5))).tolist() for _ in range(nb)],
                      "groups": [[rs.integers(1, 500, int(rs.integers(1, 4))).tolist()
                                  for _ in range(int(rs.integers(2, 5)))] for _ in range(nb)]})
    got = m.decoder_pass(trees)
    leaf = 0
    for tr, per_q in zip(trees, got):
        for groups, scores in zip(tr["groups"], per_q):
            want = [max(g) + 0.001 * leaf for g in groups]
            assert np.allclose(scores, want, atol=1e-4), (scores, want)
            leaf += 1


def test_encoder_pass_host_path_with_a_fake_library(pkg, monkeypatch):
    """The encoder pass's host side through a stand-in for dc_forward_encoder that reads ids and [start, end) bounds
    through the raw pointers and writes, per sequence, the sum of its ids and its length."""
    import ctypes
    from decision_js_b200 import decision as dmod

    class FakeLib:
        def dc_forward_encoder(self, h, ids, bounds, T, S, out):
            i = np.ctypeslib.as_array((ctypes.c_int32 * T).from_address(ids))
            b = np.ctypeslib.as_array((ctypes.c_int32 * (2 * S)).from_address(bounds)).reshape(S, 2)
            assert b[0, 0] == 0 and b[-1, 1] == T and (b[1:, 0] == b[:-1, 1]).all()
            o = np.ctypeslib.as_array((ctypes.c_float * (S * 2)).from_address(out)).reshape(S, 2)
            for s, (a, e) in enumerate(b):
                o[s] = (i[a:e].sum(), e - a)
            return 0

    monkeypatch.setattr(dmod, "lib", lambda: FakeLib())
    m = object.__new__(dmod._Model)
    m.h, m._n_out = None, 2
    seqs = [[5, 6, 7], np.array([1, 2], np.int32), [100] * 9, [3]]
    got = m.encoder_pass(seqs)
    assert got.shape == (4, 2) and got.dtype == np.float32
    assert got.tolist() == [[18, 3], [3, 2], [900, 9], [3, 1]]


class _FakeDecoder:
    """A decoder replica without a GPU: option score = the number of token forms in the option's group."""
    closed = []

    def __init__(self, base, device):
        self.device, self.kind = device, "d1-3b"

    def decoder_pass(self, trees):
        return [[[float(len(g)) for g in groups] for groups in tr["groups"]] for tr in trees]

    def close(self):
        pass


def test_system_one_api_with_fake_replicas(pkg, tmp_path, monkeypatch):
    """systemOne / systemOneBatch / probabilities / probabilitiesBatch (src/d1.ts:82-105) on two fake replicas:
    typed answers from the softmax of the option scores, usage = the request's packed tokens, request order kept
    across devices, progress reported per pass, malformed questions refused before any pass."""
    import math
    from decision_js_b200 import decision as dmod
    from decision_js_b200.questions import QuestionError
    (tmp_path / "manifest.json").write_text("{}")
    monkeypatch.setattr(dmod, "_Model", _FakeDecoder)
    d = dmod.Decision.load(str(tmp_path), devices=[0, 1], tokensPerPass=40)
    noul = {"type": "noul", "instructions": "", "branch": [1, 2], "groups": [[5, 6, 7], [8]]}
    choice = {"type": "choice", "instructions": "", "criteria": {"a": 1, "b": 2, "c": 3}, "branch": [3],
              "groups": [[1], [2, 3], [4]]}
    score = {"type": "score", "instructions": "", "criteria": ["lo", "hi"], "branch": [4, 4, 4],
             "groups": [[1, 2], [3, 4]]}
    r = d.systemOne([9] * 10, {"n": noul, "c": choice, "s": score})
    e3, e1 = math.exp(3), math.exp(1)
    assert math.isclose(r["answers"]["n"]["noul"], e3 / (e3 + e1))
    assert r["answers"]["c"]["choice"] == "b" and math.isclose(r["answers"]["c"]["confidence"],
                                                               math.exp(2) / (2 * e1 + math.exp(2)))
    assert math.isclose(r["answers"]["s"]["score"], 0.5) and r["answers"]["s"]["legend"] == {"0": "lo", "1": "hi"}
    assert r["usage"] == {"input_tokens": 10 + 2 + 1 + 3, "output_tokens": 0}
    # many requests over two replicas, in several passes, in order
    progress = []
    # request i: option i % 3 has three token forms, the others one, so it wins
    reqs = [[[7] * (5 + i), {"q": dict(choice, groups=[[1, 1, 1] if o == i % 3 else [2] for o in range(3)])}]
            for i in range(9)]
    out = d.systemOneBatch(reqs, {"onProgress": lambda done, total: progress.append((done, total))})
    assert [o["answers"]["q"]["choice"] for o in out] == ["abc"[i % 3] for i in range(9)]
    assert [o["usage"]["input_tokens"] for o in out] == [5 + i + 1 for i in range(9)]
    assert progress and progress[-1][1] == 9 and max(p[0] for p in progress) <= 9
    p = d.probabilities([1, 2], [noul, score])
    assert len(p) == 2 and math.isclose(sum(p[0]), 1.0) and p[1] == [0.5, 0.5]
    pb = d.probabilitiesBatch([[[1], [noul]], [[2, 3], [score, noul]]])
    assert [len(x) for x in pb] == [1, 2] and pb[1][0] == [0.5, 0.5]
    with pytest.raises(QuestionError):
        d.systemOne([1], {"bad": {"type": "choice", "instructions": "", "criteria": {"only": 1}, "branch": [1],
                                  "groups": [[1]]}})
    d.destroy()


def test_embed_keeps_embed_dim_then_normalises(pkg, tmp_path, monkeypatch):
    """Eg2Engine.embed (src/eg2-engine.ts:135-139): each pooled row (embedding_dim wide) is cut to its first
    embed_dim values, then L2-normalised; embed_raw returns the whole pooled row."""
    from decision_js_b200 import decision as dmod
    (tmp_path / "manifest.json").write_text("{}")
    monkeypatch.setattr(dmod, "_Model", _FakeModel)
    d = dmod.Decision.load(str(tmp_path), devices=[2])
    raw = d.embed_raw([[1, 2], [3]])
    emb = d.embed([[1, 2], [3]])
    assert [r.shape for r in raw] == [(4,), (4,)] and [e.shape for e in emb] == [(3,), (3,)]
    assert np.allclose(emb[0], 1 / np.sqrt(3)) and emb[0].dtype == np.float32
    d.destroy()


def test_oracle_short_conv_against_numpy(oracle):
    """SHORT_CONV (src/kernels.ts:65-84): y = f16(C · Σ_j w_j · B[tap_j] · U[tap_j]), a tap of -1 reads nothing."""
    rng = np.random.default_rng(12)
    T, H = 9, 64
    Z = rng.standard_normal((T, 3 * H)).astype(np.float16)
    Wc = (0.5 * rng.standard_normal((H, 3))).astype(np.float16)
    t = np.arange(T)
    taps = np.stack([t - 2, t - 1, t, 0 * t], 1)
    taps[taps < 0] = -1
    taps[4, :2] = [-1, 0]  # a branch-like token: its first tap gone, its second in another row
    got = oracle.short_conv(Z, Wc, taps.astype(np.int32))
    Zf, W = Z.astype(np.float64), Wc.astype(np.float64)
    B, C, U = Zf[:, :H], Zf[:, H:2 * H], Zf[:, 2 * H:]
    conv = np.zeros((T, H))
    for j in range(3):
        r = taps[:, j]
        ok = r >= 0
        conv[ok] += W[:, j] * B[r[ok]] * U[r[ok]]
    _f16_close(_h(got), C * conv, "short_conv", rtol=1e-3, afrac=1e-4)


def test_oracle_ple_mix_against_numpy(oracle):
    """PLE_MIX (src/eg2-kernels.ts:181-200): f16(gelu(gate) · e · rsqrt(mean(e²) + eps) · w)."""
    rng = np.random.default_rng(13)
    T, P, eps = 6, 512, 1e-6
    G = (2 * rng.standard_normal((T, P))).astype(np.float16)
    E = (3 * rng.standard_normal((T, P))).astype(np.float16)
    W = (1 + 0.1 * rng.standard_normal(P)).astype(np.float16)
    got = oracle.ple_mix(G, E, W, eps)
    g, e = G.astype(np.float64), E.astype(np.float64)
    gelu = 0.5 * g * (1 + np.tanh(np.sqrt(2 / np.pi) * (g + 0.044715 * g ** 3)))
    ref = gelu * e / np.sqrt((e ** 2).mean(1, keepdims=True) + eps) * W.astype(np.float64)
    _f16_close(_h(got), ref, "ple_mix", rtol=2e-3, afrac=0.0, atol=1e-5)


def test_oracle_readout_against_numpy(oracle):
    """READOUT (src/d3-kernels.ts:243-260): out[k] = X[row] · R[code] in f32."""
    rng = np.random.default_rng(14)
    X = rng.standard_normal((7, 256)).astype(np.float16)
    R = rng.standard_normal((5, 256)).astype(np.float32)
    pairs = np.array([[0, 4], [6, 0], [3, 3]], np.int32)
    ref = (X.astype(np.float64)[pairs[:, 0]] * R.astype(np.float64)[pairs[:, 1]]).sum(1)
    assert np.allclose(oracle.readout(X, R, pairs), ref, rtol=1e-5, atol=1e-4)


def _taps_from_ranges(rng):
    """The device's rule for the short convolution's taps (conv_taps_kernel), restated: a token's sequence is the
    part of [x, y) then of [z, w) at or before it; tap j is the token j places before it there, else -1."""
    T = len(rng)
    out = np.zeros((T, 4), np.int32)
    for t, (x, y, z, w) in enumerate(rng):
        seq = [k for k in range(x, min(y, t + 1))] + [k for k in range(z, min(w, t + 1))]
        out[t] = [seq[-3] if len(seq) >= 3 else -1, seq[-2] if len(seq) >= 2 else -1, t, 0]
    return out


def test_conv_taps_from_key_ranges_match_the_reference_taps(oracle, pkg):
    """The engine derives the conv taps from the forest's key ranges; on forests with short and one-token branches
    and one- and two-token trunks this gives exactly the taps D13BEngine.run builds (src/d1-3b-engine.ts:53-62),
    which the oracle restates from the trees; the package's own forest gives the same key ranges."""
    from decision_js_b200 import forest
    rs = np.random.default_rng(15)
    for trial in range(20):
        trees = []
        for _ in range(rs.integers(1, 5)):
            p = int(rs.integers(1, 9))
            nb = int(rs.integers(1, 4))
            trees.append({"trunk": list(rs.integers(0, 100, p)), "branches":
                          [list(rs.integers(0, 100, int(rs.integers(1, 5)))) for _ in range(nb)],
                          "groups": [[[1]]] * nb})
        ids, pos, rng, leaves, flat, taps = oracle.decoder_meta(trees, with_taps=True)
        assert np.array_equal(_taps_from_ranges(rng), taps), trial
        assert np.array_equal(forest(trees)[2], rng)


def test_reference_architecture_presets_write_valid_models(pkg, tmp_path):
    """The LFM2-hybrid decoder (conv layers, 64-wide heads) and the EmbeddingGemma 2 encoder (per-layer embeddings,
    512-wide full-layer heads, projection) presets write files the loader's checks accept, with the tensors the
    reference's exporters write (scripts/export-3b.py:36-52, scripts/export-eg2.py:103-125)."""
    from decision_js_b200 import synth
    from decision_js_b200._lib import lib
    d1, d2 = str(tmp_path / "lfm2"), str(tmp_path / "eg2")
    synth.write_decoder(d1, preset=synth.DECODER_LFM2, layers=3, vocab=512, hidden=256, intermediate=512, heads=4,
                        kv_heads=2)
    synth.write_encoder(d2, preset=synth.ENCODER_EG2, layers=6, vocab=512, hidden=256, intermediate=512, ple=128,
                        embedding_dim=384)
    assert lib().dc_check_weights(d1.encode()) == 0 and lib().dc_check_weights(d2.encode()) == 0
    m1 = json.load(open(os.path.join(d1, "manifest.json")))
    assert m1["config"]["layer_types"] == ["conv", "conv", "full_attention"]
    assert {"layers.0.in_proj", "layers.0.out_proj", "layers.0.conv", "layers.2.qkv"} <= set(m1["tensors"])
    assert m1["tensors"]["layers.0.conv"]["shape"] == [256, 3] and m1["config"]["head_dim"] == 64
    m2 = json.load(open(os.path.join(d2, "manifest.json")))
    assert {"ple.norm", "layers.5.ple_gate", "layers.5.ple_in", "layers.5.ple_proj", "layers.5.ple_norm",
            "projection"} <= set(m2["tensors"])
    assert m2["tensors"]["projection"]["shape"] == [384, 256]
    assert m2["config"]["head_dim"]["full_attention"] == 512


class _FakeEg2:
    """Stands in for an EmbeddingGemma 2 replica (no GPU): the embedding of a sequence is a one-hot on its length,
    and the head's logit of an option is its option index times 1 plus its question type index."""

    def __init__(self, base, device):
        self.device, self.kind, self.embed_dim = device, "eg2", None
        self.passes = []

    def encoder_pass(self, seqs):
        self.passes.append([len(s) for s in seqs])
        out = np.zeros((len(seqs), 64), np.float32)
        for i, s in enumerate(seqs):
            out[i, len(s) % 64] = 1.0
        return out

    def head_logits(self, S, Q, O, items):
        assert S.shape[1] == Q.shape[1] == O.shape[1] == 64
        out = np.zeros(int((items[:, 4] + items[:, 5]).max()), np.float32)
        for s, q, ty, o0, n, out0 in items:
            assert 0 <= s < len(S) and 0 <= q < len(Q) and o0 + n <= len(O)
            out[out0:out0 + n] = np.arange(n) * (1 + ty)
        return out

    def close(self):
        pass


def test_eg2_system_one_with_a_fake_replica(pkg, tmp_path, monkeypatch):
    """EmbeddingGemma 2's System One path (src/d1.ts:177-214) on a fake replica: texts rendered, tokenized, embedded
    once (a repeated schema costs no tokens the second time), the head's logits divided by the type's temperature
    and softmaxed, a noul read as [no, yes] and returned as [yes, no]; tokenized requests take the same path."""
    import math
    from decision_js_b200 import decision as dmod
    from decision_js_b200 import synth
    cfg = {"model": "eg2", "prompt": "task: classification | query: ", "max_len": 64,
           "question_types": ["choice", "score", "noul"], "temperatures": {"choice": 1.0, "score": 0.5, "noul": 2.0}}
    (tmp_path / "manifest.json").write_text(json.dumps({"config": cfg}))
    noul = {"type": "noul", "instructions": "Is it spam?"}
    choice = {"type": "choice", "instructions": "Topic?", "criteria": {"billing": "money", "bug": None, "x": "y"}}
    score = {"type": "score", "instructions": "Urgency?", "criteria": ["low", "mid", "high"]}
    from decision_js_b200 import prompts
    texts = [prompts.render_state({"a": 1}, "wf"), prompts.render_state("plain", "wf")]
    for q in (noul, choice, score):
        qt, opts = prompts.render_question(q)
        texts += [qt] + opts
    synth.write_tokenizer(str(tmp_path), texts + [cfg["prompt"]], 4096)
    monkeypatch.setattr(dmod, "_Model", _FakeEg2)
    d = dmod.Decision.load(str(tmp_path), devices=[0], workflow="wf")
    assert d.tokenizer is not None and d.workflow == "wf"
    r = d.systemOne({"a": 1}, {"n": noul, "c": choice, "s": score})
    # noul: logits [0, 3] (type 2) / 2.0 -> softmax [no, yes], returned [yes, no]
    pn = 1 / (1 + math.exp(-1.5))
    assert math.isclose(r["answers"]["n"]["noul"], pn, rel_tol=1e-6)
    assert r["answers"]["c"]["choice"] == "x"  # logits 0, 1, 2
    z = [0 / 0.5, 2 / 0.5, 4 / 0.5]  # score: type 1, logits 0, 2, 4, temperature 0.5
    e = [math.exp(v - max(z)) for v in z]
    assert math.isclose(r["answers"]["s"]["score"], sum(i * x for i, x in enumerate(e)) / sum(e), rel_tol=1e-6)
    first = r["usage"]["input_tokens"]
    assert first > 0
    # the same schema over a new state: only the state's text is embedded
    r2 = d.systemOne("plain", {"n": noul, "c": choice, "s": score})
    state_tokens = len(prompts.tokenize(d.tokenizer, prompts.render_state("plain", "wf"), cfg["prompt"], 64))
    assert r2["usage"]["input_tokens"] == state_tokens
    # tokenized requests: token-id state, question_ids and option_ids
    tq = {"type": "choice", "instructions": "", "criteria": {"a": 1, "b": 2}, "question_ids": [1, 2, 3],
          "option_ids": [[1, 4], [1, 5, 6]]}
    p = d.probabilities([7, 8, 9], [tq])
    assert math.isclose(p[0][1], math.exp(1) / (1 + math.exp(1)), rel_tol=1e-6)
    with pytest.raises(Exception):
        d.probabilities([7], [{"type": "noul", "instructions": "x"}] * 0 + [{"type": "bogus", "instructions": ""}])
    d.destroy()


def gdn_case(seed, H=2, trunk=5, branches=(7, 4), plain=(19,), scale=1.0):
    """In-projection rows and weights for the Gated DeltaNet mixer, with spans as D3Engine.logits builds them
    (src/d3-engine.ts:73-90): a shared trunk then its branches (the first branch writes the trunk), and plain
    sequences (whole, written)."""
    rng = np.random.default_rng(seed)
    QK = H * 128
    spans, t = [], 0
    tr0, t = t, t + trunk
    for b, L in enumerate(branches):
        spans.append([tr0, trunk | (0x80000000 if b == 0 else 0), t, L])
        t += L
    for L in plain:
        spans.append([t, L | 0x80000000, 0, 0])
        t += L
    T, qkv = t, 3 * QK
    stride = 4 * QK + 2 * H + 8  # a padded row
    Z = (scale * rng.standard_normal((T, stride))).astype(np.float16)
    W = (0.5 * rng.standard_normal((3 * QK, 4))).astype(np.float16)
    Alog = rng.uniform(-1.5, 0.5, H).astype(np.float16)
    dtb = rng.uniform(-1, 1, H).astype(np.float16)
    gw = (1 + 0.1 * rng.standard_normal(128)).astype(np.float16)
    return dict(Z=Z, stride=stride, qkv=qkv, H=H, W=W, Alog=Alog, dtb=dtb, gw=gw,
                spans=np.array(spans, np.uint32), eps=1e-6, T=T)


def gdn_numpy(c):
    """The mixer in float64 in the reference's other form (src/d3-kernels.ts:24-26, MLX's: S = decay S,
    delta = beta (v - S k), S += delta k^T, o = S q), with the same f16 roundings of the conv outputs."""
    Z, H, stride, qkv = c["Z"].astype(np.float64), c["H"], c["stride"], c["qkv"]
    QK = H * 128
    W = c["W"].astype(np.float64)
    Y = np.zeros((c["T"], QK))
    written = np.zeros(c["T"], bool)
    silu = lambda x: x / (1 + np.exp(-x))  # noqa: E731
    for a0, af, b0, bl in c["spans"].tolist():
        alen, wa = af & 0x7fffffff, af >> 31
        toks = list(range(a0, a0 + alen)) + list(range(b0, b0 + bl))
        for h in range(H):
            S = np.zeros((128, 128))
            for v, t in enumerate(toks):
                chans = [np.arange(128) + part * QK + h * 128 for part in range(3)]
                qkvv = []
                for ch in chans:
                    x = np.stack([Z[toks[v - back], ch] if v >= back else np.zeros(128) for back in (3, 2, 1, 0)], 1)
                    y = (W[ch] * x).sum(1)
                    qkvv.append(silu(y).astype(np.float16).astype(np.float64))
                q, k, vv = qkvv
                k = k / np.sqrt((k * k).sum() + 1e-6)
                q = q / np.sqrt((q * q).sum() + 1e-6) / np.sqrt(128)
                zr = qkv + QK
                b, a = Z[t, zr + h], Z[t, zr + H + h] + float(c["dtb"][h])
                sp = a if a > 20 else np.log1p(np.exp(a))
                dec, beta = np.exp(-np.exp(float(c["Alog"][h])) * sp), 1 / (1 + np.exp(-b))
                S = dec * S
                delta = beta * (vv - S @ k)
                S = S + np.outer(delta, k)
                o = S @ q
                if v < alen and not wa:
                    continue
                z = Z[t, qkv + h * 128: qkv + h * 128 + 128]
                Y[t, h * 128:(h + 1) * 128] = o / np.sqrt((o * o).mean() + c["eps"]) * c["gw"].astype(np.float64) * silu(z)
                written[t] = True
    return Y, written


def test_oracle_gdn_against_numpy(oracle):
    """The Gated DeltaNet mixer (src/d3-kernels.ts:23-149): the oracle's ORT form against the MLX form in float64,
    over a shared trunk with two branches (only the first writes the trunk) and a plain sequence."""
    c = gdn_case(16)
    got = oracle.gdn(c["Z"], c["stride"], c["qkv"], c["H"], c["W"], c["Alog"], c["dtb"], c["gw"], c["spans"],
                     c["eps"], c["T"])
    ref, written = gdn_numpy(c)
    assert written.all()
    _f16_close(_h(got), ref, "gdn", rtol=3e-3, afrac=1e-3)


def test_oracle_omni_head_kernels_against_numpy(oracle):
    """The d1-omni / Laya head kernels (src/kernels.ts:187-283) and GELU_MUL with erf (src/encoder-kernels.ts:26-44)
    against float64 numpy: ADD_ROWS, BIAS_ACT (none, ReLU, GELU erf), ADD_LAYERNORM (with and without the residual
    add and the bias), GATHER_ROWS, SCORE."""
    from math import erf
    rng = np.random.default_rng(21)
    T, H, nE = 9, 256, 3
    Xi = rng.standard_normal((T, H)).astype(np.float16)
    E = rng.standard_normal((nE, H)).astype(np.float16)
    idx = rng.integers(0, nE, T).astype(np.int32)
    _f16_close(_h(oracle.add_rows(Xi, idx, E)), Xi.astype(np.float64) + E.astype(np.float64)[idx], "add_rows",
               rtol=1e-3, afrac=0.0, atol=1e-6)
    Y = (2 * rng.standard_normal((T, H))).astype(np.float16)
    b = rng.standard_normal(H).astype(np.float16)
    v = Y.astype(np.float64) + b.astype(np.float64)
    gelu = 0.5 * v * (1 + np.vectorize(erf)(v / np.sqrt(2)))
    for act, ref in ((0, v), (1, np.maximum(v, 0)), (2, gelu)):
        _f16_close(_h(oracle.bias_act(Y, b, act)), ref, f"bias_act {act}", rtol=1e-3, afrac=0.0, atol=1e-5)
    A = (2 * rng.standard_normal((T, 2 * H))).astype(np.float16)
    a, u = A[:, :H].astype(np.float64), A[:, H:].astype(np.float64)
    ref = 0.5 * a * (1 + np.vectorize(erf)(a / np.sqrt(2))) * u
    _f16_close(_h(oracle.glu(A, H, 2)), ref, "gelu_mul erf", rtol=2e-3, afrac=0.0, atol=1e-5)
    W = (1 + 0.1 * rng.standard_normal(H)).astype(np.float16)
    B = (0.1 * rng.standard_normal(H)).astype(np.float16)
    for add, bias in ((False, True), (True, True), (True, False)):
        Xn, O = oracle.add_layernorm(Xi, Y if add else None, W, B if bias else None, add, 1e-5)
        x = Xi.astype(np.float64) + (Y.astype(np.float64) if add else 0)
        if add:
            assert np.array_equal(Xn, x.astype(np.float16).view(np.uint16))
        ref = (_h(Xn) - x.mean(1, keepdims=True)) / np.sqrt(x.var(1, keepdims=True) + 1e-5) * W.astype(np.float64)
        ref = ref + (B.astype(np.float64) if bias else 0)
        _f16_close(_h(O), ref, f"add_layernorm add={add} bias={bias}", rtol=2e-3, afrac=1e-3)
    rows = np.array([3, 0, 8, 3], np.int32)
    assert np.array_equal(oracle.gather_rows(Xi, rows), Xi.view(np.uint16)[rows])
    wv = rng.standard_normal(H).astype(np.float16)
    bb = np.array([0.25], np.float16)
    ref = (Y.astype(np.float64) * wv.astype(np.float64)).sum(1) + 0.25
    assert np.allclose(oracle.score(Y, wv, bb), ref, rtol=1e-5, atol=1e-3)


@pytest.mark.parametrize("D,rot,norm,heads,kv,pad", [(256, 64, True, 4, 2, 2 * 256 + 16), (64, 64, False, 3, 3, 3 * 64)])
def test_oracle_qk_rope_against_numpy(oracle, D, rot, norm, heads, kv, pad):
    """d3-lite's QK_NORM_ROPE_256 (src/d3-kernels.ts:150-172: RMSNorm over 256, RoPE on the first 64 dims) and
    Laya's ROPE (src/encoder-kernels.ts:5-24: no norm, 64-dim heads) in rows with v (and gate) heads after q, k."""
    rng = np.random.default_rng(22 + D)
    T, theta, eps = 7, 10000.0, 1e-6
    stride = (heads + kv) * D + pad
    Z = rng.standard_normal((T, stride)).astype(np.float16)
    qn = (1 + 0.1 * rng.standard_normal(D)).astype(np.float16)
    kn = (1 + 0.1 * rng.standard_normal(D)).astype(np.float16)
    pos = rng.integers(0, 900, T).astype(np.int32)
    got = oracle.qk_rope(Z, qn if norm else None, kn if norm else None, pos, heads, kv, D, rot, norm, eps, theta)
    ref = Z.astype(np.float64).copy()
    for h in range(heads + kv):
        x = ref[:, h * D:(h + 1) * D]
        if norm:
            x = x / np.sqrt((x * x).mean(1, keepdims=True) + eps) * (qn if h < heads else kn).astype(np.float64)
        d = np.arange(rot // 2)
        ang = pos[:, None].astype(np.float64) * theta ** (-2.0 * d / rot)
        a, b = x[:, :rot // 2].copy(), x[:, rot // 2:rot].copy()
        x[:, :rot // 2] = a * np.cos(ang) - b * np.sin(ang)
        x[:, rot // 2:rot] = b * np.cos(ang) + a * np.sin(ang)
        ref[:, h * D:(h + 1) * D] = x
    _f16_close(_h(got), ref, "qk_rope", rtol=2e-3, afrac=2e-3)
    assert np.array_equal(got[:, (heads + kv) * D:], Z.view(np.uint16)[:, (heads + kv) * D:])  # v / gate untouched


def test_oracle_gated_strided_attention(oracle):
    """The oracle's strided / gated attention (src/d3-kernels.ts:174-240): with the rows' own stride and no gate it
    is the plain attention; with the gate, each output is the plain one over 1 + exp(-gate)."""
    rng = np.random.default_rng(23)
    T, heads, kv, D = 11, 4, 2, 64
    r = np.array([(0, 6, 0, 0)] * 6 + [(6, 11, 0, 0)] * 5, np.int32)
    Z = rng.standard_normal((T, (2 * heads + 2 * kv) * D)).astype(np.float16)
    plain = oracle.attention(np.ascontiguousarray(Z[:, :(heads + 2 * kv) * D]), r, heads, kv, D, 0.125)
    assert np.array_equal(oracle.attention_ex(Z, r, heads, kv, D, 0.125, False), plain)
    g = Z[:, (heads + 2 * kv) * D:].astype(np.float64)
    ref = plain.view(np.float16).astype(np.float64) / (1 + np.exp(-g))
    _f16_close(_h(oracle.attention_ex(Z, r, heads, kv, D, 0.125, True)), ref, "gated attention", rtol=2e-3,
               afrac=0.0, atol=1e-4)


def test_d3_pack_matches_the_oracle_restatement(oracle, pkg):
    """The package's d3 packer and the oracle's restatement of D3Engine.logits' metadata (src/d3-engine.ts:71-92)
    agree on random groups: shared trunks (the common prefix, at least one token left per sequence), one-sequence
    groups, identical sequences, and sequences of one token."""
    from decision_js_b200.decision import d3_pack
    rs = np.random.default_rng(24)
    for trial in range(30):
        seqs, groups = [], []
        for _ in range(rs.integers(1, 5)):
            n = int(rs.integers(1, 4))
            common = list(rs.integers(0, 50, int(rs.integers(0, 6))))
            for _ in range(n):
                tail = list(rs.integers(0, 50, int(rs.integers(0 if common else 1, 5))))
                seqs.append((common + tail if common + tail else [7], int(rs.integers(1, 6))))
            groups.append(n)
        for g in (groups, None):
            got, ref = d3_pack(seqs, g), oracle.d3_meta(seqs, g)
            for a, b in zip(got, ref):
                assert np.array_equal(a, b), (trial, g)


def test_d3_prompt_text():
    """d3-lite's prompt (src/d3-prompt.ts): the chat template, the options in readout order with their codes, the
    reference's errors."""
    from decision_js_b200 import prompts
    codes = ["A", "B", "C"]
    q = {"type": "choice", "instructions": "Pick", "criteria": {"x": "first", "y": None}}
    t = prompts.d3_text({"k": [1, 2]}, q, codes)
    assert t.startswith("<|im_start|>system\nYou are a decision engine.")
    assert "<|im_start|>user\nState:\n{\"k\": [1, 2]}\n\nQuestion:\nPick\n\nOptions:\nA: x: first\nB: y\n\n" in t
    assert t.endswith("Reply with only the code of the best option.<|im_end|>\n<|im_start|>assistant\n<think>\n\n"
                      "</think>\n\n")
    assert prompts.d3_options({"type": "noul", "instructions": "?"}) == ["No / false", "Yes / true"]
    assert "State:\n(empty)" in prompts.d3_user_prompt(None, {"type": "noul", "instructions": "?"}, codes)
    with pytest.raises(ValueError, match="distinct"):
        prompts.d3_options({"type": "score", "criteria": ["a", "a"]})
    with pytest.raises(ValueError, match='"false" and "true"'):
        prompts.d3_options({"type": "noul", "criteria": {"yes": "y"}})


def test_omni_pack_matches_the_oracle_restatement(oracle, pkg):
    """The package's d1-omni packer against the oracle's restatement of D1OmniEngine.logits' metadata loop
    (src/omni-engine.ts:58-69): bidirectional ranges per sequence, centred conv taps that never cross a sequence,
    question types per token, absolute markers; one-token sequences included."""
    from decision_js_b200.decision import omni_pack
    rs = np.random.default_rng(25)
    for trial in range(20):
        seqs = []
        for _ in range(rs.integers(1, 6)):
            n = int(rs.integers(1, 30))
            seqs.append((list(rs.integers(0, 100, n)), sorted(rs.integers(0, n, int(rs.integers(1, 4))).tolist()),
                         int(rs.integers(0, 3))))
        for a, b in zip(omni_pack(seqs), oracle.omni_meta(seqs)):
            assert np.array_equal(a, b), trial


def test_omni_prompt(tmp_path, pkg):
    """d1-omni's prompt (src/omni-prompt.ts): <bos> <state> state <q> instructions, per option <opt> <mask> text
    </opt>, <decide>; each marker points at an option's <mask>; caller text cannot forge a delimiter; the option
    texts in the model's order (a noul as [false, true])."""
    from decision_js_b200 import prompts, synth
    d = str(tmp_path)
    extra = ("<|im_start|>", "<|im_end|>", *prompts.OMNI_DELIM.values(), prompts.OMNI_MARKER)
    synth.write_tokenizer(d, ["level false true no yes the statement does not hold Pick a b c x y <¦reserved_8¦>"],
                          4096, extra=extra)
    tok = prompts.TextTokenizer.load(d)
    q = {"type": "choice", "instructions": "Pick <|reserved_8|>", "criteria": {"a": "x", "b": None, "c": ""}}
    ids, markers = prompts.omni_encode(tok, {"s": 1}, q)
    assert ids[0] == tok.id(tok.bos) and ids[1] == tok.id("<|reserved_7|>") and ids[-1] == tok.id("<|reserved_11|>")
    assert [ids[m] for m in markers] == [tok.id("<|mask|>")] * 3
    assert [ids[m - 1] for m in markers] == [tok.id("<|reserved_9|>")] * 3
    assert ids.count(tok.id("<|reserved_8|>")) == 1  # the escaped copy in the instructions is not the delimiter
    assert prompts.omni_options(q) == ["a: x", "b", "c"]
    assert prompts.omni_options({"type": "noul", "instructions": "?"}) == ["false: no, the statement does not hold",
                                                                          "true: yes, the statement holds"]
    assert prompts.omni_options({"type": "score", "criteria": ["lo", "hi"]}) == ["level 0: lo", "level 1: hi"]
    assert prompts.omni_temperature_key({"type": "choice", "criteria": {"a": 1, "b": 2, "c": 3}}) == "choice:3-5"
    short, mk = prompts.omni_encode(tok, "word " * 500, q, max_len=150)
    assert len(short) <= 150 and mk[-1] < 150


def test_laya_pack_matches_the_oracle_restatement(oracle, pkg):
    """The package's Laya packer against the oracle's restatement (src/laya-engine.ts:52-63): the whole-sequence
    ranges and the +-window ranges clipped to each sequence."""
    from decision_js_b200.decision import laya_pack
    rs = np.random.default_rng(26)
    for trial in range(10):
        seqs = [(list(rs.integers(0, 100, n)), [0, n - 1], int(rs.integers(0, 3)))
                for n in rs.integers(1, 200, int(rs.integers(1, 5)))]
        for a, b in zip(laya_pack(seqs, 64), oracle.laya_meta(seqs, 64)):
            assert np.array_equal(a, b), trial


def test_laya_prompt(tmp_path, pkg):
    """Laya's prompt (src/laya-prompt.ts): [CLS] type question: instructions [SEP] [MASK] option ... [SEP] state
    [SEP]; markers at the [MASK]s; a [MASK] in caller text is blanked; a list state loses its oldest tokens."""
    import json as _json
    from decision_js_b200 import prompts, synth
    d = str(tmp_path)
    synth.write_tokenizer(d, ["choice question Pick a b level false true no yes the statement does not hold w0 w1 w2"],
                          4096, extra=("[CLS]", "[SEP]", "[MASK]"))
    cfgp = os.path.join(d, "tokenizer_config.json")
    cfg = _json.load(open(cfgp))
    cfg.update(cls_token="[CLS]", sep_token="[SEP]", mask_token="[MASK]")
    _json.dump(cfg, open(cfgp, "w"))
    tok = prompts.TextTokenizer.load(d)
    q = {"type": "choice", "instructions": "Pick [MASK]", "criteria": {"a": None, "b": "x"}}
    ids, markers = prompts.laya_encode(tok, "w0 w1", q)
    cls, sep, mask = tok.id("[CLS]"), tok.id("[SEP]"), tok.id("[MASK]")
    assert ids[0] == cls and ids[-1] == sep and [ids[m] for m in markers] == [mask, mask]
    assert ids.count(mask) == 2 and ids.count(sep) == 3
    conv = ["w0"] * 300 + ["w2"]
    long_ids, mk = prompts.laya_encode(tok, conv, q, max_len=64)
    assert len(long_ids) == 64 and tok.id("w2") in long_ids[-4:]  # the newest turn kept, the oldest cut
    with pytest.raises(ValueError, match="needs a state"):
        prompts.laya_encode(tok, None, q)
    with pytest.raises(ValueError, match="keyed only"):
        prompts.laya_options({"type": "noul", "criteria": {"yes": "y"}})
