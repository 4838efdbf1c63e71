"""Parity at BASELINE's full sizes. The kernels run on whole full-size batches; the oracle, which cannot finish those
in seconds, checks sampled parts that are independent of the rest: output rows of a matmul (each row depends only
on its own token row), and whole requests of a forward pass (requests never read each other's tokens). So every
tile, wave and persistent-CTA schedule of the full launch is exercised, and what is checked is checked exactly as
in the small-size tests (same tolerances).
"""
import numpy as np
import pytest

from conftest import f16_of, rel_err, to_dev

pytestmark = pytest.mark.gpu

T_FULL = 16384  # tokens per pass in configs 2, 3 and 4

# every linear layer shape of configs 2-4 at M = 16384: (N, K, bits, gated activation or None)
SHAPES = [
    (1280, 768, 8, None), (768, 768, 8, None), (2304, 768, 8, 1), (768, 1152, 8, None),      # config 2
    (4096, 1024, 8, None), (1024, 2048, 8, None), (6144, 1024, 8, 2), (1024, 3072, 8, None),  # config 3
    (5120, 3072, 4, None), (3072, 3072, 4, None), (16384, 3072, 4, 2), (3072, 8192, 4, None),  # config 4
]


def _sample_rows(M, seed):
    """Tile edges of the 256-token tiles, the first and last rows, the ragged last tile, and random rows."""
    rng = np.random.default_rng(seed)
    edges = [0, 1, 127, 128, 255, 256, 8191, 8192, M - 129, M - 128, M - 2, M - 1]
    r = np.unique(np.concatenate([edges, rng.integers(0, M, 20)])).astype(np.int64)
    return r[(r >= 0) & (r < M)]


def _interleave_rows(a, I):
    perm = np.stack([np.arange(I), I + np.arange(I)], axis=1).reshape(-1)
    return np.ascontiguousarray(a.reshape(2 * I, -1)[perm])


@pytest.mark.parametrize("N,K,bits,act", SHAPES)
def test_qmatmul_full_size_sampled_rows(ctx, dev, oracle, N, K, bits, act):
    import torch
    from decision_js_b200 import synth
    X, codes, S = synth.config1_inputs(seed=N + K, M=T_FULL, N=N, K=K, bits=bits)
    rows = _sample_rows(T_FULL, N ^ K)
    if act is None:
        Y = torch.full((T_FULL, N), -1, dtype=torch.int16, device=dev)
        ctx.call("qmatmul", to_dev(X, dev), to_dev(codes, dev), to_dev(S, dev), Y, T_FULL, N, K, bits, 0)
        ctx.sync(60000)
        got = f16_of(Y[torch.from_numpy(rows).to(dev)])
        ref = oracle.qmatmul(X[rows], codes, S, N, K, bits).view(np.float16).astype(np.float32)
        tol = 4e-3 * np.abs(ref) + 1e-3 * np.abs(ref).max()
        assert (np.abs(got - ref) <= tol).all(), rel_err(got, ref)
    else:
        I = N // 2
        Y = torch.full((T_FULL, I), -1, dtype=torch.int16, device=dev)
        ctx.call("qmatmul", to_dev(X, dev), to_dev(_interleave_rows(codes, I), dev),
                 to_dev(_interleave_rows(S, I), dev), Y, T_FULL, N, K, bits, act)
        ctx.sync(60000)
        got = f16_of(Y[torch.from_numpy(rows).to(dev)])
        ref = oracle.glu(oracle.qmatmul(X[rows], codes, S, N, K, bits), I, 1 if act == 1 else 0)
        ref = ref.view(np.float16).astype(np.float32)
        tol = 4e-3 * np.abs(ref) + 1e-3 * np.abs(ref).max()
        assert (np.abs(got - ref) <= tol).all(), rel_err(got, ref)


@pytest.mark.parametrize("N,K,bits,act", SHAPES)
def test_direct_full_size_sampled_rows(ctx, dev, oracle, N, K, bits, act):
    """The direct form (dc_dequant once, then dc_qmatmul_f16) on every config 2-4 linear at 16,384 tokens, as the
    model passes run it: plain and gated, against the oracle on the codes."""
    import torch
    from decision_js_b200 import synth
    X, codes, S = synth.config1_inputs(seed=N + K + 1, M=T_FULL, N=N, K=K, bits=bits)
    rows = _sample_rows(T_FULL, N ^ K ^ 5)
    I = N // 2
    c, sc = (codes, S) if act is None else (_interleave_rows(codes, I), _interleave_rows(S, I))
    W16 = torch.empty((N, K), dtype=torch.int16, device=dev)
    ctx.call("dequant", to_dev(c, dev), to_dev(sc, dev), W16, N, K, bits)
    Y = torch.full((T_FULL, N if act is None else I), -1, dtype=torch.int16, device=dev)
    ctx.call("qmatmul_f16", to_dev(X, dev), W16, Y, T_FULL, N, K, 0 if act is None else act)
    ctx.sync(60000)
    got = f16_of(Y[torch.from_numpy(rows).to(dev)])
    ref = oracle.qmatmul(X[rows], codes, S, N, K, bits)
    if act is not None:
        ref = oracle.glu(ref, I, 1 if act == 1 else 0)
    ref = ref.view(np.float16).astype(np.float32)
    tol = 4e-3 * np.abs(ref) + 1e-3 * np.abs(ref).max()
    assert (np.abs(got - ref) <= tol).all(), rel_err(got, ref)


@pytest.mark.parametrize("N,K,bits,M", [(1280, 768, 8, T_FULL - 77), (4096, 1024, 8, T_FULL), (768, 1152, 4, 5000),
                                         (3072, 3072, 4, T_FULL - 200), (384, 8192, 8, 777)])
def test_qmatmul_pair_form_forced(ctx, dev, oracle, N, K, bits, M):
    """The CTA-pair prefill form (form 7) on shapes the router gives the single-CTA form, ragged token counts
    included (a pair whose second CTA has no tokens, a last tile of 3 rows)."""
    import torch
    from decision_js_b200 import synth
    X, codes, S = synth.config1_inputs(seed=M + N, M=M, N=N, K=K, bits=bits)
    rows = _sample_rows(M, N + M)
    Y = torch.full((M, N), -1, dtype=torch.int16, device=dev)
    ctx.call("qmatmul_form", to_dev(X, dev), to_dev(codes, dev), to_dev(S, dev), Y, M, N, K, bits, 7, 0)
    ctx.sync(60000)
    got = f16_of(Y[torch.from_numpy(rows).to(dev)])
    ref = oracle.qmatmul(X[rows], codes, S, N, K, bits).view(np.float16).astype(np.float32)
    tol = 4e-3 * np.abs(ref) + 1e-3 * np.abs(ref).max()
    assert (np.abs(got - ref) <= tol).all(), rel_err(got, ref)


@pytest.mark.parametrize("act", [1, 2])
def test_gated_pair_form_q8(ctx, dev, oracle, act):
    """A q8 gated layer long enough in K for the router to give it the CTA-pair form (K >= 3072, N x K >= 8M)."""
    test_qmatmul_full_size_sampled_rows(ctx, dev, oracle, 4096, 3072, 8, act)


def test_encoder_config2_full_batch(pkg, oracle):
    """BASELINE config 2 as benchmarked: the 24-layer EmbeddingGemma-300M-architecture encoder, 64 texts x 256
    tokens in one pass; the first and last texts against the oracle."""
    from decision_js_b200 import synth
    d = synth.cached_model("encoder", device="cuda:0")
    m = pkg.Decision.load(d, devices=[0], tokensPerPass=T_FULL)
    seqs = synth.encoder_requests(64, 256, 262144, seed=21)
    got = np.stack(m.embed_raw(seqs))
    m.destroy()
    w = oracle.Weights(d)
    for i in (0, 63):
        ref = oracle.encoder_embed(w, np.asarray(seqs[i], np.int32), [256])[0]
        assert np.abs(got[i] - ref).max() <= 2e-2 * np.abs(ref).max(), (i, rel_err(got[i], ref))


def _option_scores(tree, ref):
    """Per question, each option's best logit over its group (src/d1-3b-engine.ts:111-121)."""
    out = []
    for q, groups in enumerate(tree["groups"]):
        j, rs = 0, []
        for g in groups:
            rs.append(ref[q, j:j + len(g)].max())
            j += len(g)
        out.append(np.array(rs))
    return out


def _decoder_full_batch(pkg, oracle, d, n, tokens, vocab, check, order_floor=False):
    """The full batch on the GPU; trees `check` through the oracle. With order_floor, the oracle also runs with its
    matmuls summed in the other k order, and the probability tolerance is the larger of 1e-3 and twice the spread
    between the oracle's two orders: over a deep f16 stack, rounding order alone moves the answer probabilities,
    and no implementation that sums in another order (every GPU kernel does) can agree more closely than that."""
    from decision_js_b200 import forest, synth
    m = pkg.Decision.load(d, devices=[0], tokensPerPass=n * tokens)
    trees = synth.decoder_trees(n, tokens, vocab, seed=22)
    scores = m.run(trees)
    m.destroy()
    w = oracle.Weights(d)
    for i in check:
        ids, pos, rng, leaves, leaf_ids = forest([trees[i]])
        ref = _option_scores(trees[i], oracle.decoder_logits(w, ids, pos, rng, leaves, np.array(leaf_ids, np.int32)))
        tol_p = 1e-3
        if order_floor:
            oracle.MATMUL_ORDER = 1
            try:
                alt = _option_scores(trees[i], oracle.decoder_logits(w, ids, pos, rng, leaves,
                                                                     np.array(leaf_ids, np.int32)))
            finally:
                oracle.MATMUL_ORDER = 0
            spread = max(np.abs(oracle.softmax(a) - oracle.softmax(b)).max() for a, b in zip(ref, alt))
            tol_p = max(1e-3, 2 * spread)
        for q, s in enumerate(scores[i]):
            rs = ref[q]
            assert np.abs(np.array(s) - rs).max() <= 2e-2 * np.abs(rs).max(), (i, q, s, rs)
            p, rp = np.array(pkg.softmax(s)), oracle.softmax(rs)
            assert np.abs(p - rp).max() < tol_p, (np.abs(p - rp).max(), tol_p)
            assert np.argmax(p) == np.argmax(rp) or np.sort(rp)[-1] - np.sort(rp)[-2] < tol_p


def test_decoder_config3_full_batch(pkg, oracle):
    """BASELINE config 3 as benchmarked: the 28-layer 0.6B q8 decoder, 32 trees x 512 tokens in one pass; the last
    tree's three readouts against the oracle."""
    from decision_js_b200 import synth
    d = synth.cached_model("decoder", device="cuda:0")
    _decoder_full_batch(pkg, oracle, d, 32, 512, 151936, check=(31,))


def test_decoder_config4_full_width(pkg, oracle):
    """BASELINE config 4's width and batch (3B q4: d 3072, 24/8 heads of 128, SwiGLU 8192, 16 trees x 1024 tokens
    in one pass) through 2 of its 32 layers, so that the oracle finishes; the first tree against it."""
    from decision_js_b200 import synth
    d = synth.cached_model("decoder", device="cuda:0", hidden=3072, intermediate=8192, heads=24, kv_heads=8,
                           vocab=65536, eps=1e-5, layers=2, bits=4)
    _decoder_full_batch(pkg, oracle, d, 16, 1024, 65536, check=(0,))


def test_decoder_config4_full_depth(pkg, oracle):
    """BASELINE config 4 as benchmarked, at its full depth: the 32-layer 3B q4 decoder, 16 trees x 1024 tokens in
    one pass; the last tree through all 32 layers against the oracle (the f16 range of the whole q4 stack). Logits
    within 2e-2; probabilities within 1e-3 or twice the oracle's own spread between two summation orders."""
    from decision_js_b200 import synth
    d = synth.cached_model("decoder", device="cuda:0", hidden=3072, intermediate=8192, heads=24, kv_heads=8,
                           vocab=65536, eps=1e-5, layers=32, bits=4)
    _decoder_full_batch(pkg, oracle, d, 16, 1024, 65536, check=(15,), order_floor=True)
