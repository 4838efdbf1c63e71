"""Kernel parity on the GPU: every C-ABI kernel against the CPU oracle on the same seeded inputs.

Tolerances: dequantisation is bit-exact. The matmul accumulates the same exact f16 x f16 products in f32 (in a
different order) and rounds once to f16, so results agree to about one f16 ulp: |gpu - oracle| <= 4e-3 |oracle|
+ 1e-3 max|oracle|; the gated epilogues (GeGLU / SwiGLU fused into the GEMM) meet the same bound (measured: at most
3.7e-3 |oracle| + 3.7e-6 max|oracle| over the cases below). Attention (f16 probabilities into P.V) agrees within
ATTN_TOL = 1.5e-3 of the output's max magnitude (measured at most 6.0e-4 over these masks, head dims and both
kernels); RoPE within 1e-2 of max; f32 reductions (pool, readout logits) within 1e-4 relative.
"""
import numpy as np
import pytest

from conftest import f16_of, rel_err, to_dev

pytestmark = pytest.mark.gpu

ATTN_TOL = 1.5e-3


def _mm_case(M, N, K, bits, seed):
    from decision_js_b200 import synth
    return synth.config1_inputs(seed=seed, M=M, N=N, K=K, bits=bits)


def _close_mm(got, ref):
    tol = 4e-3 * np.abs(ref) + 1e-3 * np.abs(ref).max()
    bad = ~(np.abs(got - ref) <= tol)  # NaN fails too
    assert not bad.any(), f"{bad.sum()} of {bad.size} outside tolerance; max rel {rel_err(got, ref):.3e}"


@pytest.mark.parametrize("bits", [8, 4])
@pytest.mark.parametrize("N,K", [(256, 128), (1152, 768), (384, 96)])
def test_dequant_bit_exact(ctx, dev, oracle, bits, N, K):
    import torch
    _, codes, S = _mm_case(1, N, K, bits, 3)
    out = torch.empty((N, K), dtype=torch.int16, device=dev)
    ctx.call("dequant", to_dev(codes, dev), to_dev(S, dev), out, N, K, bits)
    ctx.sync(60000)
    assert np.array_equal(out.cpu().numpy().view(np.uint16), oracle.dequant(codes, S, N, K, bits))


@pytest.mark.parametrize("form", [0, 2, 3, 6, 7])
@pytest.mark.parametrize("bits", [8, 4])
@pytest.mark.parametrize("M,N,K", [(256, 1152, 768), (128, 256, 64), (200, 384, 96), (333, 768, 1152),
                                   (1024, 2304, 768), (129, 136, 160)])
def test_qmatmul_prefill(ctx, dev, oracle, form, bits, M, N, K):
    import torch
    X, codes, S = _mm_case(M, N, K, bits, M + N)
    Y = torch.full((M, N), -1, dtype=torch.int16, device=dev)
    ctx.call("qmatmul_form", to_dev(X, dev), to_dev(codes, dev), to_dev(S, dev), Y, M, N, K, bits, form, 1)
    ctx.sync(60000)
    _close_mm(f16_of(Y), oracle.qmatmul(X, codes, S, N, K, bits).view(np.float16).astype(np.float32))


@pytest.mark.parametrize("bits", [8, 4])
@pytest.mark.parametrize("M,N,K", [(4096, 2304, 768), (8192, 1280, 768), (3000, 768, 1152), (2048, 4096, 1024)])
@pytest.mark.parametrize("form", [2, 3, 6, 7])
def test_qmatmul_persistent_many_tiles(ctx, dev, oracle, form, bits, M, N, K):
    """Several tiles per CTA: both TMEM accumulators and the stage rings' phases wrap across tiles."""
    import torch
    X, codes, S = _mm_case(M, N, K, bits, M ^ N)
    Y = torch.full((M, N), -1, dtype=torch.int16, device=dev)
    ctx.call("qmatmul_form", to_dev(X, dev), to_dev(codes, dev), to_dev(S, dev), Y, M, N, K, bits, form, 1)
    ctx.sync(60000)
    _close_mm(f16_of(Y), oracle.qmatmul(X, codes, S, N, K, bits).view(np.float16).astype(np.float32))


@pytest.mark.parametrize("form", [1, 4])
@pytest.mark.parametrize("bits", [8, 4])
@pytest.mark.parametrize("M,N,K,splits", [(1, 768, 768, 0), (3, 1152, 768, 1), (16, 256, 256, 2), (17, 384, 96, 0),
                                          (64, 3072, 1024, 0), (100, 200, 320, 3), (128, 1024, 512, 0),
                                          (1, 8192, 3072, 0), (33, 640, 4096, 5)])
def test_qmatmul_skinny(ctx, dev, oracle, form, bits, M, N, K, splits):
    import torch
    X, codes, S = _mm_case(M, N, K, bits, 7 * M + N)
    Y = torch.full((M, N), -1, dtype=torch.int16, device=dev)
    ctx.call("qmatmul_form", to_dev(X, dev), to_dev(codes, dev), to_dev(S, dev), Y, M, N, K, bits, form, splits)
    ctx.sync(60000)
    _close_mm(f16_of(Y), oracle.qmatmul(X, codes, S, N, K, bits).view(np.float16).astype(np.float32))


@pytest.mark.parametrize("bits", [8, 4])
@pytest.mark.parametrize("M,N,K,parts", [(1, 768, 768, 0), (1, 8192, 3072, 0), (2, 1152, 768, 1), (5, 200, 320, 0),
                                         (8, 1000, 96, 0), (9, 3072, 1024, 3), (16, 384, 4096, 8), (16, 2304, 768, 0),
                                         (3, 130, 8192, 0), (12, 640, 1152, 2), (7, 520, 2816, 0), (1, 48, 512, 4),
                                         (16, 8200, 3072, 0), (10, 8192, 3072, 0)])
def test_qmatmul_decode(ctx, dev, oracle, bits, M, N, K, parts):
    """The decode form (M <= 16): weight stream on mma.sync, K parts reduced across a thread-block cluster; 9-16
    tokens on 513 or 512 row blocks take the register-capped build (one wave at four CTAs per SM)."""
    import torch
    X, codes, S = _mm_case(M, N, K, bits, 5 * M + N + K)
    Y = torch.full((M, N), -1, dtype=torch.int16, device=dev)
    ctx.call("qmatmul_form", to_dev(X, dev), to_dev(codes, dev), to_dev(S, dev), Y, M, N, K, bits, 5, parts)
    ctx.sync(60000)
    _close_mm(f16_of(Y), oracle.qmatmul(X, codes, S, N, K, bits).view(np.float16).astype(np.float32))


@pytest.mark.parametrize("bits", [8, 4])
def test_qmatmul_decode_unaligned_scales(ctx, dev, oracle, bits):
    """Scales 2 bytes past a 16-byte boundary (the decode form reads each lane's scale on its own)."""
    import torch
    M, N, K = 3, 1024, 2048
    X, codes, S = _mm_case(M, N, K, bits, 17)
    raw = torch.zeros(S.size + 8, dtype=torch.int16, device=dev)
    raw[1:1 + S.size] = torch.from_numpy(S.reshape(-1).view(np.int16)).to(dev)
    s_odd = raw[1:1 + S.size]  # 2 bytes past a 16-byte boundary
    Y = torch.full((M, N), -1, dtype=torch.int16, device=dev)
    ctx.call("qmatmul_form", to_dev(X, dev), to_dev(codes, dev), s_odd, Y, M, N, K, bits, 5, 0)
    ctx.sync(60000)
    _close_mm(f16_of(Y), oracle.qmatmul(X, codes, S, N, K, bits).view(np.float16).astype(np.float32))


@pytest.mark.parametrize("M,N,K,bits,parts", [(16, 4104, 4096, 8, 0), (12, 2048, 8224, 8, 0), (16, 2048, 8192, 8, 4),
                                              (9, 5000, 2048, 4, 0), (13, 4800, 2080, 4, 0), (16, 6144, 8192, 4, 2),
                                              (11, 5120, 3072, 4, 0)])
def test_qmatmul_decode_staged(ctx, dev, oracle, M, N, K, bits, parts):
    """The staged decode form (bulk copies into shared memory; 9-16 tokens on large q8 weights and on q4 weights
    of 297-444 row blocks): ragged N, K not a multiple of the step, K parts reduced across a cluster."""
    import torch
    X, codes, S = _mm_case(M, N, K, bits, 7 * M + N + K)
    Y = torch.full((M, N), -1, dtype=torch.int16, device=dev)
    ctx.call("qmatmul_form", to_dev(X, dev), to_dev(codes, dev), to_dev(S, dev), Y, M, N, K, bits, 5, parts)
    ctx.sync(60000)
    _close_mm(f16_of(Y), oracle.qmatmul(X, codes, S, N, K, bits).view(np.float16).astype(np.float32))


@pytest.mark.parametrize("bits,M,N", [(8, 9, 4096), (4, 2, 2048)])
def test_qmatmul_decode_staged_unaligned_scales(ctx, dev, oracle, bits, M, N):
    """Scale rows 2 bytes past a 16-byte boundary: the staged form loads them without bulk copies."""
    import torch
    K = 4096
    X, codes, S = _mm_case(M, N, K, bits, 19)
    raw = torch.zeros(S.size + 8, dtype=torch.int16, device=dev)
    raw[1:1 + S.size] = torch.from_numpy(S.reshape(-1).view(np.int16)).to(dev)
    Y = torch.full((M, N), -1, dtype=torch.int16, device=dev)
    ctx.call("qmatmul_form", to_dev(X, dev), to_dev(codes, dev), raw[1:1 + S.size], Y, M, N, K, bits, 5, 0)
    ctx.sync(60000)
    _close_mm(f16_of(Y), oracle.qmatmul(X, codes, S, N, K, bits).view(np.float16).astype(np.float32))


@pytest.mark.parametrize("bits", [8, 4])
@pytest.mark.parametrize("M,N,K,parts", [(17, 768, 768, 0), (32, 1152, 768, 2), (33, 3072, 1024, 0),
                                         (64, 1024, 3072, 4), (48, 200, 320, 0), (64, 130, 8192, 0),
                                         (20, 8192, 3072, 0), (24, 5000, 3072, 0)])
def test_qmatmul_decode_wide(ctx, dev, oracle, bits, M, N, K, parts):
    """The register decode form at 17-64 tokens (four or eight 8-token tiles per MMA step): ragged N and K, K parts
    across a cluster; 24 x 5000 x 3072 takes the register-capped build (313 row blocks: one wave at three CTAs per
    SM, two at two)."""
    import torch
    X, codes, S = _mm_case(M, N, K, bits, 11 * M + N + K)
    Y = torch.full((M, N), -1, dtype=torch.int16, device=dev)
    ctx.call("qmatmul_form", to_dev(X, dev), to_dev(codes, dev), to_dev(S, dev), Y, M, N, K, bits, 5, parts)
    ctx.sync(60000)
    _close_mm(f16_of(Y), oracle.qmatmul(X, codes, S, N, K, bits).view(np.float16).astype(np.float32))


def test_qmatmul_decode_deterministic(ctx, dev, oracle):
    """Cluster partials are added in part order: repeated launches agree bit for bit."""
    import torch
    M, N, K = 4, 4096, 4096
    X, codes, S = _mm_case(M, N, K, 8, 3)
    args = [to_dev(X, dev), to_dev(codes, dev), to_dev(S, dev)]
    Ys = [torch.empty((M, N), dtype=torch.int16, device=dev) for _ in range(3)]
    for Y in Ys:
        ctx.call("qmatmul_form", *args, Y, M, N, K, 8, 5, 8)
    ctx.sync(60000)
    assert torch.equal(Ys[0], Ys[1]) and torch.equal(Ys[0], Ys[2])


@pytest.mark.parametrize("form,M", [(3, 1024), (6, 1024), (4, 64), (1, 64), (5, 8)])
def test_static_weights_chain(ctx, dev, form, M):
    """dc_static_weights lets the weight side of a matmul start before the kernel before it completes, while its
    token side still waits for that kernel: a chain of dependent matmuls gives the same bits either way."""
    import torch
    from decision_js_b200._lib import lib
    K, L = 768, 6
    rng = np.random.default_rng(form + M)
    X = to_dev((rng.standard_normal((M, K))).astype(np.float16), dev)
    dW = []
    for i in range(L):
        _, codes, S = _mm_case(1, K, K, 8, 100 + i)
        dW.append((to_dev(codes, dev), to_dev((S.astype(np.float32) / 20).astype(np.float16), dev)))  # rms ~1
    outs = []
    for on in (0, 1, 0, 1):
        assert lib().dc_static_weights(ctx.h, on) == 0
        bufs = [X] + [torch.full((M, K), -1, dtype=torch.int16, device=dev) for _ in range(L)]
        for i in range(L):
            ctx.call("qmatmul_form", bufs[i], *dW[i], bufs[i + 1], M, K, K, 8, form, 0)
        ctx.sync(60000)
        outs.append(bufs[-1].clone())
    lib().dc_static_weights(ctx.h, 0)
    assert np.isfinite(f16_of(outs[0])).all() and np.abs(f16_of(outs[0])).max() > 0
    assert all(torch.equal(outs[0], o) for o in outs[1:])


def _interleave_rows(a, I):
    """Rows of a fused gate|up weight in the load-time layout: gate row i at 2i, up row i at 2i + 1."""
    perm = np.stack([np.arange(I), I + np.arange(I)], axis=1).reshape(-1)
    return np.ascontiguousarray(a.reshape(2 * I, -1)[perm])


@pytest.mark.parametrize("epi,act", [(1, 1), (2, 0)])
@pytest.mark.parametrize("bits", [8, 4])
@pytest.mark.parametrize("M,I,K", [(1000, 1152, 768), (333, 192, 320), (4096, 3072, 1024), (40, 512, 256)])
def test_qmatmul_gated_epilogue(ctx, dev, oracle, epi, act, bits, M, I, K):
    import torch
    X, codes, S = _mm_case(M, 2 * I, K, bits, M + I + epi)
    Y = torch.full((M, I), -1, dtype=torch.int16, device=dev)
    ctx.call("qmatmul", to_dev(X, dev), to_dev(_interleave_rows(codes, I), dev), to_dev(_interleave_rows(S, I), dev),
             Y, M, 2 * I, K, bits, epi)
    ctx.sync(60000)
    ref = oracle.glu(oracle.qmatmul(X, codes, S, 2 * I, K, bits), I, act).view(np.float16).astype(np.float32)
    _close_mm(f16_of(Y), ref)


def _f16_weights(ctx, dev, codes, S, N, K, bits):
    """The weights dequantized on the device (dc_dequant), as the direct form's load step makes them."""
    import torch
    W16 = torch.empty((N, K), dtype=torch.int16, device=dev)
    ctx.call("dequant", to_dev(codes, dev), to_dev(S, dev), W16, N, K, bits)
    return W16


@pytest.mark.parametrize("bits", [8, 4])
@pytest.mark.parametrize("M,N,K", [(256, 384, 256), (300, 520, 768), (1000, 1152, 768), (513, 3072, 3104),
                                   (4096, 768, 1152), (40, 256, 96)])
def test_qmatmul_f16_direct(ctx, dev, oracle, bits, M, N, K):
    """The direct form (matmulDirect: weights dequantized to f16 once, then a CTA-pair tcgen05 GEMM fed by TMA):
    ragged M and N, K not a multiple of the 64-wide K block, against the oracle on the codes."""
    import torch
    X, codes, S = _mm_case(M, N, K, bits, 3 * M + N + K)
    W16 = _f16_weights(ctx, dev, codes, S, N, K, bits)
    Y = torch.full((M, N), -1, dtype=torch.int16, device=dev)
    ctx.call("qmatmul_f16", to_dev(X, dev), W16, Y, M, N, K, 0)
    ctx.sync(60000)
    _close_mm(f16_of(Y), oracle.qmatmul(X, codes, S, N, K, bits).view(np.float16).astype(np.float32))


@pytest.mark.parametrize("epi,act", [(1, 1), (2, 0)])
@pytest.mark.parametrize("M,I,K", [(1000, 1152, 768), (333, 192, 320), (4096, 3072, 1024)])
def test_qmatmul_f16_direct_gated(ctx, dev, oracle, epi, act, M, I, K):
    import torch
    X, codes, S = _mm_case(M, 2 * I, K, 8, M + I + epi + 7)
    W16 = _f16_weights(ctx, dev, _interleave_rows(codes, I), _interleave_rows(S, I), 2 * I, K, 8)
    Y = torch.full((M, I), -1, dtype=torch.int16, device=dev)
    ctx.call("qmatmul_f16", to_dev(X, dev), W16, Y, M, 2 * I, K, epi)
    ctx.sync(60000)
    ref = oracle.glu(oracle.qmatmul(X, codes, S, 2 * I, K, 8), I, act).view(np.float16).astype(np.float32)
    _close_mm(f16_of(Y), ref)


@pytest.mark.parametrize("form", [1, 4])
def test_qmatmul_repeat_split_counters(ctx, dev, oracle, form):
    """Split-K tile counters return to zero: the same launch twice gives the same result."""
    import torch
    M, N, K = 8, 512, 2048
    X, codes, S = _mm_case(M, N, K, 8, 11)
    args = [to_dev(X, dev), to_dev(codes, dev), to_dev(S, dev)]
    Y1 = torch.empty((M, N), dtype=torch.int16, device=dev)
    Y2 = torch.empty((M, N), dtype=torch.int16, device=dev)
    ctx.call("qmatmul_form", *args, Y1, M, N, K, 8, form, 8)
    ctx.call("qmatmul_form", *args, Y2, M, N, K, 8, form, 8)
    ctx.sync(60000)
    assert torch.equal(Y1, Y2)
    _close_mm(f16_of(Y1), oracle.qmatmul(X, codes, S, N, K, 8).view(np.float16).astype(np.float32))


@pytest.mark.parametrize("bits", [8, 4])
@pytest.mark.parametrize("M,N,K,splits", [(200, 1152, 768, 0), (256, 768, 3072, 2), (1000, 384, 1024, 3),
                                          (300, 256, 4096, 5), (129, 640, 96, 1)])
def test_qmatmul_form4_many_token_tiles(ctx, dev, oracle, bits, M, N, K, splits):
    """The 64-token form above 128 tokens (several token tiles per weight tile), with and without K splits."""
    import torch
    X, codes, S = _mm_case(M, N, K, bits, 3 * M + N)
    Y = torch.full((M, N), -1, dtype=torch.int16, device=dev)
    ctx.call("qmatmul_form", to_dev(X, dev), to_dev(codes, dev), to_dev(S, dev), Y, M, N, K, bits, 4, splits)
    ctx.sync(60000)
    _close_mm(f16_of(Y), oracle.qmatmul(X, codes, S, N, K, bits).view(np.float16).astype(np.float32))


def test_qmatmul_dispatch(ctx, dev, oracle):
    import torch
    for M in (1, 64, 129, 512, 2048, 8192):
        N, K = 768, 768
        X, codes, S = _mm_case(M, N, K, 8, M)
        Y = torch.empty((M, N), dtype=torch.int16, device=dev)
        ctx.call("qmatmul", to_dev(X, dev), to_dev(codes, dev), to_dev(S, dev), Y, M, N, K, 8, 0)
        ctx.sync(60000)
        _close_mm(f16_of(Y), oracle.qmatmul(X, codes, S, N, K, 8).view(np.float16).astype(np.float32))


def _f16(rng, shape, scale=1.0):
    return (rng.standard_normal(shape) * scale).astype(np.float16)


@pytest.mark.parametrize("H", [768, 1024, 3072, 136])
@pytest.mark.parametrize("add", [0, 1])
def test_add_rmsnorm(ctx, dev, oracle, H, add):
    import torch
    rng = np.random.default_rng(H + add)
    T = 37
    X, Y, W = _f16(rng, (T, H)), _f16(rng, (T, H)), _f16(rng, (H,), 0.3) + np.float16(1)
    dX, dO = to_dev(X, dev), torch.empty((T, H), dtype=torch.int16, device=dev)
    ctx.call("add_rmsnorm", dX, to_dev(Y, dev), to_dev(W, dev), dO, T, H, add, 1e-6)
    ctx.sync(60000)
    rX, rO = oracle.add_rmsnorm(X, Y, W, add, 1e-6)
    assert rel_err(f16_of(dX), rX.view(np.float16).astype(np.float32)) < 1e-3
    assert rel_err(f16_of(dO), rO.view(np.float16).astype(np.float32)) < 4e-3


@pytest.mark.parametrize("H", [768, 1024, 3072, 4096])
@pytest.mark.parametrize("norm2", [0, 1])
def test_sandwich(ctx, dev, oracle, H, norm2):
    import torch
    rng = np.random.default_rng(H + 3 * norm2)
    T = 29
    X, Y = _f16(rng, (T, H)), _f16(rng, (T, H))
    W1, W2 = _f16(rng, (H,), 0.3) + np.float16(1), _f16(rng, (H,), 0.3) + np.float16(1)
    dX, dO = to_dev(X, dev), torch.zeros((T, H), dtype=torch.int16, device=dev)
    ctx.call("sandwich", dX, to_dev(Y, dev), to_dev(W1, dev), to_dev(W2, dev) if norm2 else None, dO, T, H, 1e-6,
             0.75)
    ctx.sync(60000)
    rX, rO = oracle.sandwich(X, Y, W1, W2 if norm2 else None, 1e-6, 0.75)
    assert rel_err(f16_of(dX), rX.view(np.float16).astype(np.float32)) < 4e-3
    if norm2:
        assert rel_err(f16_of(dO), rO.view(np.float16).astype(np.float32)) < 4e-3


# one group of passes per token (the encoder, small heads), two groups (configs 3 and 4, D = 64 with 48 heads, D = 512
# with 16), four groups with a partly empty last one (D = 128 with 56 heads)
@pytest.mark.parametrize("D,heads,kv,vnorm", [(256, 3, 1, 1), (128, 16, 8, 0), (128, 24, 8, 0), (64, 4, 2, 1),
                                              (512, 2, 1, 1), (64, 32, 8, 1), (128, 40, 8, 1), (512, 8, 4, 1)])
def test_qkv_norm_rope(ctx, dev, oracle, D, heads, kv, vnorm):
    rng = np.random.default_rng(D + heads)
    T = 41
    Z = _f16(rng, (T, (heads + 2 * kv) * D))
    qn, kn = _f16(rng, (D,), 0.2) + np.float16(1), _f16(rng, (D,), 0.2) + np.float16(1)
    pos = rng.integers(0, 1024, T).astype(np.int32)
    dZ = to_dev(Z, dev)
    ctx.call("qkv_norm_rope", dZ, to_dev(qn, dev), to_dev(kn, dev), to_dev(pos, dev), T, heads, kv, D, 1e-6,
             10000.0, vnorm)
    ctx.sync(60000)
    ref = oracle.qkv_norm_rope(Z, qn, kn, pos, heads, kv, D, 1e-6, 10000.0, vnorm).view(np.float16).astype(np.float32)
    assert rel_err(f16_of(dZ), ref) < 1e-2
    if not vnorm:  # v heads are left exactly as they were
        v0 = (heads + kv) * D
        assert np.array_equal(dZ.cpu().numpy().reshape(T, -1)[:, v0:], Z.view(np.int16)[:, v0:])


@pytest.mark.parametrize("act", [0, 1])
def test_glu(ctx, dev, oracle, act):
    import torch
    rng = np.random.default_rng(act)
    T, I = 33, 1152
    A = _f16(rng, (T, 2 * I), 2.0)
    dH = torch.empty((T, I), dtype=torch.int16, device=dev)
    ctx.call("glu", to_dev(A, dev), dH, T, I, act)
    ctx.sync(60000)
    assert rel_err(f16_of(dH), oracle.glu(A, I, act).view(np.float16).astype(np.float32)) < 4e-3


@pytest.mark.parametrize("bits", [8, 4])
def test_gather_bit_exact(ctx, dev, oracle, bits):
    import torch
    V, H, T = 1000, 768, 77
    _, codes, S = _mm_case(1, V, H, bits, 5)
    ids = np.random.default_rng(1).integers(0, V, T).astype(np.int32)
    dX = torch.empty((T, H), dtype=torch.int16, device=dev)
    ctx.call("gather", to_dev(ids, dev), to_dev(codes, dev), to_dev(S, dev), dX, T, H, bits)
    ctx.sync(60000)
    assert np.array_equal(dX.cpu().numpy().view(np.uint16), oracle.gather(ids, codes, S, H, bits))


@pytest.mark.parametrize("proj", [False, True])
def test_pool(ctx, dev, oracle, proj):
    import torch
    rng = np.random.default_rng(9)
    H = 768
    lens = [5, 256, 1, 77]
    T = sum(lens)
    X = _f16(rng, (T, H))
    ends = np.cumsum(lens)
    seqs = np.stack([ends - lens, ends], 1).astype(np.int32)
    W = _f16(rng, (512, H), 0.05) if proj else None
    N = 512 if proj else H
    out = torch.empty((len(lens), N), dtype=torch.float32, device=dev)
    ctx.call("pool", to_dev(X, dev), to_dev(seqs, dev), to_dev(W, dev) if proj else None, out, len(lens), H, N)
    ctx.sync(60000)
    assert rel_err(out.cpu().numpy(), oracle.pool(X, seqs, W)) < 1e-4


@pytest.mark.parametrize("bits,H", [(8, 1024), (4, 3072)])
def test_leaf_logits(ctx, dev, oracle, bits, H):
    import torch
    rng = np.random.default_rng(bits)
    V, T, L, n = 5000, 50, 7, 10
    X = _f16(rng, (T, H))
    W = _f16(rng, (H,), 0.2) + np.float16(1)
    _, codes, S = _mm_case(1, V, H, bits, 8)
    leaves = rng.integers(0, T, L).astype(np.int32)
    ids = rng.integers(0, V, (L, n)).astype(np.int32)
    out = torch.empty((L, n), dtype=torch.float32, device=dev)
    ctx.call("leaf_logits", to_dev(X, dev), to_dev(leaves, dev), to_dev(W, dev), to_dev(ids, dev),
             to_dev(codes, dev), to_dev(S, dev), out, L, H, n, bits, 1e-5)
    ctx.sync(60000)
    assert rel_err(out.cpu().numpy(), oracle.leaf_logits(X, leaves, W, ids, codes, S, bits, 1e-5)) < 1e-4


def _ranges_bidir(lens):
    rng = []
    s = 0
    for n in lens:
        rng += [(s, s + n, 0, 0)] * n
        s += n
    return np.array(rng, np.int32)


def _ranges_causal(lens):
    rng = []
    s = 0
    for n in lens:
        rng += [(s, s + i + 1, 0, 0) for i in range(n)]
        s += n
    return np.array(rng, np.int32)


def _ranges_tree():
    from decision_js_b200 import forest
    trees = [{"trunk": list(range(70)), "branches": [[1] * 5, [2] * 9, [3] * 3], "groups": [[[1]], [[2]], [[3]]]},
             {"trunk": list(range(130)), "branches": [[4] * 17], "groups": [[[1]]]}]
    return forest(trees)[2]


@pytest.mark.parametrize("form", [0, 1])
@pytest.mark.parametrize("D,heads,kv", [(256, 3, 1), (128, 16, 8), (128, 24, 8)])
@pytest.mark.parametrize("mask", ["bidir", "causal", "tree", "window"])
def test_attention(ctx, dev, oracle, form, D, heads, kv, mask):
    import torch
    lens = [256, 100, 1, 63]
    if mask == "bidir":
        r = _ranges_bidir(lens)
    elif mask == "causal":
        r = _ranges_causal(lens)
    elif mask == "tree":
        r = _ranges_tree()
    else:
        r = _ranges_bidir(lens)
        t = np.arange(len(r))
        r[:, 0] = np.maximum(r[:, 0], t - 40)
        r[:, 1] = np.minimum(r[:, 1], t + 41)
    T = len(r)
    rng = np.random.default_rng(D + heads)
    Z = _f16(rng, (T, (heads + 2 * kv) * D))
    scale = 1.0 / np.sqrt(D)
    dY = torch.empty((T, heads * D), dtype=torch.int16, device=dev)
    ctx.call("attention_form", to_dev(Z, dev), to_dev(r, dev), dY, T, heads, kv, D, float(scale), form)
    ctx.sync(60000)
    ref = oracle.attention(Z, r, heads, kv, D, scale).view(np.float16).astype(np.float32)
    got = f16_of(dY)
    assert np.abs(got - ref).max() < ATTN_TOL * np.abs(ref).max(), rel_err(got, ref)


@pytest.mark.parametrize("D,heads,kv", [(256, 3, 1), (128, 24, 8)])
def test_attention_long_causal(ctx, dev, oracle, D, heads, kv):
    """Causal rows over 1024 keys (many key blocks per tile, rescales as the row max grows) and a bidirectional
    sequence of 700 (a tile straddling two sequences), tensor-core kernel against the oracle."""
    import torch
    r = np.concatenate([_ranges_causal([1024]), _ranges_bidir([700])])
    r[1024:, :2] += 1024
    T = len(r)
    rng = np.random.default_rng(D)
    Z = _f16(rng, (T, (heads + 2 * kv) * D), 2.0)
    scale = 1.0 / np.sqrt(D)
    dY = torch.empty((T, heads * D), dtype=torch.int16, device=dev)
    ctx.call("attention_form", to_dev(Z, dev), to_dev(r, dev), dY, T, heads, kv, D, float(scale), 1)
    ctx.sync(60000)
    ref = oracle.attention(Z, r, heads, kv, D, scale).view(np.float16).astype(np.float32)
    got = f16_of(dY)
    assert np.abs(got - ref).max() < ATTN_TOL * np.abs(ref).max(), rel_err(got, ref)


def test_empty_inputs_write_nothing(ctx, dev):
    """T = 0 (S = 0 sequences, L = 0 readouts): every op returns DC_OK at once and writes nothing, as the
    reference's recorder dispatches no workgroups for an empty pass."""
    import torch
    buf = torch.full((4096,), 7, dtype=torch.int16, device=dev)
    i32 = torch.zeros(64, dtype=torch.int32, device=dev)
    f32 = torch.full((64,), 5.0, dtype=torch.float32, device=dev)
    ctx.call("add_rmsnorm", buf, buf, buf, buf, 0, 256, 1, 1e-6)
    ctx.call("sandwich", buf, buf, buf, buf, buf, 0, 256, 1e-6, 1.0)
    ctx.call("qkv_norm_rope", buf, buf, buf, i32, 0, 4, 2, 128, 1e-6, 1e4, 0)
    ctx.call("attention", buf, i32, buf, 0, 4, 2, 128, 0.1)
    ctx.call("attention_form", buf, i32, buf, 0, 4, 2, 128, 0.1, 0)
    ctx.call("glu", buf, buf, 0, 256, 0)
    ctx.call("gather", i32, buf, buf, buf, 0, 256, 8)
    ctx.call("pool", buf, i32, None, f32, 0, 256, 0)
    ctx.call("leaf_logits", buf, i32, buf, i32, buf, buf, f32, 0, 256, 4, 8, 1e-6)
    ctx.call("leaf_logits", buf, i32, buf, i32, buf, buf, f32, 2, 256, 0, 8, 1e-6)
    ctx.sync(10000)
    assert bool((buf == 7).all()) and bool((f32 == 5.0).all())


def test_bounded_wait_expires_and_the_context_stays_usable(ctx, dev, oracle):
    """Failure detection without a fault: a kernel's bounded wait on a barrier that nothing completes expires after
    20 ms, flags the device error word and ends; dc_sync reports DC_ETIMEOUT once (the word is cleared), and the
    context then computes a matmul correctly."""
    import torch
    from decision_js_b200._lib import DC_ETIMEOUT, DecisionError, lib
    assert lib().dc_selftest_wait(ctx.h, 20000) == 0
    with pytest.raises(DecisionError) as e:
        ctx.sync(10000)
    assert e.value.code == DC_ETIMEOUT and "bounded wait expired" in str(e.value)
    ctx.sync(10000)  # reported once
    M, N, K = 4, 256, 512
    X, codes, S = _mm_case(M, N, K, 8, 21)
    Y = torch.empty((M, N), dtype=torch.int16, device=dev)
    ctx.call("qmatmul", to_dev(X, dev), to_dev(codes, dev), to_dev(S, dev), Y, M, N, K, 8, 0)
    ctx.sync(60000)
    _close_mm(f16_of(Y), oracle.qmatmul(X, codes, S, N, K, 8).view(np.float16).astype(np.float32))


@pytest.mark.parametrize("form,D,heads,kv", [(0, 64, 32, 8), (1, 64, 32, 8), (1, 64, 8, 8), (0, 512, 4, 1),
                                             (0, 512, 8, 2)])
@pytest.mark.parametrize("mask", ["bidir", "causal", "tree", "window"])
def test_attention_head_dims_64_512(ctx, dev, oracle, form, D, heads, kv, mask):
    """d1-3B's 64-wide heads (src/kernels.ts:117-147, both kernels) and EmbeddingGemma 2's 512-wide heads of its
    full layers (src/eg2-kernels.ts:104; the mma.sync kernel, each block one 256-wide half of the output head)."""
    import torch
    lens = [256, 100, 1, 63]
    if mask == "bidir":
        r = _ranges_bidir(lens)
    elif mask == "causal":
        r = _ranges_causal(lens)
    elif mask == "tree":
        r = _ranges_tree()
    else:
        r = _ranges_bidir(lens)
        t = np.arange(len(r))
        r[:, 0] = np.maximum(r[:, 0], t - 40)
        r[:, 1] = np.minimum(r[:, 1], t + 41)
    T = len(r)
    rng = np.random.default_rng(D + heads + form)
    Z = _f16(rng, (T, (heads + 2 * kv) * D))
    scale = 1.0 / np.sqrt(D)
    dY = torch.full((T, heads * D), -1, dtype=torch.int16, device=dev)
    ctx.call("attention_form", to_dev(Z, dev), to_dev(r, dev), dY, T, heads, kv, D, float(scale), form)
    ctx.sync(60000)
    ref = oracle.attention(Z, r, heads, kv, D, scale).view(np.float16).astype(np.float32)
    got = f16_of(dY)
    assert np.abs(got - ref).max() < ATTN_TOL * np.abs(ref).max(), rel_err(got, ref)


def test_attention_default_takes_every_head_dim(ctx, dev, oracle):
    """dc_attention (the form picked by D) at the four head dims, a causal and a bidirectional sequence."""
    import torch
    r = np.concatenate([_ranges_causal([300]), _ranges_bidir([200])])
    r[300:, :2] += 300
    T = len(r)
    for D, heads, kv in ((64, 16, 4), (128, 8, 2), (256, 3, 1), (512, 2, 1)):
        rng = np.random.default_rng(D)
        Z = _f16(rng, (T, (heads + 2 * kv) * D))
        dY = torch.full((T, heads * D), -1, dtype=torch.int16, device=dev)
        ctx.call("attention", to_dev(Z, dev), to_dev(r, dev), dY, T, heads, kv, D, float(D ** -0.5))
        ctx.sync(60000)
        ref = oracle.attention(Z, r, heads, kv, D, D ** -0.5).view(np.float16).astype(np.float32)
        got = f16_of(dY)
        assert np.abs(got - ref).max() < ATTN_TOL * np.abs(ref).max(), (D, rel_err(got, ref))


def _random_taps(T, rng):
    """Taps as the reference builds them for a forest, plus arbitrary rows and -1s."""
    t = np.arange(T)
    taps = np.stack([t - 2, t - 1, t, np.zeros(T, np.int64)], 1)
    taps[rng.random(T) < 0.1, 0] = -1
    taps[rng.random(T) < 0.05, 1] = -1
    jump = rng.random(T) < 0.1
    taps[jump, 0] = rng.integers(0, T, int(jump.sum()))
    taps[taps < -1] = -1
    return taps.astype(np.int32)


@pytest.mark.parametrize("H", [2048, 1024, 136])
def test_short_conv_bit_exact(ctx, dev, oracle, H):
    """SHORT_CONV (src/kernels.ts:65-84): the same f32 products and sums in the same order as the oracle, one f16
    rounding: bit for bit."""
    import torch
    rng = np.random.default_rng(H)
    T = 333
    Z = _f16(rng, (T, 3 * H))
    Wc = _f16(rng, (H, 3), 0.5)
    taps = _random_taps(T, rng)
    dY = torch.full((T, H), -1, dtype=torch.int16, device=dev)
    ctx.call("short_conv", to_dev(Z, dev), to_dev(Wc, dev), to_dev(taps, dev), dY, T, H)
    ctx.sync(60000)
    assert np.array_equal(dY.cpu().numpy().view(np.uint16), oracle.short_conv(Z, Wc, taps))


@pytest.mark.parametrize("P", [512, 256, 1024, 72])
def test_ple_mix(ctx, dev, oracle, P):
    """PLE_MIX (src/eg2-kernels.ts:181-200) within about one f16 rounding."""
    import torch
    rng = np.random.default_rng(P)
    T = 257
    G, E = _f16(rng, (T, P), 2.0), _f16(rng, (T, P), 3.0)
    W = _f16(rng, (P,), 0.2) + np.float16(1)
    dO = torch.full((T, P), -1, dtype=torch.int16, device=dev)
    ctx.call("ple_mix", to_dev(G, dev), to_dev(E, dev), to_dev(W, dev), dO, T, P, 1e-6)
    ctx.sync(60000)
    ref = oracle.ple_mix(G, E, W, 1e-6).view(np.float16).astype(np.float32)
    got = f16_of(dO)
    assert np.abs(got - ref).max() <= 2e-3 * np.abs(ref).max(), rel_err(got, ref)


def test_readout(ctx, dev, oracle):
    """READOUT (src/d3-kernels.ts:243-260): f32 dots of readout rows with f32 code rows."""
    import torch
    rng = np.random.default_rng(5)
    T, H, C, P = 90, 1024, 24, 37
    X = _f16(rng, (T, H))
    R = rng.standard_normal((C, H)).astype(np.float32)
    pairs = np.stack([rng.integers(0, T, P), rng.integers(0, C, P)], 1).astype(np.int32)
    out = torch.empty(P, dtype=torch.float32, device=dev)
    ctx.call("readout", to_dev(X, dev), torch.from_numpy(R).to(dev), to_dev(pairs, dev), out, P, H, T, C)
    ctx.sync(60000)
    assert rel_err(out.cpu().numpy(), oracle.readout(X, R, pairs)) < 1e-5


@pytest.mark.parametrize("H,trunk,branches,plain,big_a", [(2, 5, (7, 4), (19,), False),
                                                           (3, 37, (50, 3, 1), (300, 1, 16), True)])
def test_gdn(ctx, dev, oracle, H, trunk, branches, plain, big_a):
    """The Gated DeltaNet mixer (src/d3-kernels.ts:23-149) against the oracle: shared trunks with several branches
    (only the first writes the trunk), one-token spans, sequences of many 16-token chunks, and gate inputs past the
    softplus cut-off (a > 20)."""
    import torch
    from test_host import gdn_case
    c = gdn_case(17 + H, H=H, trunk=trunk, branches=branches, plain=plain)
    if big_a:
        c["Z"][::3, c["qkv"] + 128 * H + H:c["qkv"] + 128 * H + 2 * H] = 25.0
    ref = oracle.gdn(c["Z"], c["stride"], c["qkv"], H, c["W"], c["Alog"], c["dtb"], c["gw"], c["spans"], c["eps"],
                     c["T"]).view(np.float16).astype(np.float32)
    Y = torch.zeros((c["T"], H * 128), dtype=torch.int16, device=dev)
    ctx.call("gdn", to_dev(c["Z"], dev), c["stride"], c["qkv"], H, to_dev(c["W"], dev), to_dev(c["Alog"], dev),
             to_dev(c["dtb"], dev), to_dev(c["gw"], dev), to_dev(c["spans"].view(np.int32), dev),
             len(c["spans"]), float(c["eps"]), Y, c["T"])
    ctx.sync(60000)
    got = f16_of(Y)
    tol = 4e-3 * np.abs(ref) + 2e-3 * np.abs(ref).max()
    assert (np.abs(got - ref) <= tol).all(), rel_err(got, ref)
    Y2 = torch.zeros_like(Y)
    ctx.call("gdn", to_dev(c["Z"], dev), c["stride"], c["qkv"], H, to_dev(c["W"], dev), to_dev(c["Alog"], dev),
             to_dev(c["dtb"], dev), to_dev(c["gw"], dev), to_dev(c["spans"].view(np.int32), dev),
             len(c["spans"]), float(c["eps"]), Y2, c["T"])
    ctx.sync(60000)
    assert torch.equal(Y, Y2)  # deterministic


def _ulp_close(got, ref, ulps=1):
    """f16 results within `ulps` units in the last place (CUDA's f32 exp and the C library's differ in their last
    bits, which moves an f16 rounding by one step at most)."""
    g = np.asarray(got, np.float16).astype(np.float32)
    r = np.asarray(ref, np.float16).astype(np.float32)
    spacing = np.spacing(np.abs(r).astype(np.float16)).astype(np.float32)
    return bool((np.abs(g - r) <= ulps * np.maximum(spacing, np.float32(6e-8))).all())


def test_omni_head_kernels(ctx, dev, oracle):
    """The d1-omni / Laya head kernels (src/kernels.ts:187-283) against the oracle: ADD_ROWS and GATHER_ROWS bit for
    bit, BIAS_ACT none / ReLU bit for bit and GELU (erf) to one f16 step, SCORE to f32 rounding, ADD_LAYERNORM (with
    and without the residual add and the bias) to the f16 rounding of a row sum in another order."""
    import torch
    rng = np.random.default_rng(31)
    T, H, nE = 300, 768, 3
    Xi = rng.standard_normal((T, H)).astype(np.float16)
    E = rng.standard_normal((nE, H)).astype(np.float16)
    idx = rng.integers(0, nE, T).astype(np.int32)
    Xo = torch.empty((T, H), dtype=torch.int16, device=dev)
    ctx.call("add_rows", to_dev(Xi, dev), to_dev(idx, dev), to_dev(E, dev), Xo, T, H, nE)
    ctx.sync(60000)
    assert np.array_equal(Xo.cpu().numpy().view(np.uint16), oracle.add_rows(Xi, idx, E))
    Y = (2 * rng.standard_normal((T, H))).astype(np.float16)
    b = rng.standard_normal(H).astype(np.float16)
    for act in (0, 1, 2):
        dY = to_dev(Y, dev)
        ctx.call("bias_act", dY, to_dev(b, dev), T, H, act)
        ctx.sync(60000)
        got, ref = dY.cpu().numpy().view(np.float16), oracle.bias_act(Y, b, act).view(np.float16)
        assert np.array_equal(got, ref) if act < 2 else _ulp_close(got, ref), act
    W = (1 + 0.1 * rng.standard_normal(H)).astype(np.float16)
    B = (0.1 * rng.standard_normal(H)).astype(np.float16)
    for add, bias in ((False, True), (True, True), (True, False)):
        dX, O = to_dev(Xi, dev), torch.empty((T, H), dtype=torch.int16, device=dev)
        ctx.call("add_layernorm", dX, to_dev(Y, dev) if add else None, to_dev(W, dev),
                 to_dev(B, dev) if bias else None, O, T, H, int(add), 1e-5)
        ctx.sync(60000)
        Xr, Or = oracle.add_layernorm(Xi, Y if add else None, W, B if bias else None, add, 1e-5)
        assert np.array_equal(dX.cpu().numpy().view(np.uint16), Xr)
        got, ref = f16_of(O), Or.view(np.float16).astype(np.float32)
        assert np.abs(got - ref).max() <= 4e-3 * np.abs(ref).max(), (add, bias, rel_err(got, ref))
    rows = rng.integers(0, T, 50).astype(np.int32)
    G = torch.empty((50, H), dtype=torch.int16, device=dev)
    ctx.call("gather_rows", to_dev(Xi, dev), to_dev(rows, dev), G, 50, H, T)
    w = rng.standard_normal(H).astype(np.float16)
    bb = np.array([0.5], np.float16)
    out = torch.empty(T, dtype=torch.float32, device=dev)
    ctx.call("score", to_dev(Y, dev), to_dev(w, dev), to_dev(bb, dev), out, T, H)
    ctx.sync(60000)
    assert np.array_equal(G.cpu().numpy().view(np.uint16), oracle.gather_rows(Xi, rows))
    assert rel_err(out.cpu().numpy(), oracle.score(Y, w, bb)) < 1e-5


def test_glu_gelu_erf(ctx, dev, oracle):
    """GELU_MUL with erf (Laya's, src/encoder-kernels.ts:26-44) to one f16 step."""
    import torch
    rng = np.random.default_rng(32)
    T, I = 200, 1152
    A = (2 * rng.standard_normal((T, 2 * I))).astype(np.float16)
    Hh = torch.empty((T, I), dtype=torch.int16, device=dev)
    ctx.call("glu", to_dev(A, dev), Hh, T, I, 2)
    ctx.sync(60000)
    assert _ulp_close(Hh.cpu().numpy().view(np.float16), oracle.glu(A, I, 2).view(np.float16))


@pytest.mark.parametrize("D,rot,norm,heads,kv,pad", [(256, 64, True, 8, 2, 2 * 256 + 2 * 8 * 256),
                                                     (64, 64, False, 12, 12, 12 * 64), (128, 32, True, 4, 1, 8),
                                                     (512, 256, True, 2, 1, 0)])
def test_qk_rope(ctx, dev, oracle, D, rot, norm, heads, kv, pad):
    """Q/K (norm +) RoPE in rows of any stride: d3-lite's QK_NORM_ROPE_256 (8 q + 2 k heads of 256, RoPE on 64 dims,
    v and gate heads after them untouched), Laya's ROPE (64-dim heads, no norm), partial rotations at D = 128, 512."""
    import torch
    rng = np.random.default_rng(33 + D)
    T, theta, eps = 333, 10000000.0 if D == 256 else 160000.0, 1e-6
    stride = (heads + kv) * D + pad
    Z = rng.standard_normal((T, stride)).astype(np.float16)
    qn = (1 + 0.1 * rng.standard_normal(D)).astype(np.float16)
    kn = (1 + 0.1 * rng.standard_normal(D)).astype(np.float16)
    pos = rng.integers(0, 4096, T).astype(np.int32)
    dZ = to_dev(Z, dev)
    ctx.call("qk_rope", dZ, to_dev(qn, dev), to_dev(kn, dev), to_dev(pos, dev), T, heads, kv, D, stride, rot,
             int(norm), eps, theta)
    ctx.sync(60000)
    got = dZ.cpu().numpy().view(np.float16).astype(np.float32)
    ref = oracle.qk_rope(Z, qn, kn, pos, heads, kv, D, rot, norm, eps, theta).view(np.float16).astype(np.float32)
    assert np.abs(got - ref).max() <= 2e-3 * np.abs(ref).max(), rel_err(got, ref)
    assert np.array_equal(got[:, (heads + kv) * D:], ref[:, (heads + kv) * D:])


@pytest.mark.parametrize("form", [0, 1])
@pytest.mark.parametrize("D,heads,kv,gate,pad", [(256, 8, 2, True, 0), (128, 4, 2, True, 24), (64, 6, 3, False, 40),
                                                 (512, 2, 1, True, 8)])
def test_attention_strided_gated(ctx, dev, oracle, form, D, heads, kv, gate, pad):
    """Attention over rows of any stride and d3-lite's gated form (src/d3-kernels.ts:174-240: the output times
    sigmoid of the q head's gate, the gates after the v heads; here over a shared trunk with branches and plain
    sequences, bidirectional as d3's mode is) against the oracle, both kernels."""
    import torch
    if form == 1 and D == 512:
        pytest.skip("the tensor-core kernel takes D <= 256")
    rng = np.random.default_rng(41 + D)
    r = np.concatenate([_ranges_tree(), _ranges_bidir([300, 17])])
    n_tree = len(_ranges_tree())
    r[n_tree:, :2] += n_tree
    T = len(r)
    stride = (2 * heads + 2 * kv if gate else heads + 2 * kv) * D + pad
    Z = rng.standard_normal((T, stride)).astype(np.float16)
    Y = torch.empty((T, heads * D), dtype=torch.int16, device=dev)
    scale = 1.0 / np.sqrt(D)
    ctx.call("attention_ex", to_dev(Z, dev), to_dev(r, dev), Y, T, heads, kv, D, float(scale), stride, int(gate), form)
    ctx.sync(60000)
    got = f16_of(Y)
    ref = oracle.attention_ex(Z, r, heads, kv, D, scale, gate).view(np.float16).astype(np.float32)
    assert np.abs(got - ref).max() < ATTN_TOL * np.abs(ref).max(), rel_err(got, ref)
