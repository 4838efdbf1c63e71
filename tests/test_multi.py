"""The multi-process (one rank per GPU) host path on CPU with gloo, world size 2: request sharding and the ordered
host gather give the single-process result; the max-over-ranks timing reduction; a rank that fails between steps
makes the other rank's gather end with an error instead of hanging."""
import os
import socket
import sys
import tempfile
import time

import numpy as np
import pytest
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _init(rank, world, port, timeout_s=30):
    from datetime import timedelta
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=timeout_s))
    sys.path.insert(0, ROOT)
    import __graft_entry__ as ge
    return ge.load_package(), ge.load_oracle(), dist


def _worker_gather(rank, world, port, model_dir, out_dir):
    pkg, oracle, dist = _init(rank, world, port)
    from decision_js_b200 import multi, synth
    w = oracle.Weights(model_dir)
    reqs = synth.encoder_requests(5, 16, 512, seed=3) + synth.encoder_requests(2, 40, 512, seed=4)
    sizes = [len(r) for r in reqs]

    def engine(batch):
        emb = oracle.encoder_embed(w, np.concatenate(batch), [len(s) for s in batch])
        return [e for e in emb]

    got = multi.run_sharded(reqs, sizes, engine)
    slowest = multi.max_over_ranks(1.0 + rank)
    if rank == 0:
        np.save(os.path.join(out_dir, "got.npy"), np.stack(got))
        np.save(os.path.join(out_dir, "slowest.npy"), np.array([slowest]))
    dist.destroy_process_group()


def _worker_fail(rank, world, port, out_dir):
    pkg, oracle, dist = _init(rank, world, port, timeout_s=5)
    from decision_js_b200 import multi
    if rank == 1:
        raise RuntimeError("injected: rank 1 fails between steps")
    t0 = time.time()
    try:
        multi.run_sharded([[1], [2]], [1, 1], lambda b: b)
        status = "no error"
    except Exception as e:  # noqa: BLE001 - the peer's failure surfaces as a gloo error or timeout
        status = "error: " + type(e).__name__
    with open(os.path.join(out_dir, "rank0.txt"), "w") as f:
        f.write(f"{status} after {time.time() - t0:.1f}s")


@pytest.fixture(scope="module")
def tiny_encoder(pkg):
    from decision_js_b200 import synth
    d = tempfile.mkdtemp()
    synth.write_encoder(d, seed=2, layers=1, vocab=512, hidden=256, intermediate=256, heads=2,
                        head_dim={"sliding_attention": 128, "full_attention": 128},
                        kv_heads={"sliding_attention": 1, "full_attention": 1})
    return d


def test_gloo_sharded_gather_matches_single_process(oracle, tiny_encoder, tmp_path):
    from decision_js_b200 import synth
    port = _port()
    mp.spawn(_worker_gather, args=(2, port, tiny_encoder, str(tmp_path)), nprocs=2, join=True)
    got = np.load(tmp_path / "got.npy")
    w = oracle.Weights(tiny_encoder)
    reqs = synth.encoder_requests(5, 16, 512, seed=3) + synth.encoder_requests(2, 40, 512, seed=4)
    ref = oracle.encoder_embed(w, np.concatenate(reqs), [len(r) for r in reqs])
    assert got.shape == ref.shape
    assert np.array_equal(got, ref) or np.abs(got - ref).max() <= 1e-6 * np.abs(ref).max()
    assert float(np.load(tmp_path / "slowest.npy")[0]) == 2.0


def test_gloo_failed_rank_does_not_hang(tmp_path):
    port = _port()
    t0 = time.time()
    with pytest.raises(Exception):
        mp.spawn(_worker_fail, args=(2, port, str(tmp_path)), nprocs=2, join=True)
    assert time.time() - t0 < 120
    # rank 0 (if it got as far as the gather) reports an error rather than a result
    p = tmp_path / "rank0.txt"
    if p.exists():
        assert p.read_text().startswith("error")
