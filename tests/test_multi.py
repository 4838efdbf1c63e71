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


def _worker_forms(rank, world, port, out_dir):
    pkg, oracle, dist = _init(rank, world, port)
    from decision_js_b200 import multi
    res = {}
    # one request over two ranks: rank 1's shard is empty, the rows still come back as one tensor gather
    res["one"] = multi.run_sharded([[3.0]], [1], lambda b: [np.full(4, x[0], np.float32) for x in b])
    # rows of different widths per rank: the object path
    res["ragged"] = multi.run_sharded([[1], [2], [3]], [1, 1, 1],
                                      lambda b: [np.arange(x[0], dtype=np.float32) for x in b])
    # results that are not rows (probability lists): the object path
    res["lists"] = multi.run_sharded([[1], [2], [3]], [1, 1, 1], lambda b: [[x[0], 0.5] for x in b])
    # f64 rows of one width
    res["f64"] = multi.run_sharded([[1], [2], [3], [4]], [1, 1, 1, 1],
                                   lambda b: [np.full(2, x[0], np.float64) for x in b])
    if rank == 0:
        np.save(os.path.join(out_dir, "forms.npy"), np.array(res, dtype=object), allow_pickle=True)
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


def test_gloo_gather_forms(tmp_path):
    port = _port()
    mp.spawn(_worker_forms, args=(2, port, str(tmp_path)), nprocs=2, join=True)
    res = np.load(tmp_path / "forms.npy", allow_pickle=True).item()
    assert len(res["one"]) == 1 and res["one"][0].dtype == np.float32 and np.all(res["one"][0] == 3.0)
    assert [list(r) for r in res["ragged"]] == [[0.0], [0.0, 1.0], [0.0, 1.0, 2.0]]
    assert res["lists"] == [[1, 0.5], [2, 0.5], [3, 0.5]]
    assert [r.dtype for r in res["f64"]] == [np.float64] * 4
    assert [float(r[0]) for r in res["f64"]] == [1.0, 2.0, 3.0, 4.0]


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
