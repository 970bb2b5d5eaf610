"""CPU: batch sharding of independent images over ranks (gloo, world size 2) and failure
handling of the gather, with the oracle decode loop standing in for a GPU per rank."""
import os
import socket
import tempfile

import numpy as np
import pytest

from conftest import SMALL


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_shard_range_partitions():
    from edge_maskgit_b200.shard import shard_range
    for n in (0, 1, 5, 64, 65):
        for w in (1, 2, 3, 8):
            spans = [shard_range(n, r, w) for r in range(w)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            assert max(h - l for l, h in spans) - min(h - l for l, h in spans) <= 1


def test_batch_workload_definition():
    from edge_maskgit_b200.shard import batch_classes, batch_seeds
    c = batch_classes()
    assert c.shape == (64,) and c.min() >= 0 and c.max() < 1000
    assert np.array_equal(c, np.random.default_rng(7).integers(0, 1000, 64))
    assert np.array_equal(batch_seeds()[:3], np.array([7, 8, 9], np.uint64))


def _worker(rank, world, port, model_path, out_dir, fail_rank):
    import torch.distributed as dist
    from datetime import timedelta
    from edge_maskgit_b200 import shard
    from oracle import oracle as O
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=8))
    classes = shard.batch_classes(5)
    seeds = shard.batch_seeds(5)
    m = O.OracleModel(model_path)
    local = shard.decode_shard(lambda c, s, st, t: m.generate(c, s, st, t), classes, seeds, rank, world, steps=3)
    if rank == fail_rank:
        os._exit(3)   # a rank that dies between steps, before the gather
    try:
        full = shard.gather_tokens(local, 5, m.n_tokens + 1)
        np.save(os.path.join(out_dir, f"r{rank}.npy"), full)
    except Exception as e:   # the surviving rank learns of the failure from the collective
        open(os.path.join(out_dir, f"r{rank}.err"), "w").write(type(e).__name__ + ": " + str(e))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def _run(world, fail_rank, small_models):
    import multiprocessing as mp
    path, _ = small_models["gq8"]
    out = tempfile.mkdtemp()
    port = _port()
    ctx = mp.get_context("spawn")
    ps = [ctx.Process(target=_worker, args=(r, world, port, str(path), out, fail_rank)) for r in range(world)]
    for p in ps:
        p.start()
    for p in ps:
        p.join(120)
        if p.is_alive():
            p.kill()
    return out, [p.exitcode for p in ps]


def test_gloo_sharded_decode_matches_single_process(oracle_mod, small_models):
    out, codes = _run(2, -1, small_models)
    assert codes == [0, 0]
    from edge_maskgit_b200 import shard
    path, _ = small_models["gq8"]
    m = oracle_mod.OracleModel(path)
    ref = m.generate(shard.batch_classes(5), shard.batch_seeds(5), steps=3)
    for r in range(2):
        assert np.array_equal(np.load(os.path.join(out, f"r{r}.npy")), ref)


def test_gloo_gather_reports_a_dead_rank(oracle_mod, small_models):
    out, codes = _run(2, 1, small_models)
    assert codes[1] == 3
    assert os.path.exists(os.path.join(out, "r0.err")), "surviving rank did not see the failure"
