"""GPU (2 devices): column-split tensor parallelism over NCCL against the single-GPU runtime."""
import os
import socket

import numpy as np
import pytest

from conftest import cosine

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank(rank, world, port, path, tokens, out):
    import torch.distributed as dist
    from edge_maskgit_b200.tp import TPForward
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    logits = TPForward(path, rank, world).forward(tokens)
    torch.cuda.synchronize()
    if rank == 0:
        np.save(out, logits.cpu().numpy())
    dist.barrier()
    dist.destroy_process_group()


def test_tp2_matches_single_gpu(tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import multiprocessing as mp
    from edge_maskgit_b200 import runtime as rt, synth
    spec = synth.ModelSpec(n_layer=2, n_tokens=64, quant="gq4")
    path = synth.make_model(tmp_path / "tp.gguf", spec)
    rng = np.random.default_rng(3)
    tokens = rng.integers(0, spec.vocab_size, (2, spec.n_tokens + 1)).astype(np.int32)
    out = str(tmp_path / "tp.npy")
    ctx = mp.get_context("spawn")
    port = _port()
    ps = [ctx.Process(target=_rank, args=(r, 2, port, str(path), tokens, out)) for r in range(2)]
    for p in ps:
        p.start()
    for p in ps:
        p.join(300)
    assert [p.exitcode for p in ps] == [0, 0]
    tp = np.load(out)
    r = rt.CudaRuntime(path, max_rows=tokens.size)
    ref = r.forward(tokens)
    r.close()
    assert cosine(tp, ref) > 0.99999
    assert np.abs(tp - ref).max() < 1e-2


def _decode_rank(rank, world, port, path, out):
    import torch.distributed as dist
    from edge_maskgit_b200 import runtime as rt, shard
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    n = 6
    classes, seeds = shard.batch_classes(n), shard.batch_seeds(n)
    r = rt.CudaRuntime(path, max_rows=n * 65, device=rank)
    local = shard.decode_shard(lambda c, s, st, tp: r.generate(c, s, st, tp), classes, seeds, rank, world, steps=4)
    full = shard.gather_tokens(local, n, 65)
    if rank == 0:
        np.save(out, full)
    r.close()
    dist.barrier()
    dist.destroy_process_group()


def test_batch_sharded_decode_2gpu(tmp_path):
    """Config-4 style decode sharded by image over 2 GPUs, gathered with NCCL, equals one GPU."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import multiprocessing as mp
    from edge_maskgit_b200 import runtime as rt, shard, synth
    spec = synth.ModelSpec(n_layer=2, n_tokens=64, quant="gq8")
    path = synth.make_model(tmp_path / "dec.gguf", spec)
    out = str(tmp_path / "dec.npy")
    ctx = mp.get_context("spawn")
    port = _port()
    ps = [ctx.Process(target=_decode_rank, args=(r, 2, port, str(path), out)) for r in range(2)]
    for p in ps:
        p.start()
    for p in ps:
        p.join(300)
    assert [p.exitcode for p in ps] == [0, 0]
    r = rt.CudaRuntime(path, max_rows=6 * 65)
    ref = r.generate(shard.batch_classes(6), shard.batch_seeds(6), steps=4)
    r.close()
    assert np.array_equal(np.load(out), ref)
