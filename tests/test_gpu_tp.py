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
    from edge_maskgit_b200 import runtime as rt
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    # the host exchange of the NCCL id only needs a CPU group; the runtime makes its own NCCL comm
    dist.init_process_group("gloo", rank=rank, world_size=world)
    obj = [rt.tp_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(obj, src=0)
    r = rt.CudaRuntime(path, max_rows=tokens.size, device=rank, tp=(rank, world, obj[0]))
    logits = r.forward(tokens)                                     # graph-captured step, host logits
    again = r.forward(tokens)
    r.close()
    np.save(out + f".{rank}.npy", logits)
    assert np.array_equal(logits, again)
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("q", ["gq4", "gq8"])
def test_tp2_matches_single_gpu(tmp_path, q):
    """The C++ column-split runtime over 2 GPUs: both ranks return the single-GPU logits bit for
    bit (every output element is computed as on one GPU; the attention of a head is the same
    kernel with the same key split)."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import multiprocessing as mp
    from edge_maskgit_b200 import runtime as rt, synth
    spec = synth.ModelSpec(n_layer=2, n_tokens=64, quant=q)
    path = synth.make_model(tmp_path / "tp.gguf", spec)
    rng = np.random.default_rng(3)
    tokens = rng.integers(0, spec.vocab_size, (2, spec.n_tokens + 1)).astype(np.int32)
    out = str(tmp_path / "tp")
    ctx = mp.get_context("spawn")
    port = _port()
    ps = [ctx.Process(target=_rank, args=(r, 2, port, str(path), tokens, out)) for r in range(2)]
    for p in ps:
        p.start()
    for p in ps:
        p.join(300)
    assert [p.exitcode for p in ps] == [0, 0]
    r = rt.CudaRuntime(path, max_rows=tokens.size)
    ref = r.forward(tokens)
    r.close()
    for k in range(2):
        tp = np.load(out + f".{k}.npy")
        assert cosine(tp, ref) > 0.99999
        assert np.array_equal(tp, ref), float(np.abs(tp - ref).max())


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
