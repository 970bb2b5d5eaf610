"""CPU (gloo, world size 2): the column split the tensor-parallel runtime uses, checked with the
oracle's GEMM as each rank's compute.  Rank r multiplies by the GGUF bytes of rows
[r*N/G, (r+1)*N/G) of a Q8_0 / Q4_K weight (rows are stored back to back, so a row range is one
byte range, as mgc_runtime_create_tp slices them), the slices are all-gathered into the
rank-major layout [G][M][N/G], and reading column k of row m at block k // w gives the full
GEMM bit for bit.  Also the address rule the runtime's in-place all-gather of the ffn_up
activation tiles relies on: a rank's F/G columns (a multiple of 128) are one contiguous run."""
import os
import socket
import tempfile

import numpy as np


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _row_bytes(wtype, K):
    return K // 32 * 34 if wtype == 8 else K // 256 * 144


def _worker(rank, world, port, out_dir):
    import torch
    import torch.distributed as dist
    from oracle import oracle as O
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    rng = np.random.default_rng(21)
    M, K, N = 37, 512, 384
    x = rng.standard_normal((M, K), dtype=np.float32)
    w = (rng.standard_normal((N, K), dtype=np.float32) * 0.02).astype(np.float32)
    for wtype in (8, 12):
        blocks = O.pack_q8_0(w) if wtype == 8 else O.pack_q4_k(w)
        rb, w_loc = _row_bytes(wtype, K), N // world
        mine = blocks[rank * w_loc * rb:(rank + 1) * w_loc * rb]
        y_loc = O.qgemm(wtype, mine, x, w_loc, order="kernel")
        parts = [torch.empty((M, w_loc), dtype=torch.float32) for _ in range(world)]
        dist.all_gather(parts, torch.from_numpy(y_loc))
        g = torch.stack(parts).numpy()                      # [G][M][w]: the all-gather layout
        k = np.arange(N)
        y = g[k // w_loc, :, k % w_loc].T                   # column k of row m at block k // w
        if rank == 0:
            np.save(os.path.join(out_dir, f"y{wtype}.npy"), y)
    dist.barrier()
    dist.destroy_process_group()


def test_column_split_matches_full_gemm():
    import multiprocessing as mp
    from oracle import oracle as O
    d = tempfile.mkdtemp()
    ctx = mp.get_context("spawn")
    port = _port()
    ps = [ctx.Process(target=_worker, args=(r, 2, port, d)) for r in range(2)]
    for p in ps:
        p.start()
    for p in ps:
        p.join(300)
    assert [p.exitcode for p in ps] == [0, 0]
    rng = np.random.default_rng(21)
    M, K, N = 37, 512, 384
    x = rng.standard_normal((M, K), dtype=np.float32)
    w = (rng.standard_normal((N, K), dtype=np.float32) * 0.02).astype(np.float32)
    for wtype in (8, 12):
        blocks = O.pack_q8_0(w) if wtype == 8 else O.pack_q4_k(w)
        full = O.qgemm(wtype, blocks, x, N, order="kernel")
        assert np.array_equal(np.load(os.path.join(d, f"y{wtype}.npy")), full)


def test_activation_tile_slices_are_contiguous():
    """kernels.h: tile (kc, mt) of the quantized activation starts at ((kc*Mpad/128)+mt)*20480, so
    the chunks kc in [r*F/G/128, (r+1)*F/G/128) of every m-tile form one byte run per rank."""
    tile = 20480
    for F, G, Mpad in ((3072, 2, 16512), (3072, 4, 16512), (3072, 8, 16512), (3072, 2, 384)):
        Fg, mts = F // G, Mpad // 128
        assert Fg % 128 == 0
        for r in range(G):
            offs = sorted(((kc * mts) + mt) * tile for kc in range(r * Fg // 128, (r + 1) * Fg // 128)
                          for mt in range(mts))
            assert offs[0] == r * (Fg // 128) * mts * tile
            assert all(b - a == tile for a, b in zip(offs, offs[1:]))
