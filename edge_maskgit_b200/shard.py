"""Batch sharding of independent images over ranks (one process per GPU).

The decode loop of src/mg-generate.cpp runs per image with its own RNG, so images are
independent: rank r of W decodes a contiguous slice of the image list and the final token
grids are gathered once at the end (all_gather over the process group -- NCCL on GPUs, gloo
in the CPU tests).  There is no other collective on this path.
"""
from __future__ import annotations

import numpy as np


def batch_classes(n_images: int = 64, seed: int = 7) -> np.ndarray:
    """Classes of the batched-decode workload: default_rng(seed).integers(0, 1000, n)."""
    return np.random.default_rng(seed).integers(0, 1000, n_images).astype(np.int32)


def batch_seeds(n_images: int = 64, base: int = 7) -> np.ndarray:
    """Sampling seed of image i: base + i (each image owns an mt19937_64 stream)."""
    return (base + np.arange(n_images)).astype(np.uint64)


def shard_range(n: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous slice [lo, hi) of n items for `rank`; sizes differ by at most one."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} / world {world}")
    base, extra = divmod(n, world)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


def gather_tokens(local: np.ndarray, n_total: int, S: int, group=None) -> np.ndarray:
    """All-gather each rank's [n_local][S] int32 token grids into [n_total][S] (rank order)."""
    import torch
    import torch.distributed as dist

    world = dist.get_world_size(group)
    backend = dist.get_backend(group)
    dev = torch.device("cuda", torch.cuda.current_device()) if backend == "nccl" else torch.device("cpu")
    # pad every shard to the largest shard size so the collective has one shape
    sizes = [shard_range(n_total, r, world) for r in range(world)]
    cap = max(hi - lo for lo, hi in sizes)
    buf = torch.zeros((cap, S), dtype=torch.int32, device=dev)
    if local.shape[0]:
        buf[: local.shape[0]] = torch.from_numpy(np.ascontiguousarray(local, np.int32)).to(dev)
    outs = [torch.empty_like(buf) for _ in range(world)]
    dist.all_gather(outs, buf, group=group)
    return np.concatenate([o[: hi - lo].cpu().numpy() for o, (lo, hi) in zip(outs, sizes)], axis=0)


def decode_shard(generate, classes: np.ndarray, seeds: np.ndarray, rank: int, world: int,
                 steps: int = 8, temperature: float = 4.5) -> np.ndarray:
    """Run generate(class_ids, seeds, steps, temperature) -> [b][S] on this rank's slice."""
    lo, hi = shard_range(len(classes), rank, world)
    if hi == lo:
        return np.zeros((0, 0), np.int32)
    return generate(classes[lo:hi], seeds[lo:hi], steps, temperature)
