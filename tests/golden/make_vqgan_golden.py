"""Generate tests/golden/vqgan_golden.npz from the reference's own VQGAN decoder.

Runs build_vqgan_decoder + mg-cpu (src/mg-vqgan.cpp, src/mg-cpu/mg-cpu.cpp, through
oracle/_ref/libmgref.so) on two synthetic decoders with seeded token grids:
  small : filters 32, 4 x 4 latent (64 x 64 image), embedding 32 -- the whole image is stored;
  full  : the MaskGIT decoder (filters 128, multipliers 1,1,2,2,4, 16 x 16 latent, 256 x 256
          image) -- 4096 seeded pixel samples and per-channel sums are stored (the reference's
          scalar path takes a few minutes on it).
The synthetic weights are re-created from their seeds by edge_maskgit_b200.synth.
Usage: python tests/golden/make_vqgan_golden.py   (needs oracle/_ref/libmgref.so)
"""
import sys
import tempfile
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

from edge_maskgit_b200 import synth  # noqa: E402
from oracle import oracle  # noqa: E402

SMALL = dict(vq=synth.VqganSpec(filters=32, embedding_dim=32), n_tokens=16)
FULL = dict(vq=synth.VqganSpec(), n_tokens=256)
N_SAMPLES = 4096


def grid_for(spec, seed=7):
    return np.random.default_rng(seed).integers(0, spec.codebook, spec.n_tokens).astype(np.int32)


def sample_index(R, seed=11):
    return np.random.default_rng(seed).integers(0, R * R * 3, N_SAMPLES)


def main():
    out = {}
    with tempfile.TemporaryDirectory() as d:
        for tag, kw in (("small", SMALL), ("full", FULL)):
            spec = synth.vqgan_spec(**kw)
            path = synth.make_model(Path(d) / f"{tag}.gguf", spec)
            grid = grid_for(spec)
            img = oracle.ref_vqgan(path, grid, spec.resolution)
            out[f"{tag}_grid"] = grid
            if tag == "small":
                out["small_image"] = img
            else:
                idx = sample_index(spec.resolution)
                out["full_index"] = idx
                out["full_samples"] = img.ravel()[idx]
                out["full_channel_sum"] = img.astype(np.float64).reshape(-1, 3).sum(0)
                out["full_sq_sum"] = np.array([(img.astype(np.float64) ** 2).sum()])
            print(tag, img.shape, float(np.abs(img).max()))
    np.savez_compressed(Path(__file__).with_name("vqgan_golden.npz"), **out)


if __name__ == "__main__":
    main()
