"""CPU: the VQGAN decoder oracle (oracle.vqgan_decode, a numpy restatement of
src/mg-vqgan.cpp:67-108 over the mg-cpu kernels) pinned against the reference's own decoder --
the golden fixture tests/golden/vqgan_golden.npz (made by make_vqgan_golden.py from
oracle/_ref/libmgref.so) and, where libmgref.so is built, the reference run live -- plus the
synthetic GGUF's VQGAN metadata.  Gate: tools/verify-vqgan.cpp:69 (max_abs < 1e-2, cosine >
0.99999), and a tighter max_abs for the f32-vs-f32 oracle."""
from pathlib import Path

import numpy as np
import pytest

from conftest import cosine

GOLD = Path(__file__).resolve().parent / "golden" / "vqgan_golden.npz"


def _gold():
    if not GOLD.exists():
        pytest.skip("tests/golden/vqgan_golden.npz is missing")
    return np.load(GOLD)


def _model(tmp_path, tag):
    import importlib.util
    from edge_maskgit_b200 import synth
    spec_path = Path(__file__).resolve().parent / "golden" / "make_vqgan_golden.py"
    s = importlib.util.spec_from_file_location("mkvq", spec_path)
    mk = importlib.util.module_from_spec(s)
    s.loader.exec_module(mk)
    spec = synth.vqgan_spec(**(mk.SMALL if tag == "small" else mk.FULL))
    return synth.make_model(tmp_path / f"{tag}.gguf", spec), spec, mk


def test_vqgan_metadata_roundtrip(tmp_path, oracle_mod):
    path, spec, _ = _model(tmp_path, "small")
    kv, t = oracle_mod.read_gguf(path)
    assert kv["maskgit.vqgan.channel_multipliers"] == [1, 1, 2, 2, 4]
    assert kv["maskgit.vqgan.filters"] == 32 and kv["maskgit.vqgan.embedding_dim"] == 32
    assert kv["maskgit.resolution"] == spec.resolution == 64
    assert t["vqgan.decoder.conv_in.weight"].shape == (128, 32, 3, 3)
    assert t["vqgan.decoder.res_blocks.2.0.conv_res.weight"].shape == (64, 64, 1, 1)


def test_vqgan_oracle_vs_reference_golden_small(tmp_path, oracle_mod):
    g = _gold()
    path, spec, _ = _model(tmp_path, "small")
    img = oracle_mod.vqgan_decode(path, g["small_grid"])
    ref = g["small_image"]
    assert img.shape == ref.shape == (64, 64, 3)
    assert np.abs(img - ref).max() < 1e-3 and cosine(img, ref) > 0.99999


def test_vqgan_oracle_vs_reference_golden_full(tmp_path, oracle_mod):
    g = _gold()
    path, spec, _ = _model(tmp_path, "full")
    img = oracle_mod.vqgan_decode(path, g["full_grid"])
    assert img.shape == (256, 256, 3)
    s = img.ravel()[g["full_index"]]
    assert np.abs(s - g["full_samples"]).max() < 1e-3 and cosine(s, g["full_samples"]) > 0.99999
    np.testing.assert_allclose(img.astype(np.float64).reshape(-1, 3).sum(0), g["full_channel_sum"], rtol=1e-4)


def test_vqgan_oracle_vs_reference_live(tmp_path, oracle_mod):
    if not oracle_mod.ref_available():
        pytest.skip("oracle/_ref/libmgref.so is not built")
    from edge_maskgit_b200 import synth
    # ragged: a 3 x 3 latent with 2 multipliers (6 x 6 image), filters 32
    spec = synth.vqgan_spec(synth.VqganSpec(filters=32, embedding_dim=16, channel_multipliers=(1, 2)),
                            n_tokens=9)
    path = synth.make_model(tmp_path / "r.gguf", spec)
    grid = np.random.default_rng(3).integers(0, spec.codebook, 9).astype(np.int32)
    img = oracle_mod.vqgan_decode(path, grid)
    ref = oracle_mod.ref_vqgan(path, grid, spec.resolution)
    assert img.shape == ref.shape == (6, 6, 3)
    assert np.abs(img - ref).max() < 1e-4 and cosine(img, ref) > 0.99999
