"""GPU: the CUDA VQGAN decoder (mgc_vqgan_*, csrc/vqgan.cu) against the reference's own decoder
(build_vqgan_decoder on mg-cpu, src/mg-vqgan.cpp:67-108) under tools/verify-vqgan.cpp:69's gate
(max_abs < 1e-2, cosine > 0.99999):
  - small decoder (64 x 64 image): the whole image vs the golden fixture and vs the reference
    run live on the box's CPU;
  - the MaskGIT decoder (256 x 256): 4096 golden samples + per-channel sums of the reference's
    image, and the whole image vs the numpy oracle;
  - ragged shapes (3 x 3 latent, 64 output channels), batches, the device entry point,
    determinism and the error paths.
"""
from pathlib import Path

import numpy as np
import pytest

from conftest import cosine

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

GOLD = Path(__file__).resolve().parent / "golden" / "vqgan_golden.npz"
GATE = (1e-2, 0.99999)


def _mk():
    import importlib.util
    p = Path(__file__).resolve().parent / "golden" / "make_vqgan_golden.py"
    s = importlib.util.spec_from_file_location("mkvq", p)
    m = importlib.util.module_from_spec(s)
    s.loader.exec_module(m)
    return m


def _gate(img, ref):
    d, c = float(np.abs(img - ref).max()), cosine(img, ref)
    assert d < GATE[0] and c > GATE[1], (d, c)
    return d, c


@pytest.fixture(scope="module")
def vq_models(tmp_path_factory):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from edge_maskgit_b200 import synth
    mk = _mk()
    d = tmp_path_factory.mktemp("vq")
    out = {}
    for tag, kw in (("small", mk.SMALL), ("full", mk.FULL)):
        spec = synth.vqgan_spec(**kw)
        out[tag] = (synth.make_model(d / f"{tag}.gguf", spec), spec)
    return out, mk


def test_vqgan_small_vs_reference(vq_models, oracle_mod):
    from edge_maskgit_b200 import runtime as rt
    models, mk = vq_models
    path, spec = models["small"]
    g = np.load(GOLD)
    dec = rt.VqganDecoder(path)
    assert (dec.n_tokens, dec.resolution, dec.codebook_size) == (16, 64, 1024)
    img = dec.decode(g["small_grid"])
    _gate(img, g["small_image"])
    assert np.abs(img - g["small_image"]).max() < 1e-3
    if oracle_mod.ref_available():
        grid = np.random.default_rng(99).integers(0, 1024, 16).astype(np.int32)
        _gate(dec.decode(grid), oracle_mod.ref_vqgan(path, grid, 64))
    dec.close()


def test_vqgan_full_vs_reference_golden_and_oracle(vq_models, oracle_mod):
    from edge_maskgit_b200 import runtime as rt
    models, mk = vq_models
    path, spec = models["full"]
    g = np.load(GOLD)
    dec = rt.VqganDecoder(path)
    assert dec.resolution == 256
    img = dec.decode(g["full_grid"])
    assert img.shape == (256, 256, 3) and np.isfinite(img).all()
    _gate(img.ravel()[g["full_index"]], g["full_samples"])
    np.testing.assert_allclose(img.astype(np.float64).reshape(-1, 3).sum(0), g["full_channel_sum"], rtol=1e-4)
    _gate(img, oracle_mod.vqgan_decode(path, g["full_grid"]))
    # deterministic: the same grid decodes to the same bits
    assert np.array_equal(img, dec.decode(g["full_grid"]))
    dec.close()


def test_vqgan_batch_and_device_entry(vq_models):
    from edge_maskgit_b200 import runtime as rt
    models, _ = vq_models
    path, spec = models["full"]
    rng = np.random.default_rng(5)
    grids = rng.integers(0, 1024, (3, 256)).astype(np.int32)
    dec = rt.VqganDecoder(path, max_images=3)
    batch = dec.decode(grids)
    for i in range(3):
        one = dec.decode(grids[i])
        # the split-K choice depends on the batch: f32 reassociation, carried through the
        # layers by the bf16 hi/lo split, stays two orders under the reference gate
        assert np.abs(batch[i] - one).max() < 1e-3 and cosine(batch[i], one) > 0.999999
    gd = torch.from_numpy(grids).cuda()
    od = torch.empty((3, 256, 256, 3), dtype=torch.float32, device="cuda")
    dec.decode_device(gd, od, 3)
    torch.cuda.synchronize()
    assert np.array_equal(od.cpu().numpy(), batch)
    assert dec.launches() > 0
    dec.close()


def test_vqgan_ragged_vs_reference(tmp_path, oracle_mod):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from edge_maskgit_b200 import runtime as rt, synth
    spec = synth.vqgan_spec(synth.VqganSpec(filters=32, embedding_dim=16, channel_multipliers=(1, 2)), n_tokens=9)
    path = synth.make_model(tmp_path / "r.gguf", spec)
    grid = np.random.default_rng(3).integers(0, spec.codebook, 9).astype(np.int32)
    dec = rt.VqganDecoder(path)
    img = dec.decode(grid)
    ref = oracle_mod.ref_vqgan(path, grid, 6) if oracle_mod.ref_available() else oracle_mod.vqgan_decode(path, grid)
    assert img.shape == (6, 6, 3)
    _gate(img, ref)
    dec.close()


def test_vqgan_errors(vq_models):
    from edge_maskgit_b200 import runtime as rt
    models, _ = vq_models
    path, spec = models["small"]
    dec = rt.VqganDecoder(path)
    bad = np.zeros(16, np.int32)
    bad[3] = 1024
    with pytest.raises(rt.MgcError, match="out of range"):
        dec.decode(bad)
    with pytest.raises(rt.MgcError, match="n_images"):
        dec.decode(np.zeros((2, 16), np.int32))
    dec.close()
    # a transformer-only GGUF has no decoder
    tf = synth_tf(path.parent)
    with pytest.raises(rt.MgcError, match="VQGAN"):
        rt.VqganDecoder(tf)


def synth_tf(d):
    from edge_maskgit_b200 import synth
    return synth.make_model(d / "tf.gguf", synth.ModelSpec(n_layer=1, n_embd=64, n_head=2, n_ffn=128, quant="f32"))


def test_reference_generate_drives_cuda_vqgan(tmp_path, oracle_mod):
    """The reference's generate() (src/mg-generate.cpp:137-147) with both callbacks from
    include/mgc.hpp -- mgc::Runtime::transformer_fwd and mgc::Vqgan::vqgan_fwd -- produces the
    CUDA decode loop's grid and the CUDA decoder's image of that grid."""
    import subprocess
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    exe = Path(oracle_mod.__file__).parent / "_ref" / "mg_generate_cuda"
    if not exe.exists():
        pytest.skip("oracle/_ref/mg_generate_cuda is not built")
    from edge_maskgit_b200 import runtime as rt, synth
    spec = synth.ModelSpec(n_layer=2, n_tokens=16, quant="gq8",
                           vqgan=synth.VqganSpec(filters=32, embedding_dim=32))
    path = synth.make_model(tmp_path / "m.gguf", spec)
    p = subprocess.run([str(exe), str(path), "207", "42", "8", str(tmp_path / "g.bin"), str(tmp_path / "i.bin"),
                        str(tmp_path / "rgb.bin")], capture_output=True, text=True, timeout=600)
    assert p.returncode == 0, p.stderr
    grid = np.fromfile(tmp_path / "g.bin", np.int32)
    image = np.fromfile(tmp_path / "i.bin", np.float32).reshape(64, 64, 3)
    rgb_ref_loop = np.fromfile(tmp_path / "rgb.bin", np.uint8).reshape(64, 64, 3)
    r = rt.CudaRuntime(path, max_rows=17 * 2)
    toks = r.generate([207], [42], steps=8, temperature=4.5)
    assert np.array_equal(grid, toks[0, 1:])
    dec = rt.VqganDecoder(path, max_images=1)
    assert np.array_equal(image, dec.decode(grid))
    # mg::generate end to end in the library: the same tokens and the same bytes as the
    # reference's generate() (its own float -> byte conversion) driving the CUDA callbacks;
    # two images in batches of one exercise the chunked decode
    rgb, tok2 = r.generate_images(dec, [207, 207], [42, 42], steps=8, temperature=4.5)
    assert np.array_equal(tok2[0, 1:], grid) and np.array_equal(tok2[1], tok2[0])
    assert np.array_equal(rgb[0], rgb_ref_loop) and np.array_equal(rgb[1], rgb_ref_loop)
    assert np.array_equal(dec.decode_rgb8(grid), rgb_ref_loop)
    dec.close()
    r.close()
    if oracle_mod.ref_available():
        ref_img = oracle_mod.ref_vqgan(path, grid, 64)
        _gate(image, ref_img)
        # bytes from the reference's CPU decoder: equal but where a value sits on a rounding edge
        ref_rgb = (np.minimum(np.maximum(ref_img, np.float32(0)), np.float32(1)) * np.float32(255)
                   + np.float32(0.5)).astype(np.uint8)
        diff = np.abs(ref_rgb.astype(int) - rgb_ref_loop.astype(int))
        assert diff.max() <= 1 and (diff == 0).mean() > 0.99


def test_vqgan_tensor_core_and_simt_paths_agree(vq_models, monkeypatch):
    """The same decode with every conv on the SIMT f32 path (MGC_VQGAN_SIMT=1) and with the
    tcgen05 bf16x3 path: both within the reference gate of each other, and of the golden."""
    from edge_maskgit_b200 import runtime as rt
    models, _ = vq_models
    path, spec = models["full"]
    g = np.load(GOLD)
    tc = rt.VqganDecoder(path)
    img_tc = tc.decode(g["full_grid"])
    tc.close()
    monkeypatch.setenv("MGC_VQGAN_SIMT", "1")
    sm = rt.VqganDecoder(path)
    img_sm = sm.decode(g["full_grid"])
    sm.close()
    d, c = _gate(img_tc, img_sm)
    assert d < 2e-3, d
    for img in (img_tc, img_sm):
        _gate(img.ravel()[g["full_index"]], g["full_samples"])
