"""CPU: the oracle and the library's host-side packers against the reference's own outputs."""
import numpy as np
import pytest

from conftest import SMALL, TIERS, cosine


@pytest.mark.parametrize("i", [0, 1, 2])
def test_oracle_packers_match_reference_converter(oracle_mod, golden, i):
    w = golden[f"w{i}"]
    assert np.array_equal(oracle_mod.pack_q8_0(w), golden[f"q8_{i}"])
    assert np.array_equal(oracle_mod.pack_q4_k(w), golden[f"q4_{i}"])


@pytest.mark.parametrize("i", [0, 1, 2])
def test_library_packers_match_reference_converter(golden, i):
    from edge_maskgit_b200 import runtime as rt
    w = golden[f"w{i}"]
    assert np.array_equal(rt.pack_q8_0(w), golden[f"q8_{i}"])
    assert np.array_equal(rt.pack_q4_k(w), golden[f"q4_{i}"])


@pytest.mark.parametrize("wtype,key", [(8, "q8"), (12, "q4")])
def test_dequant_library_equals_oracle(oracle_mod, golden, wtype, key):
    from edge_maskgit_b200 import runtime as rt
    for i in range(3):
        w = golden[f"w{i}"]
        N, K = w.shape
        a = rt.dequant(wtype, golden[f"{key}_{i}"], N, K)
        b = oracle_mod.dequant(wtype, golden[f"{key}_{i}"], N, K)
        assert np.array_equal(a, b)
        # dequantised weights approximate the originals (round-trip encode -> decode)
        if i < 2:
            assert cosine(a, w) > (0.9999 if wtype == 8 else 0.99)


def test_quantizer_semantics(oracle_mod):
    # k_quantize_q8: half away from zero, d = amax/127, all-zero block -> d = 0, q = 0
    x = np.zeros((2, 64), np.float32)
    x[0, :32] = np.linspace(-1, 1, 32)
    x[0, 3] = 1.27          # amax -> d = 0.01
    x[0, 4] = 0.005         # 0.5 exactly representable? -> half-away rounding of x*id
    qx, dx, sx = oracle_mod.quantize_act(x)
    assert dx[1, 0] == 0 and (qx[1] == 0).all()
    assert dx[0, 0] == np.float32(1.27) / np.float32(127.0)
    idv = np.float32(1.0) / dx[0, 0]
    ref = np.trunc(x[0, :32] * idv + np.copysign(np.float32(0.5), x[0, :32] * idv)).astype(np.int32)
    assert np.array_equal(qx[0, :32].astype(np.int32), ref)
    assert sx[0, 0] == qx[0, :32].astype(np.int32).sum()


@pytest.mark.parametrize("q,tier", [("gq8", "q8"), ("gq4", "q4")])
def test_oracle_forward_matches_reference_cpu(oracle_mod, golden, small_models, q, tier):
    """Oracle int8-dot forward vs the reference's own F32 executor on the dequantised twin:
    the 51-tensor gate of verification/compare_intermediates.py at the quant tier."""
    from edge_maskgit_b200 import synth
    path, spec = small_models[q]
    m = oracle_mod.OracleModel(path)
    _, named = m.forward(synth.config1_tokens(spec), dump=True)
    max_tol, cos_tol = TIERS[tier]
    for name in oracle_mod.named_tensor_names(spec.n_layer):
        ref = golden[f"ref_{q}_{name}"]
        assert np.abs(named[name] - ref).max() <= max_tol, name
        assert cosine(named[name], ref) >= cos_tol, name
    # the logit gate of tools/verify-opencl-transformer.cpp:98-101
    ref = golden[f"ref_{q}_output_logits"]
    assert np.abs(named["output_logits"] - ref).max() < 1.0
    assert cosine(named["output_logits"], ref) > 0.9999


def test_oracle_generate_matches_reference_generate(oracle_mod, golden, small_models):
    path, spec = small_models["gq8"]
    m = oracle_mod.OracleModel(path)
    toks = m.generate([207], [42], steps=8)
    assert toks[0, 0] == 207 + spec.codebook
    assert np.array_equal(toks[0, 1:], golden["ref_grid_gq8"])


def test_oracle_generate_batch_is_per_image(oracle_mod, small_models):
    path, _ = small_models["gq8"]
    m = oracle_mod.OracleModel(path)
    a = m.generate([207, 5, 999], [42, 7, 9], steps=4)
    for i, (c, s) in enumerate([(207, 42), (5, 7), (999, 9)]):
        assert np.array_equal(a[i], m.generate([c], [s], steps=4)[0])
