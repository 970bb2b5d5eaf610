"""GPU: every kernel through the C ABI against the CPU oracle on the same inputs.

Integer outputs (qx, block dots via act=0 GEMM results) and every pure-IEEE path are
bit-exact; paths through erf / exp (GELU epilogue, attention softmax) use CUDA's erff /
expf against the C library's, so they are held to a few ulp (rtol 1e-5)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")


def _t(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def _x(M, K, seed=0):
    return np.random.default_rng(seed).standard_normal((M, K), dtype=np.float32)


@pytest.mark.parametrize("M,K", [(1, 32), (31, 768), (257, 768), (300, 3072)])
def test_quantize_act_bit_exact(dev, oracle_mod, M, K):
    from edge_maskgit_b200 import runtime as rt
    x = _x(M, K, 3)
    x[0, :32] = 0.0
    x[-1, 5] = 1e4
    qx, dx, sx = rt.quantize_act(_t(x, dev), want_sum=True)
    oq, od, os_ = oracle_mod.quantize_act(x)
    assert np.array_equal(qx.cpu().numpy(), oq)
    assert np.array_equal(dx.cpu().numpy(), od)
    assert np.array_equal(sx.cpu().numpy(), os_)


SHAPES = [(768, 2304), (768, 768), (768, 3072), (3072, 768), (768, 2025)]


def close_to_oracle(y, ref):
    """Split-K sums per-split partials in split order instead of one chain: a few ulp of the
    output scale."""
    np.testing.assert_allclose(y, ref, rtol=1e-5, atol=1e-5 * float(np.abs(ref).max()))


def close_to_reference_order(y, ref):
    """Q4_K: the kernel accumulates each block as two fused multiply-adds into acc; the
    reference (mg-opencl.cpp:572) forms scl*dx*idot - mnl*dx*sumx first and adds it once.
    Both are one-rounding-per-step f32 chains over K/32 blocks: a few ulp of the output scale."""
    np.testing.assert_allclose(y, ref, rtol=2e-5, atol=2e-5 * float(np.abs(ref).max()))


@pytest.mark.parametrize("wtype", [8, 12])
@pytest.mark.parametrize("M", [1, 31, 257, 1025])
@pytest.mark.parametrize("K,N", SHAPES)
@pytest.mark.parametrize("split", ["1", "auto"])
def test_qgemm_vs_oracle(dev, oracle_mod, monkeypatch, wtype, M, K, N, split):
    """split "1": one K chain per output, bit-exact against the oracle in the kernel's
    accumulation order (and within a few ulp of the reference's order); "auto": the
    library's split-K choice."""
    from edge_maskgit_b200 import runtime as rt
    if split == "1":
        monkeypatch.setenv("MGC_QGEMM_SPLITK", "1")
    else:
        monkeypatch.delenv("MGC_QGEMM_SPLITK", raising=False)
    rng = np.random.default_rng(0)
    x = rng.standard_normal((M, K), dtype=np.float32)
    w = (rng.standard_normal((N, K), dtype=np.float32) * 0.02).astype(np.float32)
    blocks = rt.pack_q8_0(w) if wtype == 8 else rt.pack_q4_k(w)
    qw = rt.QWeight(wtype, blocks, N, K)
    y = qw.qgemm(_t(x, dev)).cpu().numpy()
    ref = oracle_mod.qgemm(wtype, blocks, x, N, order="kernel")
    if split == "1":
        assert np.array_equal(y, ref), f"max diff {np.abs(y - ref).max()}"
        if wtype == 12:
            close_to_reference_order(y, oracle_mod.qgemm(wtype, blocks, x, N))
        else:
            assert np.array_equal(y, oracle_mod.qgemm(wtype, blocks, x, N))
    else:
        close_to_oracle(y, ref)


@pytest.mark.parametrize("wtype", [8, 12])
@pytest.mark.parametrize("act", [0, 1])
def test_qgemm_epilogue(dev, oracle_mod, monkeypatch, wtype, act):
    from edge_maskgit_b200 import runtime as rt
    rng = np.random.default_rng(5)
    M, K, N = 257, 768, 3072
    x = rng.standard_normal((M, K), dtype=np.float32)
    w = (rng.standard_normal((N, K), dtype=np.float32) * 0.02).astype(np.float32)
    b = rng.standard_normal(N, dtype=np.float32)
    r = rng.standard_normal((M, N), dtype=np.float32)
    blocks = rt.pack_q8_0(w) if wtype == 8 else rt.pack_q4_k(w)
    qw = rt.QWeight(wtype, blocks, N, K)
    monkeypatch.setenv("MGC_QGEMM_SPLITK", "1")
    y = qw.qgemm(_t(x, dev), bias=_t(b, dev), act=act, resid=_t(r, dev)).cpu().numpy()
    ref = oracle_mod.qgemm(wtype, blocks, x, N, bias=b, act=act, resid=r, order="kernel")
    if act == 0:
        assert np.array_equal(y, ref)
    else:
        np.testing.assert_allclose(y, ref, rtol=1e-5, atol=1e-6)
    monkeypatch.delenv("MGC_QGEMM_SPLITK")
    # split-K with the fused epilogue (768 -> 3072 at M=257 is split by default only for
    # smaller N; force it)
    monkeypatch.setenv("MGC_QGEMM_SPLITK", "3")
    y = qw.qgemm(_t(x, dev), bias=_t(b, dev), act=act, resid=_t(r, dev)).cpu().numpy()
    close_to_oracle(y, ref)
    # the arrival counters re-arm: a second split call gives the same result
    y2 = qw.qgemm(_t(x, dev), bias=_t(b, dev), act=act, resid=_t(r, dev)).cpu().numpy()
    assert np.array_equal(y, y2)


@pytest.mark.parametrize("wtype", [8, 12])
@pytest.mark.parametrize("K,N", SHAPES)
def test_qgemm_large_m(dev, oracle_mod, wtype, K, N):
    """M=4097 (config 2's largest sweep size; more tiles than SMs, so the CTAs walk several
    tiles each): every row, bit-exact against the oracle in the kernel's order."""
    from edge_maskgit_b200 import runtime as rt
    rng = np.random.default_rng(9)
    M = 4097
    x = rng.standard_normal((M, K), dtype=np.float32)
    w = (rng.standard_normal((N, K), dtype=np.float32) * 0.02).astype(np.float32)
    blocks = rt.pack_q8_0(w) if wtype == 8 else rt.pack_q4_k(w)
    y = rt.QWeight(wtype, blocks, N, K).qgemm(_t(x, dev)).cpu().numpy()
    ref = oracle_mod.qgemm(wtype, blocks, x, N, order="kernel")
    assert np.array_equal(y, ref), f"max diff {np.abs(y - ref).max()}"


@pytest.mark.parametrize("M,N,K", [(17, 2025, 768), (257, 2025, 768), (5, 70, 48)])
def test_gemm_f32_bit_exact(dev, oracle_mod, M, N, K):
    from edge_maskgit_b200 import runtime as rt
    rng = np.random.default_rng(1)
    w = rng.standard_normal((N, K), dtype=np.float32)
    x = rng.standard_normal((M, K), dtype=np.float32)
    b = rng.standard_normal(N, dtype=np.float32)
    y = rt.gemm_f32(_t(w, dev), _t(x, dev), bias=_t(b, dev)).cpu().numpy()
    assert np.array_equal(y, oracle_mod.gemm_f32(w, x, bias=b))


@pytest.mark.parametrize("rows,D", [(1, 768), (257, 768), (33, 64)])
def test_layernorm_bit_exact(dev, oracle_mod, rows, D):
    from edge_maskgit_b200 import runtime as rt
    rng = np.random.default_rng(2)
    x = rng.standard_normal((rows, D), dtype=np.float32) * 3 + 1
    g = rng.standard_normal(D, dtype=np.float32)
    b = rng.standard_normal(D, dtype=np.float32)
    y = rt.layernorm_affine(_t(x, dev), _t(g, dev), _t(b, dev), 1e-12).cpu().numpy()
    assert np.array_equal(y, oracle_mod.layernorm_affine(x, g, b, 1e-12))


@pytest.mark.parametrize("B,S", [(1, 257), (2, 17), (1, 1), (1, 33), (3, 257), (1, 1025), (2, 129)])
def test_flash_attn(dev, oracle_mod, B, S):
    from edge_maskgit_b200 import runtime as rt
    H, Dh = 16, 48
    rng = np.random.default_rng(4)
    qkv = rng.standard_normal((B * S, 3 * H * Dh), dtype=np.float32)
    scale = 1.0 / np.sqrt(np.float32(Dh))
    y = rt.flash_attn(_t(qkv, dev), B, S, H, Dh, float(scale)).cpu().numpy()
    ref = oracle_mod.flash_attn(qkv, B, S, H, Dh, float(scale))
    np.testing.assert_allclose(y, ref, rtol=2e-5, atol=2e-6)


def test_flash_attn_config5(dev, oracle_mod):
    """Config 5's attention: B=4 images of S=4097 tokens (33 key tiles, key ranges split over
    CTAs).  The kernel runs all 16 heads; the oracle checks two heads of two images (the
    heads are independent, so a head's columns alone are a complete input)."""
    from edge_maskgit_b200 import runtime as rt
    B, S, H, Dh = 4, 4097, 16, 48
    E = H * Dh
    rng = np.random.default_rng(11)
    qkv = rng.standard_normal((B * S, 3 * E), dtype=np.float32)
    scale = float(1.0 / np.sqrt(np.float32(Dh)))
    y = rt.flash_attn(_t(qkv, dev), B, S, H, Dh, scale).cpu().numpy().reshape(B, S, E)
    heads = [0, 13]
    cols = np.concatenate([np.arange(h * Dh, (h + 1) * Dh) for h in heads])
    for b in (0, 3):
        rows = qkv[b * S:(b + 1) * S]
        sub = np.concatenate([rows[:, cols], rows[:, E + cols], rows[:, 2 * E + cols]], axis=1)
        ref = oracle_mod.flash_attn(sub, 1, S, len(heads), Dh, scale)
        np.testing.assert_allclose(y[b][:, cols], ref, rtol=2e-5, atol=2e-6)


def test_embed_bit_exact(dev, oracle_mod):
    from edge_maskgit_b200 import runtime as rt
    rng = np.random.default_rng(6)
    V, E, B, S = 2025, 768, 2, 257
    tok = rng.standard_normal((V, E), dtype=np.float32)
    pos = rng.standard_normal((S, E), dtype=np.float32)
    ids = rng.integers(-1, V, (B, S)).astype(np.int32)   # -1 wraps to the last row (mask)
    y = rt.embed(_t(tok, dev), _t(pos, dev), _t(ids, dev), B, S).cpu().numpy()
    assert np.array_equal(y, oracle_mod.embed(tok, pos, ids, B, S))


def test_no_device_error_left(dev):
    from edge_maskgit_b200 import runtime as rt
    torch.cuda.synchronize()
    assert rt.device_error() == 0


def test_bounded_wait_times_out_and_context_survives(dev, oracle_mod):
    """A wait that nothing completes (an mbarrier nobody arrives on) gives up after its limit,
    leaves its code in the device error word and returns; later kernels run normally."""
    import ctypes as C
    from edge_maskgit_b200 import runtime as rt
    from edge_maskgit_b200._lib import lib
    torch.cuda.synchronize()
    assert rt.device_error() == 0
    assert lib.mgc_selftest_wait_timeout(77, C.c_void_p(torch.cuda.current_stream().cuda_stream)) == 0
    assert rt.device_error() == 77
    assert rt.device_error() == 0   # read and cleared
    x = np.random.default_rng(1).standard_normal((33, 256)).astype(np.float32)
    qx, dx, _ = rt.quantize_act(_t(x, dev))
    oq, od, _ = oracle_mod.quantize_act(x)
    assert np.array_equal(qx.cpu().numpy(), oq) and np.array_equal(dx.cpu().numpy(), od)


@pytest.mark.parametrize("wtype", [8, 12])
@pytest.mark.parametrize("act", [0, 1])
def test_qgemm_large_m_epilogue(dev, oracle_mod, wtype, act):
    """M=1025 (several waves of persistent tiles) with the full epilogue: bias -> act ->
    residual, bit-exact (act 0) against the oracle in the kernel's accumulation order."""
    from edge_maskgit_b200 import runtime as rt
    rng = np.random.default_rng(12)
    M, K, N = 1025, 768, 2304
    x = rng.standard_normal((M, K), dtype=np.float32)
    w = (rng.standard_normal((N, K), dtype=np.float32) * 0.02).astype(np.float32)
    b = rng.standard_normal(N, dtype=np.float32)
    r = rng.standard_normal((M, N), dtype=np.float32)
    blocks = rt.pack_q8_0(w) if wtype == 8 else rt.pack_q4_k(w)
    qw = rt.QWeight(wtype, blocks, N, K)
    y = qw.qgemm(_t(x, dev), bias=_t(b, dev), act=act, resid=_t(r, dev)).cpu().numpy()
    ref = oracle_mod.qgemm(wtype, blocks, x, N, bias=b, act=act, resid=r, order="kernel")
    if act == 0:
        assert np.array_equal(y, ref), f"max diff {np.abs(y - ref).max()}"
    else:
        np.testing.assert_allclose(y, ref, rtol=1e-5, atol=1e-6)
