"""GPU: mgc_qgemm_noalloc, the quantized linear layer for callers that must not allocate
device memory (a host whose own pool allocator owns the GPU's memory, or code that may not
allocate once it is running).  It is called through the C ABI and must give the same
output as mgc_qgemm -- within the tolerance the other qGEMM tests use -- on two calls in
a row, the second reusing the fixed scratch array the first one left behind.

This file is collected last on purpose, so a run that stops at the first failure has
already run every other test."""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


def _case(rt, wtype, M, K, N, seed):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((M, K), dtype=np.float32)
    w = (rng.standard_normal((N, K), dtype=np.float32) * 0.02).astype(np.float32)
    b = rng.standard_normal(N, dtype=np.float32)
    r = rng.standard_normal((M, N), dtype=np.float32)
    blocks = rt.pack_q8_0(w) if wtype == 8 else rt.pack_q4_k(w)
    return rt.QWeight(wtype, blocks, N, K), *(torch.from_numpy(a).cuda() for a in (x, b, r))


def _noalloc(lib, qw, x, bias, act, resid):
    y = torch.empty((x.shape[0], qw.N), dtype=torch.float32, device=x.device)
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    rc = lib.mgc_qgemm_noalloc(qw._h, C.c_void_p(x.data_ptr()), x.shape[0], C.c_void_p(bias.data_ptr()), act,
                               C.c_void_p(resid.data_ptr()), C.c_void_p(y.data_ptr()), stream)
    return rc, y


def test_noalloc_matches_qgemm_two_calls_in_a_row():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from edge_maskgit_b200 import runtime as rt
    from edge_maskgit_b200._lib import lib
    cases = [(8, 257, 3072, 768, 0, 1), (12, 31, 768, 2304, 1, 2)]   # (wtype, M, K, N, act, seed)
    for wtype, M, K, N, act, seed in cases:
        qw, x, b, r = _case(rt, wtype, M, K, N, seed)
        rc, y = _noalloc(lib, qw, x, b, act, r)
        assert rc == 0, lib.mgc_last_error().decode()
        ref = qw.qgemm(x, bias=b, act=act, resid=r)
        torch.cuda.synchronize()
        # mgc_qgemm may split K over CTAs (partials summed in split order); the fixed-scratch
        # variant never does -- so equal to a few ulp of the output scale, the qGEMM tolerance
        yn, rn = y.cpu().numpy(), ref.cpu().numpy()
        np.testing.assert_allclose(yn, rn, rtol=1e-5, atol=1e-5 * float(np.abs(rn).max()))
    assert rt.device_error() == 0


def test_noalloc_rejects_sizes_beyond_the_fixed_scratch():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from edge_maskgit_b200 import runtime as rt
    from edge_maskgit_b200._lib import lib
    qw, x, b, r = _case(rt, 8, 4, 3072, 128, 3)
    big = torch.zeros((2049, 3072), dtype=torch.float32, device="cuda")   # 2176 * 3072 > 6 Mi
    rc, _ = _noalloc(lib, qw, big, b, 0, torch.zeros((2049, 128), device="cuda"))
    assert rc != 0
    assert "MGC_NOALLOC_MAX_ELEMS" in lib.mgc_last_error().decode()
