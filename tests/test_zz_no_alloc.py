"""qne_gemm_noalloc (the batched GEMM with its buffers in a static device array) against qne_gemm on
the same inputs, called through the C ABI twice in a row; and its size limit. Kept in its own file,
collected last, and self-contained so that it also passes alone in a fresh process."""
import ctypes as C

import numpy as np
import pytest
import torch

import qne

pytestmark = pytest.mark.gpu
REL_TOL = 1e-6  # both entry points launch the same kernels; a relative error bound, not bitwise


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def noalloc(m, x, batch, y, epilogue):
    st = qne.lib.qne_gemm_noalloc(C.byref(m), C.c_void_p(x.data_ptr()), batch, C.c_void_p(y.data_ptr()),
                                  qne.EPILOGUES[epilogue], None)
    if st != 0:
        raise qne.QneError(st, qne.lib.qne_last_error().decode())


def rel_err(a, b):
    a = a.astype(np.float64)
    b = b.astype(np.float64)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


@pytest.mark.parametrize("epilogue,rows,k,batch", [("store", 1024, 1024, 5), ("accumulate", 1024, 3584, 8),
                                                   ("swiglu", 2 * 3584, 1024, 3), ("swiglu", 2 * 6144, 6144, 32)])
def test_noalloc_gemm_matches_gemm_twice_in_a_row(cuda, epilogue, rows, k, batch):
    rng = np.random.default_rng(rows + k + batch)
    w = dev((rng.standard_normal(rows * k) * 0.05).astype(np.float16))
    m = qne.matrix("f16", rows, k, w)
    out_rows = rows // 2 if epilogue == "swiglu" else rows
    y0 = rng.standard_normal((batch, out_rows)).astype(np.float32)
    want = dev(y0)
    got = [dev(y0), dev(y0)]
    for call in range(2):
        x = dev(rng.standard_normal((batch, k)).astype(np.float32))
        want.copy_(dev(y0))
        qne.gemm(m, x, batch, want, epilogue)
        noalloc(m, x, batch, got[call], epilogue)
        torch.cuda.synchronize()
        w_np, g_np = want.cpu().numpy(), got[call].cpu().numpy()
        assert np.all(np.isfinite(g_np))
        assert rel_err(g_np, w_np) <= REL_TOL, (call, rel_err(g_np, w_np))


def test_noalloc_gemm_rejects_calls_beyond_its_scratch(cuda):
    w = dev(np.zeros(16, np.float16))  # never read: the call is rejected before any launch
    m = qne.matrix("f16", 2 * 10000, 8192, w)
    x = dev(np.zeros((32, 16), np.float32))
    y = dev(np.zeros((32, 16), np.float32))
    with pytest.raises(qne.QneError) as e:
        noalloc(m, x, 32, y, "swiglu")
    assert e.value.name == "EINVAL" and "static array holds 2097152" in str(e.value)
