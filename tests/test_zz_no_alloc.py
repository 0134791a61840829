"""qne_gemm_noalloc (the batched GEMM with its buffers in a static device array) against qne_gemm
and against a float64 restatement of the GEMM and its epilogue, called through the C ABI twice in a
row; and its size limit. Kept in its own file, collected last, and self-contained so that it also
passes alone in a fresh process."""
import ctypes as C

import numpy as np
import pytest
import torch

import qne

pytestmark = pytest.mark.gpu
REL_TOL = 1e-6  # both entry points launch the same kernels; a relative error bound, not bitwise
# against float64: x enters the tensor cores as f16 hi + lo planes (x to ~2^-22 relative) and the
# sums accumulate in f32, so the result is within the batched paths' logit tolerance
F64_REL_TOL = 1e-4


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


def gemm_f64(w16, x, y0, epilogue):
    """y (=, +=, SwiGLU) W x in float64 (kernels/src/shaders.rs:36-43 epilogues)."""
    acc = x.astype(np.float64) @ w16.astype(np.float64).T
    if epilogue == "store":
        return acc
    if epilogue == "accumulate":
        return y0.astype(np.float64) + acc
    half = acc.shape[1] // 2
    g, u = acc[:, :half], acc[:, half:]
    return g / (1.0 + np.exp(-g)) * u


def check_against_both(m, w16, x_np, y0, batch, epilogue, got):
    want = dev(y0)
    qne.gemm(m, dev(x_np), batch, want, epilogue)
    torch.cuda.synchronize()
    g_np, w_np = got.cpu().numpy(), want.cpu().numpy()
    assert np.all(np.isfinite(g_np))
    assert rel_err(g_np, w_np) <= REL_TOL, rel_err(g_np, w_np)
    exact = gemm_f64(w16, x_np, y0, epilogue)
    assert rel_err(g_np, exact) <= F64_REL_TOL, rel_err(g_np, exact)


@pytest.mark.parametrize("epilogue,rows,k,batch", [("store", 1024, 1024, 5), ("accumulate", 1024, 3584, 8),
                                                   ("swiglu", 2 * 3584, 1024, 3), ("swiglu", 2 * 6144, 2048, 32),
                                                   ("store", 2048, 2048, 64)])
def test_noalloc_gemm_matches_gemm_and_float64_twice_in_a_row(cuda, epilogue, rows, k, batch):
    rng = np.random.default_rng(rows + k + batch)
    w16 = (rng.standard_normal(rows * k) * 0.05).astype(np.float16)
    m = qne.matrix("f16", rows, k, dev(w16))
    w16 = w16.reshape(rows, k)
    out_rows = rows // 2 if epilogue == "swiglu" else rows
    y0 = rng.standard_normal((batch, out_rows)).astype(np.float32)
    for call in range(2):
        x_np = rng.standard_normal((batch, k)).astype(np.float32)
        got = dev(y0)
        noalloc(m, dev(x_np), batch, got, epilogue)
        check_against_both(m, w16, x_np, y0, batch, epilogue, got)


def test_noalloc_gemm_after_a_larger_call_ignores_stale_scratch(cuda):
    """A 64-row SwiGLU call fills the static array (activation planes and the gate/up intermediate);
    the smaller calls that follow find its rows past their own batch still holding that data."""
    rng = np.random.default_rng(7)
    rows, k = 2 * 3584, 1024
    w16 = (rng.standard_normal(rows * k) * 0.05).astype(np.float16)
    m = qne.matrix("f16", rows, k, dev(w16))
    w16 = w16.reshape(rows, k)
    for batch, epilogue in ((64, "swiglu"), (5, "swiglu"), (3, "accumulate"), (1, "store")):
        out_rows = rows // 2 if epilogue == "swiglu" else rows
        mk = m if epilogue == "swiglu" else qne.matrix("f16", out_rows, k, dev(w16[:out_rows]))
        wk = w16 if epilogue == "swiglu" else w16[:out_rows]
        # the first call's inputs are 4x larger, so every byte it leaves behind differs from what
        # the later calls would write (the SwiGLU intermediate stays within the f16 planes' range)
        x_np = (rng.standard_normal((batch, k)) * (4.0 if batch == 64 else 1.0)).astype(np.float32)
        y0 = rng.standard_normal((batch, out_rows)).astype(np.float32)
        got = dev(y0)
        noalloc(mk, dev(x_np), batch, got, epilogue)
        check_against_both(mk, wk, x_np, y0, batch, epilogue, got)


def test_noalloc_gemm_rejects_calls_beyond_its_limits(cuda):
    w = dev(np.zeros(16, np.float16))  # never read: the calls are rejected before any launch
    m = qne.matrix("f16", 2 * 10000, 8192, w)
    x = dev(np.zeros((32, 16), np.float32))
    y = dev(np.zeros((32, 16), np.float32))
    with pytest.raises(qne.QneError) as e:
        noalloc(m, x, 32, y, "swiglu")
    assert e.value.name == "EINVAL" and "static array holds 2097152" in str(e.value)
    with pytest.raises(qne.QneError) as e:
        noalloc(qne.matrix("f16", 64, 64, w), x, 65, y, "store")
    assert e.value.name == "EINVAL" and "1..64" in str(e.value)
