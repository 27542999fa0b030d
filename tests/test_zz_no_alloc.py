"""mc_linear_run_static, the allocation-free projection, against mc_linear_run.

Both entry points run the same encoder and GEMV kernels; the static one keeps
its activation scratch in a fixed device array inside the library.  Each case
makes two static calls in a row on the same input, plus one mc_linear_run
call, and checks that all three agree.  Tolerance per output row:
|y_static - y_run| <= 1e-6 * ||w_row|| * ||x||, the same form the projection
tests use against the oracle but 100x tighter (the kernels are deterministic,
so the results are expected to be identical).  The file sorts last so that it
also runs after every other GPU test in one process.
"""

import numpy as np
import pytest

import modelc_b200 as mb
from modelc_b200 import _lib

pytestmark = pytest.mark.gpu

STATIC_MAX_K = 16384


def _linear(n, k, seed):
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal((n, k), dtype=np.float32) * np.float32(0.02)).astype(np.float32)
    q, s = mb.quantize_int8_rows(w)
    return mb.Linear(mb.QTensor("i8_row", q, s)), q.astype(np.float32) * s[:, None]


def _static(lin, x, y, stream):
    return _lib.lib().mc_linear_run_static(lin.handle, x.data_ptr(), x.shape[0], y.data_ptr(),
                                           stream)


@pytest.mark.parametrize("n,k,m", [(4096, 4096, 1), (4096, 4096, 5), (256, 14336, 16),
                                   (300, 517, 20), (1024, STATIC_MAX_K, 3)])
def test_static_matches_run_twice(n, k, m):
    import torch
    lin, wd = _linear(n, k, seed=n + k + m)
    rng = np.random.default_rng(m)
    x = torch.from_numpy(rng.standard_normal((m, k), dtype=np.float32)).cuda()
    stream = torch.cuda.current_stream().cuda_stream
    y_run = torch.empty((m, n), dtype=torch.float32, device="cuda")
    lin.run_ptr(x.data_ptr(), m, y_run.data_ptr(), stream)
    ys = []
    for _ in range(2):
        y = torch.full((m, n), float("nan"), dtype=torch.float32, device="cuda")
        _lib.check(_static(lin, x, y, stream))
        ys.append(y)
    torch.cuda.synchronize()
    ref = y_run.cpu().numpy().astype(np.float64)
    wn = np.linalg.norm(wd.astype(np.float64), axis=1)
    xn = np.linalg.norm(x.cpu().numpy().astype(np.float64), axis=1)
    tol = 1e-6 * xn[:, None] * wn[None, :] + 1e-30
    for y in ys:
        got = y.cpu().numpy().astype(np.float64)
        assert np.isfinite(got).all()
        err = np.abs(got - ref)
        assert (err <= tol).all(), float((err / tol).max())
    lin.close()


def test_static_rejects_in_features_over_limit():
    import torch
    lin, _ = _linear(16, STATIC_MAX_K + 32, seed=7)
    x = torch.zeros((1, STATIC_MAX_K + 32), dtype=torch.float32, device="cuda")
    y = torch.full((1, 16), 123.0, dtype=torch.float32, device="cuda")
    rc = _static(lin, x, y, torch.cuda.current_stream().cuda_stream)
    assert rc == -10, rc  # MC_E_CAPACITY
    assert "static scratch limit" in _lib.last_error()
    torch.cuda.synchronize()
    assert (y.cpu().numpy() == 123.0).all()  # nothing launched
    lin.close()


def test_static_zero_tokens_is_a_no_op():
    import torch
    lin, _ = _linear(16, 64, seed=3)
    assert _lib.lib().mc_linear_run_static(lin.handle, None, 0, None,
                                           torch.cuda.current_stream().cuda_stream) == 0
    lin.close()
