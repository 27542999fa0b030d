"""mc_linear_run_static, the allocation-free projection, against mc_linear_run.

Some callers cannot allocate device memory once they are serving: a process
whose HBM is already split between weights and KV pages under a hard budget,
or a decode loop that must not let cudaMalloc/cudaFree synchronise a GPU it
shares.  For them the library keeps the projection's activation scratch in a
fixed device array of its own.  Each case makes two static calls in a row on
the same input, plus one mc_linear_run call, and checks that all three agree.
Tolerance per output row: |y_static - y_run| <= 1e-6 * ||w_row|| * ||x||, the
form the projection tests use against the oracle but 100x tighter (both
routes sum exactly in int32, so the results are expected to be identical).

The cases cover int8 rows and q4_0 weights; matrices with few rows, where the
GEMV splits k inside a CTA; and more than 16 tokens on 8192 rows, where
mc_linear_run takes the tcgen05 GEMM and the static call the GEMV.  One case
runs in a fresh process whose first static call is on a non-default stream.
The file sorts last so that it also runs after every other GPU test in one
process.
"""

import os
import subprocess
import sys
import textwrap

import numpy as np
import pytest

import modelc_b200 as mb
from modelc_b200 import _lib

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
STATIC_MAX_K = 16384


def _linear(n, k, seed, fmt="i8_row"):
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal((n, k), dtype=np.float32) * np.float32(0.02)).astype(np.float32)
    if fmt == "q4_0":
        blk = mb.model.quantize_q4_0(w)
        return (mb.Linear(mb.QTensor("q4_0", blk, None, (n, k))),
                mb.model.dequant_q4_0(blk, n, k))
    q, s = mb.quantize_int8_rows(w)
    return mb.Linear(mb.QTensor("i8_row", q, s)), q.astype(np.float32) * s[:, None]


def _static(lin, x, y, stream):
    return _lib.lib().mc_linear_run_static(lin.handle, x.data_ptr(), x.shape[0], y.data_ptr(),
                                           stream)


@pytest.mark.parametrize("n,k,m,fmt", [
    (4096, 4096, 1, "i8_row"), (4096, 4096, 5, "i8_row"), (256, 14336, 16, "i8_row"),
    (300, 517, 20, "i8_row"), (1024, STATIC_MAX_K, 3, "i8_row"),
    (16, 64, 4, "i8_row"), (40, 517, 7, "i8_row"),        # few stripes: k split inside a CTA
    (8192, 1024, 24, "i8_row"),                           # mc_linear_run takes tcgen05 here
    (512, 4096, 5, "q4_0"), (40, 1024, 3, "q4_0"), (300, 2048, 18, "q4_0")])
def test_static_matches_run_twice(n, k, m, fmt):
    import torch
    lin, wd = _linear(n, k, seed=n + k + m, fmt=fmt)
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


_FRESH = textwrap.dedent("""
    import sys
    import numpy as np
    import torch
    sys.path.insert(0, {root!r})
    import modelc_b200 as mb
    from modelc_b200 import _lib
    rng = np.random.default_rng(5)
    w = (rng.standard_normal((1024, 4096), dtype=np.float32) * np.float32(0.02))
    q, s = mb.quantize_int8_rows(w)
    lin = mb.Linear(mb.QTensor("i8_row", q, s))
    x = torch.from_numpy(rng.standard_normal((5, 4096), dtype=np.float32)).cuda()
    side = torch.cuda.Stream()          # non-blocking with respect to the legacy stream
    torch.cuda.synchronize()
    with torch.cuda.stream(side):
        y0 = torch.full((5, 1024), float("nan"), device="cuda")
        y1 = torch.full((5, 1024), float("nan"), device="cuda")
    side.synchronize()
    # the first static call of this process runs on the side stream
    _lib.check(_lib.lib().mc_linear_run_static(lin.handle, x.data_ptr(), 5, y0.data_ptr(),
                                               side.cuda_stream))
    _lib.check(_lib.lib().mc_linear_run_static(lin.handle, x.data_ptr(), 5, y1.data_ptr(),
                                               side.cuda_stream))
    yr = torch.empty((5, 1024), device="cuda")
    lin.run_ptr(x.data_ptr(), 5, yr.data_ptr(), side.cuda_stream)
    side.synchronize()
    a, b, r = (t.cpu().numpy().astype(np.float64) for t in (y0, y1, yr))
    wn = np.linalg.norm((q.astype(np.float32) * s[:, None]).astype(np.float64), axis=1)
    xn = np.linalg.norm(x.cpu().numpy().astype(np.float64), axis=1)
    tol = 1e-6 * xn[:, None] * wn[None, :]
    assert np.isfinite(a).all() and np.isfinite(b).all()
    assert (np.abs(a - r) <= tol).all() and (np.abs(b - r) <= tol).all()
    print("fresh-process static ok")
""")


def test_static_first_call_on_side_stream_in_fresh_process():
    res = subprocess.run([sys.executable, "-c", _FRESH.format(root=ROOT)], capture_output=True,
                         text=True, timeout=600)
    assert res.returncode == 0, res.stdout[-2000:] + res.stderr[-4000:]
    assert "fresh-process static ok" in res.stdout


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
