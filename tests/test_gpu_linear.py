"""Quantized projection (the verify-step GEMV/skinny GEMM) against the oracle.

y = x . dequant(W)^T with per-row int8 W (linear_with, transformer.rs:825-843,
dequant model.rs:182-185).  The device path sums exact int8 x int8 digit
products in int32, so its only rounding is the per-token fixed-point encoding
of x (2^-21 of the token's largest magnitude) and the final scaling; the
oracle accumulates sequentially in f32.  Tolerance: |y - y_oracle| <=
1e-4 * ||w_row|| * ||x||, far above both rounding budgets and far below any
real defect.  Results must also be bit-deterministic and independent of how
tokens are batched.
"""
import os
import sys

import numpy as np
import pytest

sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "oracle"))
import oracle as o  # noqa: E402

import modelc_b200 as mb  # noqa: E402

pytestmark = pytest.mark.gpu


def _case(n, k, m, seed=0):
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal((n, k), dtype=np.float32) * np.float32(0.02)).astype(np.float32)
    q, s = mb.quantize_int8_rows(w)
    x = rng.standard_normal((m, k), dtype=np.float32)
    return q, s, x


def _run(q, s, x):
    import torch
    lin = mb.Linear(mb.QTensor("i8_row", q, s))
    xt = torch.from_numpy(x).cuda()
    y = lin(xt)
    torch.cuda.synchronize()
    return lin, y.cpu().numpy()


def _check(q, s, x, y):
    wd = o.dequant_int8_rows(q, s)
    wn = np.linalg.norm(wd.astype(np.float64), axis=1)
    for i in range(x.shape[0]):
        ref = o.linear(wd, x[i])
        tol = 1e-4 * wn * np.linalg.norm(x[i].astype(np.float64)) + 1e-30
        err = np.abs(y[i].astype(np.float64) - ref)
        assert (err <= tol).all(), (i, float((err / tol).max()))


@pytest.mark.parametrize("n,k", [(16, 32), (300, 517), (1024, 4096), (4096, 4096),
                                 (256, 14336), (8, 12)])
@pytest.mark.parametrize("m", [1, 4, 5, 16])
def test_linear_matches_oracle(n, k, m):
    q, s, x = _case(n, k, m, seed=n + k + m)
    _, y = _run(q, s, x)
    _check(q, s, x, y)


def test_linear_chunked_tokens_and_ragged():
    q, s, x = _case(77, 200, 37, seed=3)  # 37 tokens -> 16 + 16 + 5
    _, y = _run(q, s, x)
    _check(q, s, x, y)


def test_linear_deterministic_and_batch_invariant():
    import torch
    q, s, x = _case(2000, 4096, 5, seed=9)
    lin, y1 = _run(q, s, x)
    y2 = lin(torch.from_numpy(x).cuda()).cpu().numpy()
    assert np.array_equal(y1, y2)
    for i in range(5):
        yi = lin(torch.from_numpy(x[i:i + 1].copy()).cuda()).cpu().numpy()
        assert np.array_equal(yi[0], y1[i])


def test_linear_extreme_activations():
    q, s, x = _case(64, 256, 3, seed=4)
    x[0] *= 1e-30
    x[1] *= 1e30
    x[2] = 0.0
    _, y = _run(q, s, x)
    assert (y[2] == 0).all()
    _check(q, s, x[:2], y[:2])


def test_linear_nonfinite_propagates():
    q, s, x = _case(32, 64, 2, seed=5)
    x[1, 3] = np.inf
    _, y = _run(q, s, x)
    assert np.isfinite(y[0]).all() and np.isnan(y[1]).all()
