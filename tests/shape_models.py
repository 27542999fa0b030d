"""Models at the benchmarked widths for the GPU parity tests.

The weights are drawn on the GPU (``synth_weights_torch``: N(0, 0.02), the
per-row int8 or q4_0 rule) and copied to the host, where they feed both the
device loader and the oracle.  The oracle receives dequantized f32 arrays;
tensors shared between two models (a prefix draft reuses the target's
embedding, norms, first layer and head) are dequantized once and shared, so
an 8B-width pair needs about 6 GB of host memory.
"""
from __future__ import annotations

import os
import sys

import numpy as np

sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "oracle"))
import oracle as o  # noqa: E402

import modelc_b200 as mb  # noqa: E402

LOGIT_RTOL = 1e-3
N_THREADS = os.cpu_count() or 1


def host_weights(cfg, seed, fmt):
    """Seeded weights of cfg as host QTensors (drawn on cuda:0)."""
    import torch
    tt = mb.synth_weights_torch(cfg, seed=seed, device=torch.device("cuda", 0), fmt=fmt)
    out = {}
    for name in list(tt):
        dt, t, extra = tt.pop(name)
        if dt == "f32":
            out[name] = mb.QTensor("f32", t.cpu().numpy())
        elif dt == "i8_row":
            out[name] = mb.QTensor("i8_row", t.cpu().numpy(), extra.cpu().numpy())
        else:
            out[name] = mb.QTensor("q4_0", t.cpu().numpy(), None, tuple(extra))
        del t, extra
    torch.cuda.empty_cache()
    return out


def prefix_draft(tw):
    """The target's embedding, norms, first layer and head: a draft that
    agrees with the target on some rounds and not on others."""
    return {k: v for k, v in tw.items()
            if not k.startswith("model.layers.") or k.startswith("model.layers.0.")}


class Dequant:
    """f32 copies of QTensors, made once per tensor object."""

    def __init__(self):
        self._cache = {}

    def __call__(self, qt):
        hit = self._cache.get(id(qt))
        if hit is None:
            hit = (qt, qt.dequant())
            self._cache[id(qt)] = hit
        return hit[1]


def oracle_model(ws, cfg, deq):
    c = cfg.resolved()
    return o.OracleModel({k: deq(v) for k, v in ws.items()}, c.n_layers, c.hidden, c.vocab,
                         c.ffn, mode=cfg.mode, n_heads=c.n_heads, n_kv_heads=c.n_kv_heads,
                         head_dim=c.head_dim, rope_base=c.rope_theta, eps=c.eps,
                         n_threads=N_THREADS)


def logits_report(got, ref):
    """Checks every row of device logits against the oracle's: max error
    within LOGIT_RTOL of the row's largest |logit|, and the same argmax
    wherever the oracle's top-1/top-2 margin exceeds twice that row's error
    (where it does not, the two orders are within rounding).  Returns the
    smallest relative top-1/top-2 margin and the largest relative error."""
    assert got.shape == ref.shape
    min_margin, max_err = np.inf, 0.0
    for i in range(ref.shape[0]):
        scale = float(np.abs(ref[i]).max())
        err = float(np.abs(got[i].astype(np.float64) - ref[i]).max())
        assert err <= LOGIT_RTOL * scale, (i, err / scale)
        top2 = np.sort(ref[i])[-2:]
        margin = float(top2[1] - top2[0])
        min_margin = min(min_margin, margin / scale)
        max_err = max(max_err, err / scale)
        if margin > 2 * err:
            assert int(np.argmax(got[i])) == o.argmax(ref[i]), i
    return min_margin, max_err
