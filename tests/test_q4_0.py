"""q4_0 weights (ggml blocks of 32 along K, one fp16 scale per block;
parsers/gguf/dequant.rs:23-46) through the device path.

CPU: the numpy and torch quantizers produce the oracle's bytes, and the
dequantization matches the oracle's restatement of dequantize_q4_0.

GPU: the q4_0 projection against the oracle (dequantized f32 weights, f32
sequential sums).  The device sums each 32-wide block exactly in int32, then
scales it by the block's fp16 scale and accumulates in f32, so its error is a
few f32 roundings per block: tolerance |y - y_oracle| <= 1e-4 * ||w_row|| *
||x||, as for int8 rows.  Results are deterministic and independent of how
many tokens share a launch (the k-split of a q4_0 matrix does not depend on
the token count).  A q4_0 model's forward logits match the oracle within
1e-3, and greedy speculative decoding reproduces the oracle's tokens and
accepted counts.
"""
import os
import sys

import numpy as np
import pytest

sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "oracle"))
import oracle as o  # noqa: E402

import modelc_b200 as mb  # noqa: E402
from modelc_b200.model import LlamaConfig, MODE_GENERAL  # noqa: E402

gpu = pytest.mark.gpu

Q4_GQA = LlamaConfig(2, 128, 4, 2, 32, 192, 260, 10000.0, 1e-5, MODE_GENERAL, "q4-gqa")
Q4_MID = LlamaConfig(2, 512, 8, 2, 64, 1024, 2048, 10000.0, 1e-5, MODE_GENERAL, "q4-mid")


def _w(rows, cols, seed, std=0.02):
    rng = np.random.default_rng(seed)
    return (rng.standard_normal((rows, cols), dtype=np.float32) * np.float32(std)).astype(np.float32)


def test_q4_quantizers_match_oracle_bytes():
    import torch
    w = _w(24, 160, 0)
    w[3, :32] = 0.0                       # all-zero block
    w[5, 40] = -w[5, 41]                  # equal magnitudes: first one wins
    w[7, 64:96] = np.float32(0.5)         # uniform block
    blk = mb.model.quantize_q4_0(w)
    assert blk.shape == (24, 160 // 32 * 18)
    assert np.array_equal(blk.reshape(-1), np.asarray(o.quantize_q4_0(w)).reshape(-1))
    assert np.array_equal(mb.model._q4_0_torch(torch.from_numpy(w)).numpy(), blk)
    ref = np.asarray(o.dequant_q4_0(blk, w.size)).reshape(w.shape)
    assert np.array_equal(mb.model.dequant_q4_0(blk, 24, 160), ref)
    assert np.array_equal(mb.QTensor("q4_0", blk, None, (24, 160)).dequant(), ref)


def test_q4_rejects_ragged_rows():
    with pytest.raises(ValueError):
        mb.model.quantize_q4_0(_w(4, 40, 1))


def _check(wd, x, y):
    wn = np.linalg.norm(wd.astype(np.float64), axis=1)
    for i in range(x.shape[0]):
        ref = o.linear(wd, x[i])
        tol = 1e-4 * wn * np.linalg.norm(x[i].astype(np.float64)) + 1e-30
        err = np.abs(y[i].astype(np.float64) - ref)
        assert (err <= tol).all(), (i, float((err / tol).max()))


@gpu
@pytest.mark.parametrize("n,k", [(16, 32), (300, 512), (1024, 4096), (256, 14336), (4096, 4096)])
@pytest.mark.parametrize("m", [1, 4, 5, 16])
def test_q4_linear_matches_oracle(n, k, m):
    import torch
    w = _w(n, k, n + k)
    blk = mb.model.quantize_q4_0(w)
    wd = mb.model.dequant_q4_0(blk, n, k)
    x = np.random.default_rng(m).standard_normal((m, k), dtype=np.float32)
    lin = mb.Linear(mb.QTensor("q4_0", blk, None, (n, k)))
    y = lin(torch.from_numpy(x).cuda()).cpu().numpy()
    _check(wd, x, y)
    assert lin.weight_bytes == n * k // 32 * 18


@gpu
def test_q4_linear_deterministic_and_batch_invariant():
    import torch
    n, k = 2000, 4096
    blk = mb.model.quantize_q4_0(_w(n, k, 9))
    x = np.random.default_rng(3).standard_normal((16, k), dtype=np.float32)
    lin = mb.Linear(mb.QTensor("q4_0", blk, None, (n, k)))
    xt = torch.from_numpy(x).cuda()
    y1 = lin(xt).cpu().numpy()
    assert np.array_equal(y1, lin(xt).cpu().numpy())
    for sl in [slice(0, 1), slice(3, 8), slice(8, 13)]:
        yi = lin(xt[sl].contiguous()).cpu().numpy()
        assert np.array_equal(yi, y1[sl])


@gpu
def test_q4_linear_nonfinite_propagates():
    import torch
    blk = mb.model.quantize_q4_0(_w(32, 64, 5))
    x = np.random.default_rng(1).standard_normal((2, 64), dtype=np.float32)
    x[1, 3] = np.nan
    lin = mb.Linear(mb.QTensor("q4_0", blk, None, (32, 64)))
    y = lin(torch.from_numpy(x).cuda()).cpu().numpy()
    assert np.isfinite(y[0]).all() and np.isnan(y[1]).all()


def _oracle_for(ws, cfg):
    c = cfg.resolved()
    return o.OracleModel({k: v.dequant() for k, v in ws.items()}, c.n_layers, c.hidden,
                         c.vocab, c.ffn, mode=cfg.mode, n_heads=c.n_heads,
                         n_kv_heads=c.n_kv_heads, head_dim=c.head_dim, rope_base=c.rope_theta,
                         eps=c.eps)


@gpu
@pytest.mark.parametrize("cfg", [Q4_GQA, Q4_MID], ids=lambda c: c.name)
def test_q4_forward_logits_match_oracle(cfg):
    ws = mb.synth_weights(cfg, seed=0, fmt="q4_0")
    ids = np.random.default_rng(7).integers(0, cfg.vocab, 21).tolist()
    om = _oracle_for(ws, cfg)
    ref = om.forward_ids(ids, om.new_kv(64))
    s = mb.Session(mb.Weights(ws, cfg), None, gamma=1, max_context=64)
    got = s.forward(ids)
    for i in range(ref.shape[0]):
        scale = np.abs(ref[i]).max()
        assert np.abs(got[i] - ref[i]).max() <= 1e-3 * scale, i


@gpu
@pytest.mark.parametrize("gamma", [2, 5])
def test_q4_spec_generate_matches_oracle(gamma):
    cfg = Q4_GQA
    tw = mb.synth_weights(cfg, seed=0, fmt="q4_0")
    dw = mb.synth_weights(cfg.with_layers(1), seed=1, fmt="q4_0")
    prompt = np.random.default_rng(11).integers(0, cfg.vocab, 13).tolist()
    ot, oacc = _oracle_for(tw, cfg).speculative_generate(
        prompt, 24, gamma, o.OracleLlamaDraft(_oracle_for(dw, cfg.with_layers(1)), 128))
    s = mb.Session(mb.Weights(tw, cfg), mb.Weights(dw, cfg.with_layers(1)), gamma=gamma,
                   max_context=128)
    gt, gacc = s.speculative_generate(prompt, 24)
    assert gt == ot
    assert gacc == oacc


@gpu
def test_q4_head_dim_not_multiple_of_16_is_shape_error():
    cfg = LlamaConfig(1, 96, 4, 2, 24, 64, 64, 10000.0, 1e-5, MODE_GENERAL, "q4-hd24")
    ws = mb.synth_weights(cfg, seed=0, fmt="q4_0")
    with pytest.raises(mb.McError) as e:
        mb.Weights(ws, cfg)
    assert e.value.status == -2  # MC_E_SHAPE
