"""Stochastic speculative decoding (temperature > 0).

The device draws every random number from Philox4x32-10 keyed by the
session seed with counter (slot, round); the oracle restates the same
scheme and stream.  Checks:

* Philox4x32-10 against the published Random123 known-answer vectors.
* The oracle's first emitted token follows the target distribution
  softmax(p / T) (chi-square, p > 0.01): the defining property of the
  min(1, p/q) scheme with residual resampling.
* GPU == oracle token for token on fixed seeds (both sample from nearly
  identical f32 distributions with the same uniforms; only a uniform landing
  within ~1e-6 of a CDF boundary could split them).
* GPU first-token frequencies against the exact target distribution
  (chi-square, p > 0.01), and the first-position acceptance rate against its
  analytic value: sum_v min(p(v), q(v)) for min(1, p/q), sum_v p(v) q(v) for
  the reference's sample == draft rule (within 4 standard deviations).
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

CFG = LlamaConfig(2, 64, 2, 1, 32, 128, 48, 10000.0, 1e-5, MODE_GENERAL, "stoch-tiny")
TEMP = 0.8
STD = 0.25  # wider than 0.02 so that p and q are far from uniform
PROMPT = [3, 17, 5, 40, 22, 9, 1]


def test_philox_random123_vectors():
    assert o.philox4x32_10([0, 0, 0, 0], [0, 0]) == [0x6627e8d5, 0xe169c58d, 0xbc57ac4c,
                                                    0x9b00dbd8]
    assert o.philox4x32_10([0xffffffff] * 4, [0xffffffff] * 2) == [0x408f276d, 0x41c83b0e,
                                                                  0xa20bc7c6, 0x6d5451fd]
    assert o.philox4x32_10([0x243f6a88, 0x85a308d3, 0x13198a2e, 0x03707344],
                           [0xa4093822, 0x299f31d0]) == [0xd16cfe09, 0x94fdcceb, 0x5001e420,
                                                         0x24126ea1]


def test_philox_uniform_range_and_streams():
    u = [o.philox_uniform(7, r, s) for r in range(20) for s in range(8)]
    assert all(0.0 <= x < 1.0 for x in u)
    assert len(set(u)) == len(u)
    assert o.philox_uniform(7, 3, 2) == o.philox_uniform(7, 3, 2)
    assert o.philox_uniform(7, 3, 2) != o.philox_uniform(8, 3, 2)


def _models():
    tw = mb.synth_weights(CFG, seed=0, std=STD)
    dw = mb.synth_weights(CFG.with_layers(1), seed=1, std=STD)
    return tw, dw


def _oracle(ws, cfg):
    c = cfg.resolved()
    return o.OracleModel({k: v.dequant() for k, v in ws.items()}, c.n_layers, c.hidden,
                         c.vocab, c.ffn, mode=cfg.mode, n_heads=c.n_heads,
                         n_kv_heads=c.n_kv_heads, head_dim=c.head_dim, rope_base=c.rope_theta,
                         eps=c.eps)


def _softmax_t(logits):
    z = (logits.astype(np.float64) - logits.max()) / TEMP
    e = np.exp(z)
    return e / e.sum()


def _first_distributions(tw, dw):
    """p1: target after the primed prompt plus the last prompt token again
    (quirk Q1); q1: draft after the prompt."""
    ot = _oracle(tw, CFG)
    p_logits = ot.forward_ids(PROMPT + [PROMPT[-1]], ot.new_kv(32))[-1]
    od = _oracle(dw, CFG.with_layers(1))
    q_logits = od.forward_ids(PROMPT, od.new_kv(32))[-1]
    return _softmax_t(p_logits), _softmax_t(q_logits)


def _chi2_pvalue(counts, probs):
    from scipy.stats import chi2
    n = counts.sum()
    exp = probs * n
    order = np.argsort(exp)
    # merge the rarest categories until every bin expects >= 5
    bins_o, bins_e, acc_o, acc_e = [], [], 0.0, 0.0
    for i in order:
        acc_o += counts[i]
        acc_e += exp[i]
        if acc_e >= 5:
            bins_o.append(acc_o)
            bins_e.append(acc_e)
            acc_o = acc_e = 0.0
    if acc_e > 0:
        bins_o[-1] += acc_o
        bins_e[-1] += acc_e
    bins_o, bins_e = np.array(bins_o), np.array(bins_e)
    stat = ((bins_o - bins_e) ** 2 / bins_e).sum()
    return float(chi2.sf(stat, len(bins_o) - 1))


def test_oracle_first_token_follows_target_distribution():
    tw, dw = _models()
    p1, _ = _first_distributions(tw, dw)
    ot = _oracle(tw, CFG)
    od = _oracle(dw, CFG.with_layers(1))
    counts = np.zeros(CFG.vocab)
    for seed in range(1500):
        toks, _ = ot.speculative_sample(PROMPT, 1, 3, o.OracleLlamaDraft(od, 32), TEMP, seed)
        counts[toks[0]] += 1
    assert _chi2_pvalue(counts, p1) > 0.01


@gpu
@pytest.mark.parametrize("mode", [0, 1])
@pytest.mark.parametrize("gamma,bonus", [(2, False), (4, False), (3, True)])
def test_gpu_matches_oracle_on_fixed_seeds(mode, gamma, bonus):
    tw, dw = _models()
    ot, od = _oracle(tw, CFG), _oracle(dw, CFG.with_layers(1))
    W, D = mb.Weights(tw, CFG), mb.Weights(dw, CFG.with_layers(1))
    for seed in (1, 2, 3):
        ref, racc = ot.speculative_sample(PROMPT, 20, gamma, o.OracleLlamaDraft(od, 64), TEMP,
                                          seed, accept_mode=mode, bonus=bonus)
        s = mb.Session(W, D, gamma=gamma, max_context=64, bonus=bonus, temperature=TEMP,
                       seed=seed, accept_mode=mode)
        got, gacc = s.speculative_generate(PROMPT, 20)
        s.close()
        assert got == ref, (seed, got, ref)
        assert gacc == racc


def _gpu_first_tokens(mode, n_seeds, gamma=3):
    tw, dw = _models()
    s = mb.Session(mb.Weights(tw, CFG), mb.Weights(dw, CFG.with_layers(1)), gamma=gamma,
                   max_context=64, temperature=TEMP, accept_mode=mode)
    s.prime(PROMPT)
    first, acc0 = np.zeros(CFG.vocab), 0
    for seed in range(n_seeds):
        s.set_seed(10_000 + seed)
        s.rewind()
        s.decode(1)
        toks, acc = s.read(8)
        first[toks[0]] += 1
        acc0 += acc[0] > 0
    s.close()
    return tw, dw, first, acc0


@gpu
@pytest.mark.parametrize("mode", [0, 1])
def test_gpu_first_token_distribution_and_acceptance(mode):
    n = 4000
    tw, dw, first, acc0 = _gpu_first_tokens(mode, n)
    p1, q1 = _first_distributions(tw, dw)
    assert _chi2_pvalue(first, p1) > 0.01
    rate = np.minimum(p1, q1).sum() if mode == 0 else (p1 * q1).sum()
    sd = np.sqrt(rate * (1 - rate) / n)
    assert abs(acc0 / n - rate) < 4 * sd + 1e-3, (acc0 / n, rate)
