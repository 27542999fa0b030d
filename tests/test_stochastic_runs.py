"""Stochastic speculative decoding, validated over whole runs.

1. Accepted-length histograms at the TinyLlama benchmark widths (d 2048, 32/4
   heads, FFN 5632, vocab 32000, q4_0, gamma 5, temperature 0.8, bonus
   token), for the distribution-preserving min(1, p/q) rule and for the
   reference's rule (the target's own sample must equal the draft,
   generate.rs:695-726), over runs of 60 new tokens from one prompt.  The
   device runs >= 10^4 rounds (many seeds); the oracle's restatement of the
   same scheme runs >= 400 rounds on disjoint seeds; a two-sample
   chi-square test of homogeneity must not reject (p > 0.01).  (On equal
   seeds the two agree token for token, which test_stochastic.py checks;
   here the samples are independent.)
2. Whole-run token frequencies against the exact target distribution: a
   target whose layers are all zero is a Markov chain (its next-token
   distribution softmax(head . rmsnorm(embed(prev)) / T) depends on the
   previous token only), so every emitted token -- not only the first of a
   run -- must follow its row of the transition matrix, whatever the draft
   proposes.  Chi-square over all (previous, next) cells, p > 0.01, for both
   acceptance rules.
"""
import os
import sys

import numpy as np
import pytest

sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "oracle"))
import oracle as o  # noqa: E402

import modelc_b200 as mb  # noqa: E402
import shape_models as sm  # noqa: E402
from modelc_b200.model import LlamaConfig, MODE_GENERAL  # noqa: E402

pytestmark = pytest.mark.gpu

TL = mb.TINYLLAMA.with_layers(2)
TEMP = 0.8
GAMMA = 5


def _chi2_sf(stat, dof):
    from scipy.stats import chi2
    return float(chi2.sf(stat, dof))


def two_sample_pvalue(a, b, min_expected=5.0):
    """Chi-square test of homogeneity of two count vectors over the same
    bins; bins expecting fewer than min_expected are merged from the tail."""
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    na, nb = a.sum(), b.sum()
    bins_a, bins_b, acc_a, acc_b = [], [], 0.0, 0.0
    for x, y in zip(a[::-1], b[::-1]):  # merge from the rare tail
        acc_a += x
        acc_b += y
        tot = acc_a + acc_b
        if min(tot * na / (na + nb), tot * nb / (na + nb)) >= min_expected:
            bins_a.append(acc_a)
            bins_b.append(acc_b)
            acc_a = acc_b = 0.0
    if acc_a + acc_b > 0:
        if bins_a:
            bins_a[-1] += acc_a
            bins_b[-1] += acc_b
        else:
            bins_a.append(acc_a)
            bins_b.append(acc_b)
    ca, cb = np.array(bins_a), np.array(bins_b)
    tot = ca + cb
    ea, eb = tot * na / (na + nb), tot * nb / (na + nb)
    stat = ((ca - ea) ** 2 / ea).sum() + ((cb - eb) ** 2 / eb).sum()
    return _chi2_sf(stat, max(len(ca) - 1, 1))


@pytest.fixture(scope="module")
def tinyllama_pair():
    tw = sm.host_weights(TL, seed=0, fmt="q4_0")
    dw = sm.prefix_draft(tw)  # the target's first layer: p and q overlap
    dcfg = TL.with_layers(1)
    deq = sm.Dequant()
    W, D = mb.Weights(tw, TL), mb.Weights(dw, dcfg)
    yield W, D, sm.oracle_model(tw, TL, deq), sm.oracle_model(dw, dcfg, deq)
    W.close()
    D.close()


@pytest.mark.parametrize("mode", [0, 1], ids=["min1pq", "reference-rule"])
def test_tinyllama_width_accepted_length_histogram(tinyllama_pair, mode):
    W, D, ot, od = tinyllama_pair
    # runs of 60 new tokens from one prompt: the process both sides sample
    prompt = np.random.default_rng(2).integers(0, TL.vocab, 16).tolist()
    n_new = 60
    gpu = np.zeros(GAMMA + 1, np.int64)
    s = mb.Session(W, D, gamma=GAMMA, max_context=160, temperature=TEMP, seed=1000,
                   accept_mode=mode, bonus=True)
    s.prime(prompt)
    seed = 100_000
    while gpu.sum() < 10_000:
        s.set_seed(seed)
        s.rewind()
        s.decode(n_new)
        _, acc = s.read(cap=256)
        gpu += np.bincount(acc, minlength=GAMMA + 1)[:GAMMA + 1]
        seed += 1
    s.close()
    ref = np.zeros(GAMMA + 1, np.int64)
    seed = 1
    while ref.sum() < 400:
        _, racc = ot.speculative_sample(prompt, n_new, GAMMA, o.OracleLlamaDraft(od, 160), TEMP,
                                        seed, accept_mode=mode, bonus=True)
        ref += np.bincount(racc, minlength=GAMMA + 1)[:GAMMA + 1]
        seed += 1
    p = two_sample_pvalue(gpu, ref)
    print(f"mode {mode}: device {gpu.tolist()} ({gpu.sum()} rounds, mean "
          f"{(gpu * np.arange(GAMMA + 1)).sum() / gpu.sum():.3f}), oracle {ref.tolist()} "
          f"({ref.sum()} rounds, mean {(ref * np.arange(GAMMA + 1)).sum() / ref.sum():.3f}), "
          f"p = {p:.3g}")
    assert gpu.sum() >= 10_000
    assert p > 0.01, (gpu.tolist(), ref.tolist(), p)


# a Markov target: zero layers, so the logits depend on the previous token only
MK = LlamaConfig(2, 64, 2, 1, 32, 128, 48, 10000.0, 1e-5, MODE_GENERAL, "markov-v48")
MK_STD = 0.25


def _markov_models():
    tw = mb.synth_weights(MK, seed=0, std=MK_STD)
    for k, v in list(tw.items()):
        if k.startswith("model.layers.") and v.dtype == "i8_row":
            tw[k] = mb.QTensor("i8_row", np.zeros_like(v.data), v.scales)
    dw = mb.synth_weights(MK.with_layers(1), seed=1, std=MK_STD)
    return tw, dw


def _transition_matrix(tw):
    """P[i, j] = softmax(logits(i) / T)_j of the zero-layer target, from the
    oracle's forward of the single token i."""
    c = MK.resolved()
    om = o.OracleModel({k: v.dequant() for k, v in tw.items()}, c.n_layers, c.hidden, c.vocab,
                       c.ffn, mode=MK.mode, n_heads=c.n_heads, n_kv_heads=c.n_kv_heads,
                       head_dim=c.head_dim, rope_base=c.rope_theta, eps=c.eps)
    P = np.zeros((MK.vocab, MK.vocab))
    for i in range(MK.vocab):
        lg = om.forward_ids([i], om.new_kv(4))[0].astype(np.float64)
        z = (lg - lg.max()) / TEMP
        e = np.exp(z)
        P[i] = e / e.sum()
    return P


@pytest.mark.parametrize("mode", [0, 1], ids=["min1pq", "reference-rule"])
def test_whole_run_token_frequencies_follow_the_target(mode):
    tw, dw = _markov_models()
    P = _transition_matrix(tw)
    W, D = mb.Weights(tw, MK), mb.Weights(dw, MK.with_layers(1))
    prompt = [3, 17, 5, 40, 22, 9, 1]
    counts = np.zeros((MK.vocab, MK.vocab))
    s = mb.Session(W, D, gamma=4, max_context=1100, temperature=TEMP, seed=7, accept_mode=mode,
                   bonus=True)
    s.prime(prompt)
    for seed in range(40):
        s.set_seed(20_000 + seed)
        s.rewind()
        s.decode(1000)
        toks, _ = s.read(cap=1100)
        seq = [prompt[-1]] + toks[:1000]
        np.add.at(counts, (np.array(seq[:-1]), np.array(seq[1:])), 1.0)
    s.close()
    # chi-square over the cells of every previous token, merged per row where
    # they expect fewer than 5
    stat, dof = 0.0, 0
    for i in range(MK.vocab):
        n = counts[i].sum()
        if n < 50:
            continue
        exp = P[i] * n
        order = np.argsort(exp)
        acc_o = acc_e = 0.0
        bo, be = [], []
        for j in order:
            acc_o += counts[i, j]
            acc_e += exp[j]
            if acc_e >= 5:
                bo.append(acc_o)
                be.append(acc_e)
                acc_o = acc_e = 0.0
        if acc_e > 0 and bo:
            bo[-1] += acc_o
            be[-1] += acc_e
        bo, be = np.array(bo), np.array(be)
        stat += ((bo - be) ** 2 / be).sum()
        dof += len(bo) - 1
    p = _chi2_sf(stat, dof)
    print(f"mode {mode}: {int(counts.sum())} transitions, chi2 {stat:.1f} on {dof} dof, p = {p:.3g}")
    assert counts.sum() >= 40_000
    assert p > 0.01, p
