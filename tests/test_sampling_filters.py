"""Top-p and min-p (generate.rs:1034-1086) on the sampling paths.

The filters are restated on the exact weights e_v = exp((l_v - max) / T)
(max e = 1): top-p keeps the shortest prefix of (e descending, index
ascending) whose integer mass sum floor(e_v * 2^32) reaches
ceil(top_p * total); min-p drops e_v < min_p.  The reference's f32
cumulative sum can land on the other side of top_p only when it passes
within its accumulated rounding (up to about n * 2^-24 after n terms) of
it; the restatement then keeps the exact nucleus.  On the CPU the kept sets
are compared with the reference's apply_top_p / apply_min_p wherever the
reference's f32 cut equals its exact-arithmetic cut with a clear margin, runs
of tied probabilities included (the stable sort keeps the lower indices).

On the GPU:
* mc_sample_rows == the oracle's sample for every row (random logits up to
  a 128256 vocabulary, tie-heavy rows whose cut ends inside a run of equal
  logits, greedy rows with NaN, -inf and -0.0);
* stochastic sessions with top-p and min-p == the oracle's speculative_sample
  token for token on fixed seeds, both acceptance rules;
* first-token frequencies follow the filtered target distribution.
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


def _reference_kept(logits, t, top_p, min_p):
    """The reference's kept set (generate.rs:948-969 without the draw) and
    whether its decisions had a clear margin."""
    scaled = (np.asarray(logits, np.float32) / np.float32(t)).astype(np.float32)
    p = o.softmax(scaled)
    clear = True
    if 0.0 < top_p < 1.0:
        order = sorted(range(len(p)), key=lambda i: (-p[i], i))
        cum32 = np.cumsum(p[order], dtype=np.float32)  # the reference's running sum
        e = np.exp(scaled.astype(np.float64) - float(scaled.max()))
        cum64 = np.cumsum(e[order]) / e.sum()  # the exact nucleus mass
        tp = float(np.float32(top_p))
        k32 = int(np.argmax(cum32 >= np.float32(top_p))) if (cum32 >= np.float32(top_p)).any() else -1
        k64 = int(np.argmax(cum64 >= tp)) if (cum64 >= tp).any() else -1
        lo = cum64[k64 - 1] if k64 > 0 else 0.0
        clear &= k32 == k64 and abs(cum64[k64] - tp) > 1e-6 and abs(lo - tp) > 1e-6
        p = o.apply_top_p(p, top_p)
    if 0.0 < min_p < 1.0:
        thr = float(p.max()) * min_p
        clear &= bool((np.abs(p[p > 0].astype(np.float64) - thr) > 1e-6 * thr).all())
        p = o.apply_min_p(p, min_p)
    return p > 0, clear


def _cases(rng, n):
    for i in range(n):
        V = int(rng.choice([7, 50, 1000, 5000]))
        kind = i % 3
        if kind == 0:
            logits = rng.standard_normal(V).astype(np.float32) * np.float32(3.0)
        elif kind == 1:  # runs of equal logits
            logits = rng.integers(-4, 1, V).astype(np.float32)
        else:  # a few large logits over a flat tail
            logits = np.zeros(V, np.float32)
            logits[rng.integers(0, V, 5)] = rng.uniform(2, 6, 5).astype(np.float32)
        yield logits


@pytest.mark.parametrize("top_p,min_p", [(0.5, 0.0), (0.9, 0.0), (0.95, 0.05), (0.0, 0.1),
                                         (0.7, 0.3), (1.0, 0.0), (0.0, 1.0)])
def test_filtered_weights_keep_the_reference_set(top_p, min_p):
    rng = np.random.default_rng(int(top_p * 100) + int(min_p * 1000))
    compared = 0
    for logits in _cases(rng, 60):
        for t in (0.7, 1.0, 1.6):
            ref, clear = _reference_kept(logits, t, top_p, min_p)
            w, s = o.filtered_weights(logits, t, top_p, min_p)
            if not clear:
                continue
            compared += 1
            assert np.array_equal(w > 0, ref), (len(logits), t)
            assert s == pytest.approx(float(w.astype(np.float64).sum()), rel=1e-3)  # f32 running sum
    assert compared >= 150


def test_filtered_weights_kats():
    """generate.rs:1153-1231 restated on logits = log(p): the nucleus of
    [0.5, 0.3, 0.15, 0.05] at 0.7 is the first two, at 0.85 three, at 0.99
    all four; min-p 0.5 of [0.5, 0.2, 0.15, 0.15] keeps only the first, of
    [0.4, 0.3, 0.2, 0.1] at 0.6 the first two; min-p 0 changes nothing."""
    lp = np.log(np.array([0.5, 0.3, 0.15, 0.05], np.float32))
    for top_p, n in [(0.7, 2), (0.85, 3), (0.99, 4)]:
        w, _ = o.filtered_weights(lp, 1.0, top_p)
        assert (w > 0).tolist() == [True] * n + [False] * (4 - n)
    w, _ = o.filtered_weights(np.log(np.array([0.5, 0.2, 0.15, 0.15], np.float32)), 1.0, 0.0, 0.5)
    assert (w > 0).tolist() == [True, False, False, False]
    w, _ = o.filtered_weights(np.log(np.array([0.4, 0.3, 0.2, 0.1], np.float32)), 1.0, 0.0, 0.6)
    assert (w > 0).tolist() == [True, True, False, False]
    x = np.array([1.0, 2.0, 3.0], np.float32)
    assert (o.filtered_weights(x, 1.0, 0.0, 0.0)[0] > 0).all()


def test_ties_keep_lower_indices():
    """All-equal logits: the nucleus is the first ceil(top_p * V) indices
    (the reference's stable sort keeps index order among equal p)."""
    for V, top_p in [(64, 0.3), (1000, 0.5), (10, 0.95)]:
        w, _ = o.filtered_weights(np.zeros(V, np.float32), 1.0, top_p)
        k = int(np.ceil(top_p * V))
        assert (w > 0).tolist() == [True] * k + [False] * (V - k)


CFG = LlamaConfig(2, 64, 2, 1, 32, 128, 48, 10000.0, 1e-5, MODE_GENERAL, "stoch-tiny")
TEMP, STD = 0.8, 0.25
PROMPT = [3, 17, 5, 40, 22, 9, 1]
TOP_P, MIN_P = 0.8, 0.05


def _models():
    return (mb.synth_weights(CFG, seed=0, std=STD),
            mb.synth_weights(CFG.with_layers(1), seed=1, std=STD))


def _oracle(ws, cfg):
    c = cfg.resolved()
    return o.OracleModel({k: v.dequant() for k, v in ws.items()}, c.n_layers, c.hidden,
                         c.vocab, c.ffn, mode=cfg.mode, n_heads=c.n_heads,
                         n_kv_heads=c.n_kv_heads, head_dim=c.head_dim, rope_base=c.rope_theta,
                         eps=c.eps)


def _first_target_filtered(tw):
    """Target distribution of the first emitted token (the primed prompt plus
    the last prompt token again, quirk Q1) after the filters."""
    ot = _oracle(tw, CFG)
    logits = ot.forward_ids(PROMPT + [PROMPT[-1]], ot.new_kv(32))[-1]
    w, _ = o.filtered_weights(logits, TEMP, TOP_P, MIN_P)
    w = w.astype(np.float64)
    return w / w.sum()


def _chi2_pvalue(counts, probs):
    from scipy.stats import chi2
    keep = probs > 0
    assert counts[~keep].sum() == 0  # nothing outside the kept set
    n = counts.sum()
    exp = probs[keep] * n
    obs = counts[keep]
    order = np.argsort(exp)
    bins_o, bins_e, ao, ae = [], [], 0.0, 0.0
    for i in order:
        ao += obs[i]
        ae += exp[i]
        if ae >= 5:
            bins_o.append(ao)
            bins_e.append(ae)
            ao = ae = 0.0
    if ae > 0:
        bins_o[-1] += ao
        bins_e[-1] += ae
    bins_o, bins_e = np.array(bins_o), np.array(bins_e)
    if len(bins_o) < 2:
        return 1.0
    stat = ((bins_o - bins_e) ** 2 / bins_e).sum()
    return float(chi2.sf(stat, len(bins_o) - 1))


def test_oracle_first_token_follows_filtered_target():
    tw, dw = _models()
    p1 = _first_target_filtered(tw)
    assert 2 <= (p1 > 0).sum() < CFG.vocab  # the filters bite
    ot, od = _oracle(tw, CFG), _oracle(dw, CFG.with_layers(1))
    counts = np.zeros(CFG.vocab)
    for seed in range(1200):
        toks, _ = ot.speculative_sample(PROMPT, 1, 3, o.OracleLlamaDraft(od, 32), TEMP, seed,
                                        top_p=TOP_P, min_p=MIN_P)
        counts[toks[0]] += 1
    assert _chi2_pvalue(counts, p1) > 0.01


# ------------------------------------------------------------------ GPU


def _device_tokens(rows, t, top_p, min_p, seed, rnd):
    import torch
    x = torch.from_numpy(np.ascontiguousarray(rows, np.float32)).cuda()
    out = mb.sample_rows(x, t, top_p, min_p, seed, rnd)
    return out.cpu().numpy().astype(np.int64).tolist()


@gpu
@pytest.mark.parametrize("V", [10, 1000, 32000, 128256])
@pytest.mark.parametrize("top_p,min_p", [(0.0, 0.0), (0.9, 0.0), (0.0, 0.05), (0.6, 0.02)])
def test_sample_rows_match_oracle(V, top_p, min_p):
    rng = np.random.default_rng(V + int(top_p * 10) + int(min_p * 100))
    rows = (rng.standard_normal((6, V)) * 2.5).astype(np.float32)
    for t in (0.7, 1.3):
        for rnd in range(3):
            got = _device_tokens(rows, t, top_p, min_p, 11, rnd)
            ref = [o.sample_philox(rows[r], t, 11, rnd, r, top_p, min_p) for r in range(6)]
            assert got == ref, (t, rnd)


@gpu
@pytest.mark.parametrize("V,levels,top_p", [(64, 1, 0.3), (5000, 3, 0.5), (40000, 2, 0.9),
                                            (2048, 1, 0.999)])
def test_sample_rows_cut_inside_tie_runs(V, levels, top_p):
    """Logits from a few integer levels: the nucleus ends inside a run of
    equal weights, so the device must find the k-th tied index."""
    rng = np.random.default_rng(V)
    rows = rng.integers(-levels + 1, 1, (4, V)).astype(np.float32)
    seen = [set() for _ in range(4)]
    for rnd in range(40):
        got = _device_tokens(rows, 1.0, top_p, 0.0, 5, rnd)
        ref = [o.sample_philox(rows[r], 1.0, 5, rnd, r, top_p) for r in range(4)]
        assert got == ref, rnd
        for r in range(4):
            seen[r].add(got[r])
    for r in range(4):
        w, _ = o.filtered_weights(rows[r], 1.0, top_p)
        assert seen[r] <= set(np.flatnonzero(w > 0).tolist())


@gpu
def test_sample_rows_greedy_edge_values():
    """generate.rs:1088-1098 argmax: NaN and -inf never win; equal values,
    -0.0 and +0.0 included, go to the first; nothing qualifying gives 0."""
    nan, inf = np.float32(np.nan), np.float32(np.inf)
    rows = [[nan, 1.0, 3.0, 3.0], [-inf, -inf, -inf, -inf], [nan, nan, -inf, nan],
            [-0.0, 0.0, -1.0, nan], [-inf, -2.0, nan, -2.0], [inf, nan, inf, 1.0]]
    rows = np.array(rows, np.float32)
    got = _device_tokens(rows, 0.0, 0.9, 0.1, 0, 0)
    assert got == [o.argmax(r) for r in rows] == [2, 0, 0, 0, 1, 0]


@gpu
def test_sample_rows_rejects_bad_arguments():
    import torch
    x = torch.zeros((2, 8), device="cuda")
    with pytest.raises(mb.McError):
        mb.sample_rows(x, float("nan"))
    with pytest.raises(mb.McError):
        mb.sample_rows(torch.zeros((1, 262145), device="cuda"), 1.0)
    assert mb.sample_rows(x[:0], 1.0).numel() == 0


@gpu
@pytest.mark.parametrize("mode", [0, 1])
@pytest.mark.parametrize("gamma,bonus", [(2, False), (4, True)])
def test_spec_with_filters_matches_oracle(mode, gamma, bonus):
    tw, dw = _models()
    ot, od = _oracle(tw, CFG), _oracle(dw, CFG.with_layers(1))
    W, D = mb.Weights(tw, CFG), mb.Weights(dw, CFG.with_layers(1))
    for seed in (1, 2, 3):
        ref, racc = ot.speculative_sample(PROMPT, 20, gamma, o.OracleLlamaDraft(od, 64), TEMP,
                                          seed, accept_mode=mode, bonus=bonus, top_p=TOP_P,
                                          min_p=MIN_P)
        s = mb.Session(W, D, gamma=gamma, max_context=64, bonus=bonus, temperature=TEMP,
                       seed=seed, accept_mode=mode, top_p=TOP_P, min_p=MIN_P)
        got, gacc = s.speculative_generate(PROMPT, 20)
        s.close()
        assert got == ref, (seed, got, ref)
        assert gacc == racc


@gpu
def test_gpu_first_token_follows_filtered_target():
    tw, dw = _models()
    p1 = _first_target_filtered(tw)
    s = mb.Session(mb.Weights(tw, CFG), mb.Weights(dw, CFG.with_layers(1)), gamma=3,
                   max_context=64, temperature=TEMP, top_p=TOP_P, min_p=MIN_P)
    s.prime(PROMPT)
    counts = np.zeros(CFG.vocab)
    for seed in range(3000):
        s.set_seed(20_000 + seed)
        s.rewind()
        s.decode(1)
        toks, _ = s.read(8)
        counts[toks[0]] += 1
    s.close()
    assert _chi2_pvalue(counts, p1) > 0.01
