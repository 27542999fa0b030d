"""Concurrent requests (batched sessions) and forwards of more than 16 tokens.

A batched session decodes B greedy requests in lock step: each round runs
the draft steps over B tokens (one per request, each at its own position),
one verify forward over B x (gamma or gamma+1) positions, and B acceptances.
Every request must produce exactly the tokens and accepted counts that the
oracle's single-request speculative_generate (generate.rs:598-767) produces
for its prompt: requests share weights and launches, never state.  Requests
finish at different rounds; a finished request's state stays frozen
(generate.rs:638 checks the budget at round start).

Forwards of 17..64 tokens run int8 projections on the tcgen05 GEMM with
48 digit columns per group of 16 tokens, and q4_0 projections as one GEMV
pass per group; both must match the oracle (logits within 1e-3) and be
bit-identical to the same tokens in smaller launches.
"""
import os
import sys

import numpy as np
import pytest

sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "oracle"))
import oracle as o  # noqa: E402

import modelc_b200 as mb  # noqa: E402
from modelc_b200.model import LlamaConfig, MODE_GENERAL, MODE_REFERENCE  # noqa: E402

pytestmark = pytest.mark.gpu

SMALL_REF = LlamaConfig(2, 128, 2, 2, 64, 160, 300, mode=MODE_REFERENCE, name="small-ref")
SMALL_GQA = LlamaConfig(2, 128, 4, 2, 32, 176, 260, 500000.0, 1e-5, MODE_GENERAL, "small-gqa")
MID_GQA = LlamaConfig(2, 512, 8, 2, 64, 1024, 2048, 500000.0, 1e-5, MODE_GENERAL, "mid-gqa")


def oracle_for(ws, cfg):
    c = cfg.resolved()
    return o.OracleModel({k: v.dequant() for k, v in ws.items()}, c.n_layers, c.hidden,
                         c.vocab, c.ffn, mode=cfg.mode, n_heads=c.n_heads,
                         n_kv_heads=c.n_kv_heads, head_dim=c.head_dim, rope_base=c.rope_theta,
                         eps=c.eps)


def prefix_draft(tw):
    """The target's embedding, head, norms and first layer: a draft that
    agrees with the target often but not always (accepted counts vary)."""
    return {k: v for k, v in tw.items() if not k.startswith("model.layers.") or
            k.startswith("model.layers.0.")}


def prompts_for(cfg, B, seed=11):
    rng = np.random.default_rng(seed)
    lens = [13, 7, 30, 21, 5, 17, 9, 26][:B]
    return [rng.integers(0, cfg.vocab, n).tolist() for n in lens]


@pytest.mark.parametrize("cfg", [SMALL_REF, SMALL_GQA], ids=lambda c: c.name)
@pytest.mark.parametrize("B,gamma,bonus", [(2, 4, False), (4, 2, True), (8, 4, False),
                                           (8, 4, True), (3, 1, False)])
@pytest.mark.parametrize("draft_kind", ["random", "prefix"])
def test_batch_spec_generate_matches_oracle(cfg, B, gamma, bonus, draft_kind):
    tw = mb.synth_weights(cfg, seed=0)
    dcfg = cfg.with_layers(1)
    dw = mb.synth_weights(dcfg, seed=1) if draft_kind == "random" else prefix_draft(tw)
    prompts = prompts_for(cfg, B)
    n_new = 24
    od = oracle_for(dw, dcfg)
    ot = oracle_for(tw, cfg)
    refs = [ot.speculative_generate(p, n_new, gamma, o.OracleLlamaDraft(od, 128), bonus=bonus)
            for p in prompts]
    s = mb.Session(mb.Weights(tw, cfg), mb.Weights(dw, dcfg), gamma=gamma, max_context=128,
                   bonus=bonus, n_requests=B)
    got = s.speculative_generate_batch(prompts, n_new)
    s.close()
    for z, ((gt, gacc), (rt, racc)) in enumerate(zip(got, refs)):
        assert gt == rt, z
        assert gacc == racc, z


def test_batch_decode_resumable_and_rewind():
    cfg = SMALL_GQA
    tw = mb.synth_weights(cfg, seed=0)
    dw = prefix_draft(tw)
    prompts = prompts_for(cfg, 4, seed=3)
    s = mb.Session(mb.Weights(tw, cfg), mb.Weights(dw, cfg.with_layers(1)), gamma=3,
                   max_context=128, n_requests=4)
    s.prime_batch(prompts)
    s.decode(10)
    s.decode(20)
    first = [s.read(request=z) for z in range(4)]
    s.rewind()
    s.decode(20)
    again = [s.read(request=z) for z in range(4)]
    assert first == again
    whole = s.speculative_generate_batch(prompts, 20)
    assert whole == first
    for toks, _ in first:
        assert len(toks) >= 20
    s.close()


def test_batch_rejects_bad_configs():
    cfg = SMALL_GQA
    W = mb.Weights(mb.synth_weights(cfg, seed=0), cfg)
    D = mb.Weights(mb.synth_weights(cfg.with_layers(1), seed=1), cfg.with_layers(1))
    with pytest.raises(mb.McError):  # 16 x 5 positions > 64 tokens per forward
        mb.Session(W, D, gamma=4, bonus=True, max_context=64, n_requests=16)
    with pytest.raises(mb.McError):  # batched sessions are greedy
        mb.Session(W, D, gamma=4, max_context=64, n_requests=2, temperature=0.8)
    s = mb.Session(W, D, gamma=2, max_context=64, n_requests=2)
    with pytest.raises(mb.McError):  # one prompt per request
        s.prime_batch([[1, 2, 3]])
    with pytest.raises(mb.McError):  # the single-request call on a batched session
        s.prime([1, 2, 3])
    s.close()


@pytest.mark.parametrize("cfg,fmt", [(SMALL_GQA, "i8_row"), (MID_GQA, "i8_row"),
                                     (MID_GQA, "q4_0")], ids=["small", "mid", "mid-q4"])
def test_long_forward_matches_oracle_and_splits(cfg, fmt):
    ws = mb.synth_weights(cfg, seed=0, fmt=fmt)
    ids = np.random.default_rng(7).integers(0, cfg.vocab, 150).tolist()  # 64 + 64 + 22
    om = oracle_for(ws, cfg)
    ref = om.forward_ids(ids, om.new_kv(192))
    W = mb.Weights(ws, cfg)
    s = mb.Session(W, None, gamma=1, max_context=192)
    got = s.forward(ids)
    for i in range(ref.shape[0]):
        scale = np.abs(ref[i]).max()
        assert np.abs(got[i] - ref[i]).max() <= 1e-3 * scale, i
    s2 = mb.Session(W, None, gamma=1, max_context=192)
    parts = [s2.forward(ids[:16]), s2.forward(ids[16:17]), s2.forward(ids[17:57]),
             s2.forward(ids[57:150])]
    assert np.array_equal(np.concatenate(parts), got)


def _lin_case(n, k, m, seed):
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal((n, k), dtype=np.float32) * np.float32(0.02)).astype(np.float32)
    x = rng.standard_normal((m, k), dtype=np.float32)
    return w, x


@pytest.mark.parametrize("fmt", ["i8_row", "q4_0"])
@pytest.mark.parametrize("n,k", [(300, 512), (4096, 4096), (1024, 14336)])
@pytest.mark.parametrize("m", [17, 33, 40, 64])
def test_linear_wide_matches_oracle_and_is_batch_invariant(fmt, n, k, m):
    import torch
    w, x = _lin_case(n, k, m, seed=n + k + m)
    if fmt == "i8_row":
        q, sc = mb.quantize_int8_rows(w)
        qt = mb.QTensor("i8_row", q, sc)
        wd = o.dequant_int8_rows(q, sc)
    else:
        blk = mb.model.quantize_q4_0(w)
        qt = mb.QTensor("q4_0", blk, None, (n, k))
        wd = mb.model.dequant_q4_0(blk, n, k)
    lin = mb.Linear(qt)
    xt = torch.from_numpy(x).cuda()
    y = lin(xt).cpu().numpy()
    wn = np.linalg.norm(wd.astype(np.float64), axis=1)
    for i in range(m):
        ref = o.linear(wd, x[i])
        tol = 1e-4 * wn * np.linalg.norm(x[i].astype(np.float64)) + 1e-30
        assert (np.abs(y[i].astype(np.float64) - ref) <= tol).all(), i
    for sl in [slice(0, 1), slice(3, 12), slice(5, 21), slice(m - 17, m)]:
        yi = lin(xt[sl].contiguous()).cpu().numpy()
        assert np.array_equal(yi, y[sl]), sl


def test_linear_token_counts_across_routes():
    """A matrix of 8192 rows runs 1..8 tokens on the GEMV (two and three
    digit tiles) and 9..64 on the tcgen05 GEMM: every slice must equal the
    same rows of one 20-token call bit for bit, and match the oracle."""
    import torch
    w, x = _lin_case(8192, 512, 20, seed=5)
    q, sc = mb.quantize_int8_rows(w)
    lin = mb.Linear(mb.QTensor("i8_row", q, sc))
    wd = o.dequant_int8_rows(q, sc)
    xt = torch.from_numpy(x).cuda()
    y = lin(xt).cpu().numpy()
    wn = np.linalg.norm(wd.astype(np.float64), axis=1)
    for i in range(20):
        tol = 1e-4 * wn * np.linalg.norm(x[i].astype(np.float64)) + 1e-30
        assert (np.abs(y[i].astype(np.float64) - o.linear(wd, x[i])) <= tol).all(), i
    for a, b in [(0, 1), (1, 6), (2, 8), (3, 11), (2, 12), (4, 20)]:
        assert np.array_equal(lin(xt[a:b].contiguous()).cpu().numpy(), y[a:b]), (a, b)
