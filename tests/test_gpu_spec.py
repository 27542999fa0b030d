"""Greedy speculative decoding on the B200 against the oracle.

The device round (draft k tokens -> one batched verify -> acceptance -> KV
rollback, captured in a CUDA graph) must reproduce the oracle's restatement
of speculative_generate (generate.rs:598-767) exactly: the same generated
ids and the same accepted-draft count for every round.
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


def oracle_for(ws, cfg):
    c = cfg.resolved()
    return o.OracleModel({k: v.dequant() for k, v in ws.items()}, c.n_layers, c.hidden,
                         c.vocab, c.ffn, mode=cfg.mode, n_heads=c.n_heads,
                         n_kv_heads=c.n_kv_heads, head_dim=c.head_dim, rope_base=c.rope_theta,
                         eps=c.eps)


def models(cfg, draft_layers=1, tseed=0, dseed=1):
    tw = mb.synth_weights(cfg, seed=tseed)
    dw = mb.synth_weights(cfg.with_layers(draft_layers), seed=dseed)
    return tw, dw


@pytest.mark.parametrize("cfg", [SMALL_REF, SMALL_GQA], ids=lambda c: c.name)
@pytest.mark.parametrize("gamma", [1, 2, 4])
@pytest.mark.parametrize("bonus", [False, True])
def test_spec_generate_matches_oracle(cfg, gamma, bonus):
    tw, dw = models(cfg)
    prompt = np.random.default_rng(11).integers(0, cfg.vocab, 13).tolist()
    ot, oacc = oracle_for(tw, cfg).speculative_generate(
        prompt, 24, gamma, o.OracleLlamaDraft(oracle_for(dw, cfg.with_layers(1)), 128),
        bonus=bonus)
    W, D = mb.Weights(tw, cfg), mb.Weights(dw, cfg.with_layers(1))
    s = mb.Session(W, D, gamma=gamma, max_context=128, bonus=bonus)
    gt, gacc = s.speculative_generate(prompt, 24)
    assert gt == ot
    assert gacc == oacc


def test_spec_self_draft_matches_oracle():
    # the draft shares the target's weights: many accepted rounds
    cfg = SMALL_REF
    tw = mb.synth_weights(cfg, seed=0)
    prompt = [5, 9, 1, 200, 33, 7, 12, 99]
    ot, oacc = oracle_for(tw, cfg).speculative_generate(
        prompt, 30, 4, o.OracleLlamaDraft(oracle_for(tw, cfg), 128))
    W = mb.Weights(tw, cfg)
    s = mb.Session(W, W, gamma=4, max_context=128)
    gt, gacc = s.speculative_generate(prompt, 30)
    assert gt == ot and gacc == oacc
    assert sum(gacc) > len(gacc)


def test_tiny_config_spec_decode():
    # the tiny reference-mode workload: 4L target (seed 0), 1L draft (seed 1),
    # 32-id prompt (seed 2), gamma 4, greedy, 128 new tokens
    cfg = mb.TINY
    tw, dw = models(cfg)
    prompt = np.random.default_rng(2).integers(0, cfg.vocab, 32).tolist()
    ot, oacc = oracle_for(tw, cfg).speculative_generate(
        prompt, 128, 4, o.OracleLlamaDraft(oracle_for(dw, cfg.with_layers(1)), 256))
    s = mb.Session(mb.Weights(tw, cfg), mb.Weights(dw, cfg.with_layers(1)), gamma=4,
                   max_context=256)
    gt, gacc = s.speculative_generate(prompt, 128)
    assert gt == ot and gacc == oacc


def test_draft_model_trait_matches_oracle():
    cfg = SMALL_GQA
    tw, dw = models(cfg)
    od = o.OracleLlamaDraft(oracle_for(dw, cfg.with_layers(1)), 128)
    gd = mb.LlamaDraftModel(mb.Weights(tw, cfg), mb.Weights(dw, cfg.with_layers(1)), 128)
    ctx = np.random.default_rng(5).integers(0, cfg.vocab, 40).tolist()
    for n, g in [(10, 4), (14, 3), (40, 5), (20, 2)]:
        assert gd.draft(ctx[:n], g) == od.draft(ctx[:n], g)


def test_decode_is_resumable_and_repeatable():
    cfg = SMALL_REF
    tw, dw = models(cfg)
    W, D = mb.Weights(tw, cfg), mb.Weights(dw, cfg.with_layers(1))
    prompt = list(range(3, 20))
    s = mb.Session(W, D, gamma=3, max_context=160)
    s.prime(prompt)
    s.decode(10)
    s.decode(40)
    a = s.read()
    s.prime(prompt)
    s.decode(40)
    assert s.read() == a
