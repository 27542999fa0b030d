"""The oracle's transformer forward and speculative loop, cross-checked.

* the reference's Llama test fixture (tests/common/mod.rs:278-358) and seeded
  synthetic models against an independent float64 forward;
* speculative_generate invariants that follow from generate.rs:598-767:
  greedy output equals plain greedy decoding of the prompt with its last
  token repeated (the re-forward at generate.rs:697, quirk Q1); tokens per
  round are accepted+1 except for fully accepted rounds; the bonus variant
  emits the same greedy stream;
* the parallel (row-split) linear is bit-identical to the sequential one.
"""
import os
import sys

import numpy as np
import pytest

HERE = os.path.dirname(__file__)
sys.path.insert(0, os.path.join(os.path.dirname(HERE), "oracle"))
import oracle as o  # noqa: E402
from mc_fixtures import (LLAMA_HIDDEN, LLAMA_INTER, LLAMA_VOCAB,  # noqa: E402
                         f64_forward_seq, reference_llama_fixture)

from modelc_b200.model import LlamaConfig, MODE_GENERAL, MODE_REFERENCE, synth_weights  # noqa: E402


def dequant_all(ws):
    return {k: v.dequant() for k, v in ws.items()}


def oracle_model(w, cfg, n_threads=1):
    c = cfg.resolved()
    return o.OracleModel(w, c.n_layers, c.hidden, c.vocab, c.ffn, mode=cfg.mode,
                         n_heads=c.n_heads, n_kv_heads=c.n_kv_heads, head_dim=c.head_dim,
                         rope_base=c.rope_theta, eps=c.eps, n_threads=n_threads)


SMALL_REF = LlamaConfig(2, 128, 2, 2, 64, 160, 300, mode=MODE_REFERENCE, name="small-ref")
SMALL_GQA = LlamaConfig(2, 128, 4, 2, 32, 176, 260, 500000.0, 1e-5, MODE_GENERAL, "small-gqa")


def test_fixture_forward_matches_f64():
    w = reference_llama_fixture()
    m = o.OracleModel(w, 1, LLAMA_HIDDEN, LLAMA_VOCAB, LLAMA_INTER)
    assert (m.m.n_heads, m.m.head_dim) == (1, 12)  # hidden/64 -> 1 head (arch.rs:136)
    ids = [1, 4, 7, 2, 9]
    kv = m.new_kv(16)
    got = m.forward_ids(ids, kv)
    ref = f64_forward_seq(w, ids, 1, 1, 1, 12, 10000.0, 1e-6)
    scale = np.abs(ref).max(axis=1, keepdims=True)
    assert np.all(np.abs(got - ref) <= 1e-4 * scale + 1e-4)
    assert len(kv) == len(ids)


@pytest.mark.parametrize("cfg", [SMALL_REF, SMALL_GQA], ids=lambda c: c.name)
def test_synthetic_forward_matches_f64(cfg):
    ws = synth_weights(cfg, seed=5)
    w = dequant_all(ws)
    m = oracle_model(w, cfg)
    ids = np.random.default_rng(1).integers(0, cfg.vocab, 9).tolist()
    got = m.forward_ids(ids, m.new_kv(32))
    c = cfg.resolved()
    ref = f64_forward_seq(w, ids, c.n_layers, c.n_heads, c.n_kv_heads, c.head_dim,
                          c.rope_theta, c.eps)
    rel = np.abs(got - ref).max() / np.abs(ref).max()
    assert rel < 1e-5, rel


def test_forward_without_cache_is_single_position():
    # kv_cache None: pos = 0, attention over the token itself (transformer.rs:779-787)
    ws = synth_weights(SMALL_REF, seed=2)
    m = oracle_model(dequant_all(ws), SMALL_REF)
    a = m.forward_ids([7])
    b = m.forward_ids([7], m.new_kv(4))
    assert np.array_equal(a, b)


def test_no_head_returns_none():  # transformer.rs:94-95
    w = reference_llama_fixture()
    del w["lm_head.weight"], w["model.embed_tokens.weight"]
    m = o.OracleModel(w, 1, LLAMA_HIDDEN, LLAMA_VOCAB, LLAMA_INTER)
    assert m.forward_ids([1]) is None


def test_tied_head_uses_embedding():
    w = reference_llama_fixture()
    w2 = dict(w)
    del w2["lm_head.weight"]
    a = o.OracleModel(w, 1, LLAMA_HIDDEN, LLAMA_VOCAB, LLAMA_INTER).forward_ids([3])
    b = o.OracleModel(w2, 1, LLAMA_HIDDEN, LLAMA_VOCAB, LLAMA_INTER).forward_ids([3])
    assert np.array_equal(a, b)  # fixture lm_head == embed_tokens


def test_parallel_linear_bit_identical():
    rng = np.random.default_rng(0)
    w = rng.standard_normal((203, 517)).astype(np.float32)
    x = rng.standard_normal(517).astype(np.float32)
    assert np.array_equal(o.linear(w, x), o.linear_par(w, x, 7))


@pytest.mark.parametrize("gamma", [1, 3, 4])
def test_spec_greedy_equals_plain_greedy_with_repeat(gamma):
    cfg = SMALL_REF
    m = oracle_model(dequant_all(synth_weights(cfg, seed=0)), cfg)
    dm = oracle_model(dequant_all(synth_weights(cfg.with_layers(1), seed=1)), cfg.with_layers(1))
    prompt = np.random.default_rng(2).integers(0, cfg.vocab, 12).tolist()
    draft = o.OracleLlamaDraft(dm, 128)
    toks, acc = m.speculative_generate(prompt, 20, gamma, draft)
    plain = m.generate_core(prompt + [prompt[-1]], 40)
    assert toks == plain[: len(toks)]
    assert 20 <= len(toks) <= 20 + gamma - 1  # overshoot bound (generate.rs:638, :751)
    assert len(acc) >= 1 and all(0 <= a <= gamma for a in acc)
    # tokens per round: accepted + 1 unless every draft was accepted
    assert sum(a + (a < gamma) for a in acc) == len(toks)


def test_self_draft_high_acceptance():
    # A drafter with the target's weights still sees the context without the
    # re-forwarded last prompt token (Q1), so it agrees often but not always.
    cfg = SMALL_REF
    w = dequant_all(synth_weights(cfg, seed=0))
    m = oracle_model(w, cfg)
    prompt = [5, 9, 1, 200, 33, 7]
    toks, acc = m.speculative_generate(prompt, 16, 4, o.OracleLlamaDraft(oracle_model(w, cfg), 64))
    assert sum(acc) >= len(acc)  # far above the ~1/vocab of an unrelated draft
    plain = m.generate_core(prompt + [prompt[-1]], 40)
    assert toks == plain[: len(toks)]


def test_bonus_variant_same_greedy_stream():
    cfg = SMALL_REF
    m = oracle_model(dequant_all(synth_weights(cfg, seed=0)), cfg)
    dm = oracle_model(dequant_all(synth_weights(cfg.with_layers(1), seed=1)), cfg.with_layers(1))
    prompt = np.random.default_rng(4).integers(0, cfg.vocab, 10).tolist()
    a, _ = m.speculative_generate(prompt, 15, 3, o.OracleLlamaDraft(dm, 128))
    b, accb = m.speculative_generate(prompt, 15, 3, o.OracleLlamaDraft(dm, 128), bonus=True)
    n = min(len(a), len(b))
    assert a[:n] == b[:n]
    assert sum(x + 1 for x in accb) == len(b)


def test_llama_draft_prefix_reuse_matches_fresh():
    cfg = SMALL_REF
    dm = oracle_model(dequant_all(synth_weights(cfg.with_layers(1), seed=1)), cfg.with_layers(1))
    ctx = np.random.default_rng(6).integers(0, cfg.vocab, 20).tolist()
    warm = o.OracleLlamaDraft(dm, 64)
    warm.draft(ctx[:12], 4)
    warm.draft(ctx[:15], 3)
    assert warm.draft(ctx, 4) == o.OracleLlamaDraft(dm, 64).draft(ctx, 4)


def test_ngram_speculation_on_fixture():
    # n-gram drafter (the reference's default drafter, generate.rs:642-646)
    w = reference_llama_fixture()
    m = o.OracleModel(w, 1, LLAMA_HIDDEN, LLAMA_VOCAB, LLAMA_INTER)
    prompt = [1, 2, 3, 1, 2, 3, 1, 2]
    toks, acc = m.speculative_generate(prompt, 8, 3)
    plain = m.generate_core(prompt + [prompt[-1]], 16)
    assert toks == plain[: len(toks)]


def test_empty_prompt_generates_nothing():  # generate.rs:609-611
    m = o.OracleModel(reference_llama_fixture(), 1, LLAMA_HIDDEN, LLAMA_VOCAB, LLAMA_INTER)
    assert m.speculative_generate([], 5, 2)[0] == []
    assert m.generate_core([], 5) == []
