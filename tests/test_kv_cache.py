"""The reference's KV cache features on the device, against the oracle.

* INT8 KV (use_int8_kv, KvLayer::Int8, transformer.rs:167-420): every
  appended token's K and V quantized with one scale per token; forward
  logits within 1e-3 of the oracle's INT8 cache, greedy speculative decoding
  token for token.
* The context shift (GenerationConfig::max_context / anchor_tokens,
  generate.rs:26-63 after every round and fallback step, generate.rs:671-681
  and :738-748): plain and anchored, FP32 and INT8 caches, with the
  reference's n-gram drafter, its MLP drafter and a transformer draft; the
  generated ids and accepted counts of every round equal the oracle's.
* Prefix-cache restore (speculative_generate with a CacheLookup,
  generate.rs:617-636; the server inserts prompt + generated ids with the
  returned cache, serve/infer.rs:122-175): a second request whose prompt
  starts with the first one's tokens restores their K/V from a snapshot and
  primes only the rest, and decodes as the oracle does from the first run's
  final cache.
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
SMALL_GQA = LlamaConfig(2, 128, 4, 2, 32, 176, 64, 500000.0, 1e-5, MODE_GENERAL, "small-gqa-v64")
MID_GQA = LlamaConfig(2, 512, 8, 2, 64, 1024, 2048, 500000.0, 1e-5, MODE_GENERAL, "mid-gqa")


def _oracle(ws, cfg):
    c = cfg.resolved()
    return o.OracleModel({k: v.dequant() for k, v in ws.items()}, c.n_layers, c.hidden, c.vocab,
                         c.ffn, mode=cfg.mode, n_heads=c.n_heads, n_kv_heads=c.n_kv_heads,
                         head_dim=c.head_dim, rope_base=c.rope_theta, eps=c.eps)


def _prompt(cfg, n_motif=5, seed=5):
    rng = np.random.default_rng(seed)
    motif = rng.integers(0, cfg.vocab, n_motif).tolist()
    noise = rng.integers(0, cfg.vocab, 6).tolist()
    return motif + noise[:3] + motif + noise[3:] + motif[:4]


def _weak_layers(tw, scale=0.05):
    """The target's layers scaled down: its logits are dominated by the head
    on the embedding, so their top-2 margins are wide.  With an INT8 cache,
    a K/V code of the device and the oracle can differ by one where the two
    f32 values straddle a rounding boundary (their arithmetic differs in the
    last bits); wide margins keep such a code from changing a greedy token."""
    for k, v in tw.items():
        if k.startswith("model.layers.") and v.dtype == "i8_row":
            tw[k] = mb.QTensor("i8_row", v.data, (v.scales * np.float32(scale)).astype(np.float32))
    return tw


def _mirror_mlp(tw, scale=0.05):
    """A target with weak layers and an MLP drafter whose logits are the
    target head applied to the raw embedding (often accepted)."""
    tw = _weak_layers(tw, scale)
    emb = tw["model.embed_tokens.weight"].dequant()
    head = tw["lm_head.weight"].dequant()
    eye = np.eye(emb.shape[1], dtype=np.float32)
    t = {"draft.embed.weight": emb, "draft.fc1.weight": np.concatenate([eye, -eye]),
         "draft.fc1.bias": np.zeros(2 * emb.shape[1], np.float32),
         "draft.fc2.weight": np.concatenate([head, -head], axis=1),
         "draft.fc2.bias": np.zeros(head.shape[0], np.float32)}
    ref = o.OracleMlpDraft(t["draft.embed.weight"], t["draft.fc1.weight"], t["draft.fc1.bias"],
                           t["draft.fc2.weight"], t["draft.fc2.bias"])
    return tw, t, ref


def _prefix_draft(tw):
    """The target's embedding, norms, first layer and head: a one-layer draft
    that agrees with the target on some rounds."""
    return {k: v for k, v in tw.items()
            if not k.startswith("model.layers.") or k.startswith("model.layers.0.")}


def _close_enough(got, ref, rtol=1e-3):
    for i in range(ref.shape[0]):
        scale = np.abs(ref[i]).max()
        assert np.abs(got[i] - ref[i]).max() <= rtol * scale, i


# ---------------------------------------------------------------- INT8 KV
@pytest.mark.parametrize("cfg", [SMALL_REF, SMALL_GQA, MID_GQA], ids=lambda c: c.name)
def test_int8_kv_forward_matches_oracle(cfg):
    ws = mb.synth_weights(cfg, seed=0)
    ids = np.random.default_rng(7).integers(0, cfg.vocab, 21).tolist()
    om = _oracle(ws, cfg)
    kv = om.new_kv(64)
    kv.set_mode(o.KV_INT8)
    ref = np.concatenate([om.forward_ids(ids[:13], kv), om.forward_ids(ids[13:], kv)])
    s = mb.Session(mb.Weights(ws, cfg), None, gamma=1, max_context=64, kv_mode=mb.KV_INT8)
    got = np.concatenate([s.forward(ids[:13]), s.forward(ids[13:])])
    s.close()
    _close_enough(got, ref)
    # the int8 cache differs from the f32 one
    kv32 = om.new_kv(64)
    assert np.abs(om.forward_ids(ids, kv32) - ref).max() > 0


@pytest.mark.parametrize("drafter", ["llama", "ngram"])
def test_int8_kv_spec_decode_matches_oracle(drafter):
    cfg = SMALL_GQA
    tw = _weak_layers(mb.synth_weights(cfg, seed=0), 0.25)
    dw = _prefix_draft(tw)
    ot, od = _oracle(tw, cfg), _oracle(dw, cfg.with_layers(1))
    prompt = _prompt(cfg)
    D = mb.Weights(dw, cfg.with_layers(1)) if drafter == "llama" else None
    odraft = o.OracleLlamaDraft(od, 128) if drafter == "llama" else None
    ref, racc = ot.speculative_generate(prompt, 40, 3, odraft, kv_mode=o.KV_INT8)
    s = mb.Session(mb.Weights(tw, cfg), D, gamma=3, max_context=128, kv_mode=mb.KV_INT8)
    got, gacc = s.speculative_generate(prompt, 40)
    s.close()
    assert got == ref
    assert gacc == racc


# ---------------------------------------------------------------- context shift
CASES = [("ngram", 0, o.KV_FP32), ("ngram", 4, o.KV_FP32), ("ngram", 4, o.KV_INT8),
         ("ngram", 0, o.KV_INT8), ("mlp", 0, o.KV_FP32), ("mlp", 3, o.KV_FP32),
         ("llama", 0, o.KV_FP32), ("llama", 5, o.KV_INT8)]


@pytest.mark.parametrize("drafter,anchor,kv_mode", CASES,
                         ids=[f"{d}-anchor{a}-kv{k}" for d, a, k in CASES])
def test_context_shift_matches_oracle(drafter, anchor, kv_mode):
    cfg = SMALL_GQA
    tw = mb.synth_weights(cfg, seed=2)
    if kv_mode == o.KV_INT8:
        tw = _weak_layers(tw, 0.25)
    odraft, D = None, None
    if drafter == "mlp":
        tw, t, odraft = _mirror_mlp(tw)
        D = mb.MlpDraftModel(t)
    elif drafter == "llama":
        dw = _prefix_draft(tw)
        odraft = o.OracleLlamaDraft(_oracle(dw, cfg.with_layers(1)), 256)
        D = mb.Weights(dw, cfg.with_layers(1))
    ot = _oracle(tw, cfg)
    prompt = _prompt(cfg, seed=11)  # 22 tokens
    shift, n_new, gamma = 32, 22, 3  # a shift keeps 24 tokens, so 22 new ones are reached
    ref, racc = ot.speculative_generate(prompt, n_new, gamma, odraft, max_context=shift,
                                        anchor_tokens=anchor, kv_mode=kv_mode, rounds_cap=512)
    s = mb.Session(mb.Weights(tw, cfg), D, gamma=gamma, max_context=64, shift_context=shift,
                   anchor_tokens=anchor, kv_mode=kv_mode)
    s.prime(prompt)
    s.decode(n_new)
    got, gacc = s.read(cap=256)
    with pytest.raises(mb.McError):  # the shifted context no longer holds the prompt
        s.rewind()
    s.close()
    if drafter == "mlp":
        D.close()
    assert got == ref
    assert gacc == racc
    print(f"{drafter} anchor {anchor} kv {kv_mode}: {len(ref)} ids, {len(racc)} rounds, "
          f"{sum(racc)} drafts accepted")


def test_context_shift_rejects_bad_configs():
    cfg = SMALL_GQA
    W = mb.Weights(mb.synth_weights(cfg, seed=0), cfg)
    with pytest.raises(mb.McError):  # no room for a round above the threshold
        mb.Session(W, None, gamma=4, max_context=40, shift_context=36)
    with pytest.raises(mb.McError):  # greedy sessions only
        mb.Session(W, mb.Weights(mb.synth_weights(cfg.with_layers(1), seed=1),
                                 cfg.with_layers(1)), gamma=2, max_context=64,
                   shift_context=30, temperature=0.8)
    with pytest.raises(mb.McError):
        mb.Session(W, None, gamma=2, max_context=64, kv_mode=7)


# ---------------------------------------------------------------- prefix cache
@pytest.mark.parametrize("drafter,kv_mode", [("ngram", o.KV_FP32), ("llama", o.KV_FP32),
                                             ("ngram", o.KV_INT8)])
def test_prefix_cache_restore_matches_oracle(drafter, kv_mode):
    cfg = SMALL_GQA
    tw = mb.synth_weights(cfg, seed=4)
    if kv_mode == o.KV_INT8:
        tw = _weak_layers(tw, 0.25)
    dw = mb.synth_weights(cfg.with_layers(1), seed=5)
    ot, od = _oracle(tw, cfg), _oracle(dw, cfg.with_layers(1))
    W = mb.Weights(tw, cfg)
    D = mb.Weights(dw, cfg.with_layers(1)) if drafter == "llama" else None
    p1 = _prompt(cfg, seed=21)
    # request 1: decode, snapshot the final state (prompt + generated ids)
    s = mb.Session(W, D, gamma=3, max_context=128, kv_mode=kv_mode)
    s.prime(p1)
    s.decode(12)
    g1, _ = s.read()
    cache = mb.PrefixCache(4)
    cache.insert(p1 + g1, s.snapshot())
    s.close()
    okv = ot.new_kv(160)
    okv.set_mode(kv_mode)
    r1, _ = ot.speculative_generate(p1, 12, 3, o.OracleLlamaDraft(od, 160) if D else None,
                                    kv_mode=kv_mode, kv=okv)
    assert r1 == g1
    # request 2: its prompt extends request 1's tokens
    p2 = p1 + g1 + np.random.default_rng(6).integers(0, cfg.vocab, 5).tolist()
    hit = cache.lookup(p2)
    assert hit is not None and hit.matched_len == len(p1) + len(g1)
    assert hit.kv.tokens == p1 + g1
    s = mb.Session(W, D, gamma=3, max_context=128, kv_mode=kv_mode)
    s.prime_cached(hit.kv, p2)
    s.decode(16)
    got, gacc = s.read()
    s.close()
    ref, racc = ot.speculative_generate(p2, 16, 3, o.OracleLlamaDraft(od, 160) if D else None,
                                        kv_mode=kv_mode, kv=okv, matched_len=hit.matched_len)
    assert got == ref
    assert gacc == racc
    # a snapshot whose tokens are not a prefix of the prompt is refused
    s = mb.Session(W, D, gamma=3, max_context=128, kv_mode=kv_mode)
    with pytest.raises(mb.McError):
        s.prime_cached(hit.kv, [1, 2, 3] + p2)
    s.close()


# ---------------------------------------------------------------- MIXED KV
# use_mixed_kv (KvLayer::Mixed, transformer.rs:180-193, :389-419): the last 64
# tokens in f32, older ones int8.  The device appends and ages a MIXED cache
# token by token, verify steps included; the acceptance rolls back the window
# moves of the steps it drops.  Contexts past 64 tokens exercise the cold part.
def _long_prompt(cfg, n, seed):
    rng = np.random.default_rng(seed)
    motif = rng.integers(0, cfg.vocab, 6).tolist()
    out = []
    while len(out) < n:
        out += motif + rng.integers(0, cfg.vocab, 3).tolist()
    return out[:n]


@pytest.mark.parametrize("cfg", [SMALL_REF, SMALL_GQA], ids=lambda c: c.name)
def test_mixed_kv_forward_matches_oracle(cfg):
    ws = mb.synth_weights(cfg, seed=0)
    ids = np.random.default_rng(9).integers(0, cfg.vocab, 90).tolist()
    om = _oracle(ws, cfg)
    kv = om.new_kv(128)
    kv.set_mode(o.KV_MIXED, 64)
    ref = np.concatenate([om.forward_ids(ids[:50], kv), om.forward_ids(ids[50:], kv)])
    s = mb.Session(mb.Weights(ws, cfg), None, gamma=1, max_context=128, kv_mode=mb.KV_MIXED)
    got = np.concatenate([s.forward(ids[:50]), s.forward(ids[50:])])
    s.close()
    _close_enough(got, ref)


@pytest.mark.parametrize("drafter", ["llama", "ngram"])
def test_mixed_kv_spec_decode_matches_oracle(drafter):
    cfg = SMALL_GQA
    tw = _weak_layers(mb.synth_weights(cfg, seed=0), 0.25)
    dw = _prefix_draft(tw)
    ot, od = _oracle(tw, cfg), _oracle(dw, cfg.with_layers(1))
    prompt = _long_prompt(cfg, 70, seed=3)
    D = mb.Weights(dw, cfg.with_layers(1)) if drafter == "llama" else None
    odraft = o.OracleLlamaDraft(od, 256) if drafter == "llama" else None
    ref, racc = ot.speculative_generate(prompt, 30, 3, odraft, kv_mode=o.KV_MIXED)
    s = mb.Session(mb.Weights(tw, cfg), D, gamma=3, max_context=160, kv_mode=mb.KV_MIXED)
    got, gacc = s.speculative_generate(prompt, 30)
    s.close()
    assert got == ref
    assert gacc == racc
    print(f"mixed {drafter}: {len(ref)} ids, {len(racc)} rounds, {sum(racc)} drafts accepted")


@pytest.mark.parametrize("anchor", [0, 4])
def test_mixed_kv_context_shift_matches_oracle(anchor):
    cfg = SMALL_GQA
    tw = _weak_layers(mb.synth_weights(cfg, seed=2), 0.25)
    ot = _oracle(tw, cfg)
    prompt = _long_prompt(cfg, 80, seed=4)
    shift, n_new = 90, 40
    ref, racc = ot.speculative_generate(prompt, n_new, 3, None, max_context=shift,
                                        anchor_tokens=anchor, kv_mode=o.KV_MIXED, rounds_cap=512)
    s = mb.Session(mb.Weights(tw, cfg), None, gamma=3, max_context=128, shift_context=shift,
                   anchor_tokens=anchor, kv_mode=mb.KV_MIXED)
    s.prime(prompt)
    s.decode(n_new)
    got, gacc = s.read(cap=256)
    s.close()
    assert got == ref
    assert gacc == racc


def test_mixed_kv_prefix_cache_matches_oracle():
    cfg = SMALL_GQA
    tw = _weak_layers(mb.synth_weights(cfg, seed=6), 0.25)
    ot = _oracle(tw, cfg)
    W = mb.Weights(tw, cfg)
    p1 = _long_prompt(cfg, 66, seed=8)
    s = mb.Session(W, None, gamma=3, max_context=160, kv_mode=mb.KV_MIXED)
    s.prime(p1)
    s.decode(10)
    g1, _ = s.read()
    snap = s.snapshot()
    s.close()
    okv = ot.new_kv(200)
    okv.set_mode(o.KV_MIXED, 64)
    r1, _ = ot.speculative_generate(p1, 10, 3, None, kv_mode=o.KV_MIXED, kv=okv)
    assert r1 == g1
    p2 = p1 + g1 + [3, 1, 4, 1, 5]
    s = mb.Session(W, None, gamma=3, max_context=160, kv_mode=mb.KV_MIXED)
    s.prime_cached(snap, p2)
    s.decode(14)
    got, gacc = s.read()
    s.close()
    ref, racc = ot.speculative_generate(p2, 14, 3, None, kv_mode=o.KV_MIXED, kv=okv,
                                        matched_len=len(p1) + len(g1))
    assert got == ref
    assert gacc == racc
