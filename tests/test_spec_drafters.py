"""The reference's own drafters driving the device speculative loop.

speculative_generate (generate.rs:598-767) drafts with the DraftModel it is
given -- modelc's server wires MlpDraftModel (serve/mod.rs:151-166) -- and
with its trigram n-gram index when it has none (generate.rs:615, :642-646).
Both now run inside the session's round graph: the MLP's gamma greedy steps,
or the n-gram round (index update, up to gamma drafts, possibly none), then
the batched verify and the acceptance.  Each request must reproduce the
oracle's speculative_generate with the same drafter exactly: the generated
ids and the accepted count of every round (n-gram fallback steps, where no
key matches, run one standard generation step and log no round).

The n-gram cases use prompts with repeats and small models whose greedy
continuations fall into cycles, so rounds with long accepted drafts, short
drafts and fallback steps all occur.  The MLP drafter mirrors the target (FC1
= [I; -I] and FC2 = [H, -H] give H . e, the head on the raw embedding, while
the target's layers are scaled down), so its drafts are often accepted.
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


def _oracle(ws, cfg):
    c = cfg.resolved()
    return o.OracleModel({k: v.dequant() for k, v in ws.items()}, c.n_layers, c.hidden, c.vocab,
                         c.ffn, mode=cfg.mode, n_heads=c.n_heads, n_kv_heads=c.n_kv_heads,
                         head_dim=c.head_dim, rope_base=c.rope_theta, eps=c.eps)


def _prompts(cfg, B, seed=5):
    rng = np.random.default_rng(seed)
    out = []
    for z in range(B):
        motif = rng.integers(0, cfg.vocab, 5).tolist()
        noise = rng.integers(0, cfg.vocab, 3 + z).tolist()
        out.append(motif + noise[:2] + motif + noise[2:] + motif[:4])
    return out


@pytest.mark.parametrize("cfg", [SMALL_REF, SMALL_GQA], ids=lambda c: c.name)
@pytest.mark.parametrize("gamma,bonus", [(1, False), (3, False), (4, True), (4, False)])
def test_ngram_drafter_spec_decode_matches_oracle(cfg, gamma, bonus):
    tw = mb.synth_weights(cfg, seed=0)
    W = mb.Weights(tw, cfg)
    ot = _oracle(tw, cfg)
    prompt = _prompts(cfg, 1)[0]
    ref, racc = ot.speculative_generate(prompt, 48, gamma, None, bonus=bonus)
    s = mb.Session(W, None, gamma=gamma, max_context=128, bonus=bonus)
    got, gacc = s.speculative_generate(prompt, 48)
    s.close()
    assert got == ref
    assert gacc == racc
    print(f"{cfg.name} gamma {gamma} bonus {bonus}: {len(ref)} tokens, {len(racc)} drafted "
          f"rounds, {sum(racc)} drafts accepted")


@pytest.mark.parametrize("B", [2, 4])
def test_ngram_drafter_batched_requests(B):
    cfg = SMALL_GQA
    tw = mb.synth_weights(cfg, seed=1)
    W = mb.Weights(tw, cfg)
    ot = _oracle(tw, cfg)
    prompts = _prompts(cfg, B, seed=9)
    refs = [ot.speculative_generate(p, 30, 3, None) for p in prompts]
    s = mb.Session(W, None, gamma=3, max_context=128, n_requests=B)
    got = s.speculative_generate_batch(prompts, 30)
    s.close()
    for z, ((gt, gacc), (rt, racc)) in enumerate(zip(got, refs)):
        assert gt == rt, z
        assert gacc == racc, z


def _mirror_mlp(tw, cfg, layer_scale=0.05):
    """A target with weak layers and an MLP drafter whose logits are the
    target head applied to the raw embedding."""
    for k, v in tw.items():
        if k.startswith("model.layers.") and v.dtype == "i8_row":
            tw[k] = mb.QTensor("i8_row", v.data, (v.scales * np.float32(layer_scale)).astype(np.float32))
    emb = tw["model.embed_tokens.weight"].dequant()
    head = tw["lm_head.weight"].dequant()
    d = emb.shape[1]
    eye = np.eye(d, dtype=np.float32)
    t = {"draft.embed.weight": emb, "draft.fc1.weight": np.concatenate([eye, -eye]),
         "draft.fc1.bias": np.zeros(2 * d, np.float32),
         "draft.fc2.weight": np.concatenate([head, -head], axis=1),
         "draft.fc2.bias": np.zeros(head.shape[0], np.float32)}
    ref = o.OracleMlpDraft(t["draft.embed.weight"], t["draft.fc1.weight"], t["draft.fc1.bias"],
                           t["draft.fc2.weight"], t["draft.fc2.bias"])
    return tw, t, ref


@pytest.mark.parametrize("cfg", [SMALL_REF, SMALL_GQA], ids=lambda c: c.name)
@pytest.mark.parametrize("gamma,bonus", [(2, False), (4, True), (4, False)])
def test_mlp_drafter_spec_decode_matches_oracle(cfg, gamma, bonus):
    tw, t, odraft = _mirror_mlp(mb.synth_weights(cfg, seed=2), cfg)
    ot = _oracle(tw, cfg)
    prompt = np.random.default_rng(4).integers(0, cfg.vocab, 11).tolist()
    ref, racc = ot.speculative_generate(prompt, 40, gamma, odraft, bonus=bonus)
    mlp = mb.MlpDraftModel(t)
    s = mb.Session(mb.Weights(tw, cfg), mlp, gamma=gamma, max_context=128, bonus=bonus)
    got, gacc = s.speculative_generate(prompt, 40)
    s.close()
    mlp.close()
    assert got == ref
    assert gacc == racc
    assert sum(racc) > 0  # the mirrored drafter is accepted on some rounds


def test_mlp_drafter_batched_and_rejects_sampling():
    cfg = SMALL_GQA
    tw, t, odraft = _mirror_mlp(mb.synth_weights(cfg, seed=3), cfg)
    ot = _oracle(tw, cfg)
    rng = np.random.default_rng(8)
    prompts = [rng.integers(0, cfg.vocab, n).tolist() for n in (9, 14, 5)]
    refs = [ot.speculative_generate(p, 25, 4, odraft) for p in prompts]
    mlp = mb.MlpDraftModel(t)
    W = mb.Weights(tw, cfg)
    s = mb.Session(W, mlp, gamma=4, max_context=128, n_requests=3)
    got = s.speculative_generate_batch(prompts, 25)
    s.close()
    for z, ((gt, gacc), (rt, racc)) in enumerate(zip(got, refs)):
        assert gt == rt, z
        assert gacc == racc, z
    with pytest.raises(mb.McError):  # the reference samples the MLP unseeded
        mb.Session(W, mlp, gamma=4, max_context=64, temperature=0.8)
    s = mb.Session(W, None, gamma=4, max_context=64, temperature=0.8)
    with pytest.raises(mb.McError):  # stochastic rounds read a draft distribution
        s.prime(prompts[0])
    s.close()
    mlp.close()
