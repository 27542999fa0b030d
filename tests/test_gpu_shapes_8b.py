"""Parity at the Llama-3-8B widths of the headline benchmark, with 2 layers.

Target: d 4096, 32 query / 8 KV heads of head_dim 128 (4 query rows per KV
head), FFN 14336, vocab 128256, RoPE theta 5e5, eps 1e-5, per-row int8
weights from seed 0; the kernels the 8B benchmark runs (the tensor-core
attention at head_dim 128, the QKV epilogue's RoPE pairing at theta 5e5, the
LM-head argmax over 128256 rows, the tcgen05 GEMM of the 64-token prime) all
run here.  Checked against the oracle:

* forward logits of a 33-token prime and a 5-token verify-sized forward,
  within 1e-3 of each row's largest logit, with the same argmax wherever the
  top-1/top-2 margin exceeds the error (the smallest margin is reported);
* greedy speculative decoding from a 64-token prompt, 32 new tokens, gamma
  4: identical tokens and accepted counts per round, with a prefix draft
  (the target's first layer, accepting some rounds) with and without the
  bonus token, and with an unrelated seed-1 draft;
* the same at 8 concurrent requests (prompts of 5..64 tokens, 16 new).
"""
import numpy as np
import pytest

import modelc_b200 as mb
import shape_models as sm
import oracle as o

pytestmark = pytest.mark.gpu

CFG = mb.LLAMA3_8B.with_layers(2)
DCFG = CFG.with_layers(1)


@pytest.fixture(scope="module")
def models():
    tw = sm.host_weights(CFG, seed=0, fmt="i8_row")
    rw = sm.host_weights(DCFG, seed=1, fmt="i8_row")
    deq = sm.Dequant()
    W = mb.Weights(tw, CFG)
    prefix = sm.prefix_draft(tw)
    D = {"prefix": mb.Weights(prefix, DCFG), "random": mb.Weights(rw, DCFG)}
    ot = sm.oracle_model(tw, CFG, deq)
    od = {"prefix": sm.oracle_model(prefix, DCFG, deq), "random": sm.oracle_model(rw, DCFG, deq)}
    yield W, D, ot, od
    for x in (W, *D.values()):
        x.close()


def test_8b_width_forward_logits(models):
    W, _, ot, _ = models
    ids = np.random.default_rng(7).integers(0, CFG.vocab, 38).tolist()
    ref = ot.forward_ids(ids, ot.new_kv(64))
    s = mb.Session(W, None, gamma=4, max_context=64)
    got = np.concatenate([s.forward(ids[:33]), s.forward(ids[33:])])
    s.close()
    margin, err = sm.logits_report(got, ref)
    print(f"8B width: min top-1/top-2 margin {margin:.3e}, max rel error {err:.3e}")


@pytest.mark.parametrize("draft,bonus", [("prefix", False), ("prefix", True), ("random", False)])
def test_8b_width_spec_decode(models, draft, bonus):
    W, D, ot, od = models
    prompt = np.random.default_rng(2).integers(0, CFG.vocab, 64).tolist()
    ref, racc = ot.speculative_generate(prompt, 32, 4, o.OracleLlamaDraft(od[draft], 160),
                                        bonus=bonus)
    s = mb.Session(W, D[draft], gamma=4, max_context=160, bonus=bonus)
    got, gacc = s.speculative_generate(prompt, 32)
    s.close()
    assert got == ref
    assert gacc == racc
    if draft == "prefix":
        print(f"8B width prefix draft, bonus={bonus}: accepted per round {gacc}")


def test_8b_width_batch8_spec_decode(models):
    W, D, ot, od = models
    rng = np.random.default_rng(11)
    prompts = [rng.integers(0, CFG.vocab, n).tolist() for n in (13, 7, 30, 21, 5, 17, 9, 64)]
    refs = [ot.speculative_generate(p, 16, 4, o.OracleLlamaDraft(od["prefix"], 128))
            for p in prompts]
    s = mb.Session(W, D["prefix"], gamma=4, max_context=128, n_requests=8)
    got = s.speculative_generate_batch(prompts, 16)
    s.close()
    for z, ((gt, gacc), (rt, racc)) in enumerate(zip(got, refs)):
        assert gt == rt, z
        assert gacc == racc, z
