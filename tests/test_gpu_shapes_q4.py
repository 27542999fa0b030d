"""Parity at the q4_0 benchmark widths: TinyLlama-1.1B (2 layers) and
Llama-2-70B (1 layer).

TinyLlama width: d 2048, 32 query / 4 KV heads of head_dim 64 (8 query rows
per KV head), FFN 5632, vocab 32000, q4_0 weights.  Checked: forward logits
against the oracle within 1e-3, and stochastic speculative decoding at
temperature 0.8 with min(1, p/q) acceptance, gamma 5 and Philox seed 7 (the
TinyLlama benchmark's settings) token for token against the oracle's
restatement with the same random stream, with a prefix draft and with an
unrelated 2-layer draft.

70B width: d 8192, 64 query / 8 KV heads of head_dim 128, FFN 28672, vocab
32000, q4_0 weights, one layer.  Checked: forward logits, and greedy
speculative decoding with gamma 4 and the benchmark's draft shape (an 8B-width
int8 model with vocab 32000, here one layer): identical tokens and accepted
counts.
"""
from dataclasses import replace

import numpy as np
import pytest

import modelc_b200 as mb
import shape_models as sm
import oracle as o

pytestmark = pytest.mark.gpu

TL = mb.TINYLLAMA.with_layers(2)
BIG = mb.LLAMA2_70B.with_layers(1)
BIG_DRAFT = replace(mb.LLAMA3_8B, vocab=32000).with_layers(1)


@pytest.fixture(scope="module")
def tinyllama():
    tw = sm.host_weights(TL, seed=0, fmt="q4_0")
    rw = sm.host_weights(TL, seed=1, fmt="q4_0")
    deq = sm.Dequant()
    prefix = sm.prefix_draft(tw)
    dcfg = TL.with_layers(1)
    W = mb.Weights(tw, TL)
    D = {"prefix": (mb.Weights(prefix, dcfg), sm.oracle_model(prefix, dcfg, deq)),
         "random": (mb.Weights(rw, TL), sm.oracle_model(rw, TL, deq))}
    yield W, D, sm.oracle_model(tw, TL, deq)
    W.close()
    for w, _ in D.values():
        w.close()


def test_tinyllama_width_q4_forward_logits(tinyllama):
    W, _, ot = tinyllama
    ids = np.random.default_rng(5).integers(0, TL.vocab, 26).tolist()
    ref = ot.forward_ids(ids, ot.new_kv(64))
    s = mb.Session(W, None, gamma=5, max_context=64)
    got = np.concatenate([s.forward(ids[:20]), s.forward(ids[20:])])
    s.close()
    margin, err = sm.logits_report(got, ref)
    print(f"TinyLlama width q4_0: min top-1/top-2 margin {margin:.3e}, max rel error {err:.3e}")


@pytest.mark.parametrize("draft", ["prefix", "random"])
def test_tinyllama_width_q4_stochastic(tinyllama, draft):
    W, D, ot = tinyllama
    Dw, od = D[draft]
    prompt = np.random.default_rng(2).integers(0, TL.vocab, 48).tolist()
    ref, racc = ot.speculative_sample(prompt, 40, 5, o.OracleLlamaDraft(od, 128), 0.8, 7,
                                      accept_mode=0)
    s = mb.Session(W, Dw, gamma=5, max_context=128, temperature=0.8, seed=7, accept_mode=0)
    got, gacc = s.speculative_generate(prompt, 40)
    s.close()
    assert got == ref
    assert gacc == racc
    print(f"TinyLlama width, {draft} draft, T=0.8: accepted per round {gacc}")


@pytest.fixture(scope="module")
def llama70():
    tw = sm.host_weights(BIG, seed=0, fmt="q4_0")
    dw = sm.host_weights(BIG_DRAFT, seed=1, fmt="i8_row")
    deq = sm.Dequant()
    W, D = mb.Weights(tw, BIG), mb.Weights(dw, BIG_DRAFT)
    yield W, D, sm.oracle_model(tw, BIG, deq), sm.oracle_model(dw, BIG_DRAFT, deq)
    W.close()
    D.close()


def test_70b_width_q4_forward_logits(llama70):
    W, _, ot, _ = llama70
    ids = np.random.default_rng(9).integers(0, BIG.vocab, 21).tolist()
    ref = ot.forward_ids(ids, ot.new_kv(64))
    s = mb.Session(W, None, gamma=4, max_context=64)
    got = np.concatenate([s.forward(ids[:17]), s.forward(ids[17:])])
    s.close()
    margin, err = sm.logits_report(got, ref)
    print(f"70B width q4_0: min top-1/top-2 margin {margin:.3e}, max rel error {err:.3e}")


def test_70b_width_q4_greedy_spec_decode(llama70):
    W, D, ot, od = llama70
    prompt = np.random.default_rng(2).integers(0, BIG.vocab, 40).tolist()
    ref, racc = ot.speculative_generate(prompt, 16, 4, o.OracleLlamaDraft(od, 96))
    s = mb.Session(W, D, gamma=4, max_context=96)
    got, gacc = s.speculative_generate(prompt, 16)
    s.close()
    assert got == ref
    assert gacc == racc
