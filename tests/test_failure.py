"""Failure paths that can be exercised without faulting a GPU.

* Cancellation (generate.rs:639 checks a cancel flag between rounds): the
  session's flag, raised before a decode or while one runs, ends it with
  MC_E_CANCELLED; the rounds already run are kept and are the same tokens an
  uncancelled run produces, and after the flag is lowered the session
  rewinds and decodes as usual.
* A tensor-parallel peer that never arrives: rank 0 of a two-rank fused
  exchange runs alone on one GPU.  Rank 1's session exists (its exchange
  buffer is real memory of this process, opened directly) but never
  launches anything, so nothing ever sets its flags.  Rank 0's bounded wait
  (200 ms here) expires: the call returns MC_E_TIMEOUT, the session stays
  failed, and the CUDA context remains usable (a fresh model still matches
  the oracle).  No NCCL call is involved, so no wait is unbounded.
"""
import os
import sys
import threading
import time

import numpy as np
import pytest

sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "oracle"))
import oracle as o  # noqa: E402

import modelc_b200 as mb  # noqa: E402
from modelc_b200.model import LlamaConfig, MODE_GENERAL, MODE_REFERENCE  # noqa: E402

pytestmark = pytest.mark.gpu

SMALL_REF = LlamaConfig(2, 128, 2, 2, 64, 160, 300, mode=MODE_REFERENCE, name="small-ref")
TP2 = LlamaConfig(2, 128, 4, 2, 32, 192, 260, 500000.0, 1e-5, MODE_GENERAL, "tp2-gqa")
MC_E_TIMEOUT, MC_E_CANCELLED = -7, -8


def _pair(cfg):
    tw = mb.synth_weights(cfg, seed=0)
    dw = mb.synth_weights(cfg.with_layers(1), seed=1)
    return mb.Weights(tw, cfg), mb.Weights(dw, cfg.with_layers(1)), tw


def test_cancel_before_decode_then_resume():
    W, D, _ = _pair(SMALL_REF)
    prompt = list(range(3, 20))
    ref = mb.Session(W, D, gamma=3, max_context=160)
    ref.prime(prompt)
    ref.decode(40)
    want = ref.read()
    ref.close()
    s = mb.Session(W, D, gamma=3, max_context=160)
    s.prime(prompt)
    s.cancel()
    with pytest.raises(mb.McError) as e:
        s.decode(40)
    assert e.value.status == MC_E_CANCELLED
    assert s.read() == ([], [])  # nothing ran
    s.uncancel()
    s.decode(40)
    assert s.read() == want
    s.close()


DEEP = LlamaConfig(24, 256, 4, 2, 64, 512, 1024, 10000.0, 1e-5, MODE_GENERAL, "deep")


def test_cancel_while_decoding_keeps_a_prefix():
    # 24 target layers: each round takes long enough that the decode of 3900
    # tokens is still running when the flag goes up
    W, D, _ = _pair(DEEP)
    prompt = list(range(5, 30))
    n_max = 3900
    s = mb.Session(W, D, gamma=4, max_context=n_max + 64)
    s.prime(prompt)
    result = {}

    def run():
        try:
            result["n"] = s.decode(n_max)
        except mb.McError as e:
            result["status"] = e.status

    t = threading.Thread(target=run)
    t.start()
    time.sleep(0.5)
    s.cancel()
    t.join(timeout=300)
    assert not t.is_alive()
    toks, acc = s.read(cap=n_max + 16)
    if result.get("status") != MC_E_CANCELLED:  # finished before the flag: nothing to check
        pytest.skip(f"decode finished before the cancel ({len(toks)} tokens)")
    assert 0 < len(toks) < n_max
    # the kept rounds are those of an uncancelled run
    s.uncancel()
    s.rewind()
    s.decode(len(toks))
    again, acc2 = s.read(cap=n_max + 16)
    assert again[:len(toks)] == toks
    assert acc2[:len(acc)] == acc
    s.close()


def test_tp_peer_that_never_arrives_times_out():
    tw = mb.synth_weights(TP2, seed=0)
    shards = [mb.Weights(tw, TP2, device=0, tp_rank=r, tp_world=2) for r in range(2)]
    sessions = [mb.Session(w, None, gamma=4, max_context=64) for w in shards]
    handles = [s.tp_ipc_handle() for s in sessions]
    s0 = sessions[0]
    s0.tp_open_peers(handles)  # rank 1 is a session of this process: opened directly
    s0.set_wait_timeout(200)
    ids = np.random.default_rng(3).integers(0, TP2.vocab, 9).tolist()
    t0 = time.time()
    with pytest.raises(mb.McError) as e:
        s0.forward(ids, logits=False)
    took = time.time() - t0
    assert e.value.status == MC_E_TIMEOUT, e.value
    assert took < 30, took  # one expired wait; the later ones give up at once
    with pytest.raises(mb.McError) as e:  # the session stays failed
        s0.forward(ids[:1], logits=False)
    assert e.value.status == MC_E_TIMEOUT
    for s in sessions:
        s.close()
    for w in shards:
        w.close()
    # the context is still usable: a fresh model matches the oracle
    cfg = SMALL_REF
    ws = mb.synth_weights(cfg, seed=4)
    c = cfg.resolved()
    om = o.OracleModel({k: v.dequant() for k, v in ws.items()}, c.n_layers, c.hidden, c.vocab,
                       c.ffn, mode=cfg.mode)
    ref = om.forward_ids(ids, om.new_kv(32))
    s = mb.Session(mb.Weights(ws, cfg), None, gamma=1, max_context=32)
    got = s.forward(ids)
    s.close()
    err = np.abs(got - ref).max(axis=1)
    assert (err <= 1e-3 * np.abs(ref).max(axis=1)).all()


def test_context_beyond_the_attention_limit_is_rejected():
    W, D, _ = _pair(SMALL_REF)
    s = mb.Session(W, D, gamma=2, max_context=4030)
    s.close()
    with pytest.raises(mb.McError) as e:
        mb.Session(W, D, gamma=2, max_context=4031)
    assert e.value.status == -10


def test_wait_timeout_rejects_bad_values():
    W, D, _ = _pair(SMALL_REF)
    s = mb.Session(W, D, gamma=2, max_context=32)
    with pytest.raises(mb.McError):
        s.set_wait_timeout(0)
    s.set_wait_timeout(50)
    s.close()
