"""Encoding tails against separate encoder launches.

An encoding tail runs the next encoder inside the kernel that produced its
input: after its epilogues the grid meets at a bounded barrier and each CTA
encodes a slice of k-blocks.  Bit 0 of MODELC_CUDA_ENCODER_TAILS (read at
session creation) gives the o, gate/up and down GEMVs of one token group
their tails (GemvArgs::bar), bit 1 the tensor-core attention with one
m-tile whose grid is one wave (AttnArgs::bar: the O projection's page
combine and encoding).  The digits are those the separate k_quant /
k_quant_att launches write, so every forward must be bit for bit the same
under every mask, at the small test widths, at the Llama-3-8B widths (int8)
and at the TinyLlama widths (q4_0); and a round graph must hold exactly the
launches the mask removes.
"""
import os

import numpy as np
import pytest

import modelc_b200 as mb
import shape_models as sm
from modelc_b200.model import LlamaConfig, MODE_GENERAL, MODE_REFERENCE

pytestmark = pytest.mark.gpu

SMALL_REF = LlamaConfig(2, 128, 2, 2, 64, 160, 300, mode=MODE_REFERENCE, name="small-ref")
SMALL_GQA = LlamaConfig(2, 128, 4, 2, 32, 176, 260, 500000.0, 1e-5, MODE_GENERAL, "small-gqa")
MID_GQA = LlamaConfig(3, 512, 8, 2, 64, 1024, 2048, 500000.0, 1e-5, MODE_GENERAL, "mid-gqa")
ENV = "MODELC_CUDA_ENCODER_TAILS"


def _session(mask, *args, **kw):
    old = os.environ.get(ENV)
    os.environ[ENV] = str(mask)
    try:
        return mb.Session(*args, **kw)
    finally:
        if old is None:
            del os.environ[ENV]
        else:
            os.environ[ENV] = old


def _chunked_forward(W, ids, mask, chunks=(5, 1, 7, 16, 3)):
    s = _session(mask, W, None, gamma=4, max_context=64)
    out, i = [], 0
    for c in chunks:
        out.append(s.forward(ids[i:i + c]))
        i += c
    s.close()
    return np.concatenate(out)


@pytest.mark.parametrize("cfg", [SMALL_REF, SMALL_GQA, MID_GQA], ids=lambda c: c.name)
def test_small_widths_forward_bit_identical(cfg):
    W = mb.Weights(mb.synth_weights(cfg, seed=3), cfg)
    ids = np.random.default_rng(1).integers(0, cfg.vocab, 32).tolist()
    off = _chunked_forward(W, ids, 0)
    for mask in (1, 2, 3):
        assert np.array_equal(_chunked_forward(W, ids, mask), off), mask
    W.close()


@pytest.mark.parametrize("base,fmt", [(mb.LLAMA3_8B, "i8_row"), (mb.TINYLLAMA, "q4_0")],
                         ids=["8b-int8", "tinyllama-q4_0"])
def test_benchmark_widths_forward_and_decode_bit_identical(base, fmt):
    cfg = base.with_layers(2)
    tw = sm.host_weights(cfg, seed=0, fmt=fmt)
    W = mb.Weights(tw, cfg)
    D = mb.Weights(sm.prefix_draft(tw), cfg.with_layers(1))
    ids = np.random.default_rng(2).integers(0, cfg.vocab, 32).tolist()
    assert np.array_equal(_chunked_forward(W, ids, 3), _chunked_forward(W, ids, 0))
    prompt = ids[:20]
    runs = []
    for mask in (3, 0):
        s = _session(mask, W, D, gamma=4, max_context=96)
        runs.append(s.speculative_generate(prompt, 24))
        s.close()
    assert runs[0] == runs[1]
    W.close()
    D.close()


@pytest.mark.parametrize("mask", [0, 1, 2, 3])
def test_round_graph_launch_counts(mask):
    # per forward without tails: embedding, then per layer the attention
    # encoder, qkv, attention, O encoder, o, MLP encoder, gate/up, SwiGLU
    # encoder, down, then the final encoder and the LM head; the GEMV tails
    # take three encoders per layer, the attention tail one
    cfg = SMALL_GQA.with_layers(3)
    W = mb.Weights(mb.synth_weights(cfg, seed=0), cfg)
    D = mb.Weights(mb.synth_weights(cfg.with_layers(1), seed=1), cfg.with_layers(1))
    gamma, prompt = 3, list(range(1, 12))

    def fwd(L):
        return 3 + (9 - 3 * (mask & 1) - (mask >> 1 & 1)) * L

    s = _session(mask, W, D, gamma=gamma, max_context=64)
    s.prime(prompt)
    s.decode(4)
    want = gamma * fwd(1) + fwd(3) + 1  # draft steps, verify, acceptance
    assert s.round_launches == want, (s.round_launches, want)
    s.close()
    W.close()
    D.close()
