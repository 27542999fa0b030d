"""bench.py's workload table against the benchmark's configurations (CPU).

Each named workload must carry the shapes, formats, seeds and run lengths of
the configuration it stands for, and the default must be the headline
(Llama-3-8B shape, int8 rows, batch 1).  The flags the multi-GPU runs use
must parse.  Nothing here touches a GPU.
"""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
import bench  # noqa: E402


def _shape(c):
    r = c.resolved()
    return (r.n_layers, r.hidden, r.n_heads, r.n_kv_heads, r.head_dim, r.ffn, r.vocab)


# (layers, d_model, heads, kv heads, head_dim, ffn, vocab), target then draft
SHAPES = {
    "tiny": ((4, 256, 4, 4, 64, 688, 4096), (1, 256, 4, 4, 64, 688, 4096)),
    "tinyllama": ((22, 2048, 32, 4, 64, 5632, 32000), (2, 2048, 32, 4, 64, 5632, 32000)),
    "llama3-8b": ((32, 4096, 32, 8, 128, 14336, 128256), (2, 4096, 32, 8, 128, 14336, 128256)),
    "llama3-8b-bs8": ((32, 4096, 32, 8, 128, 14336, 128256),
                      (2, 4096, 32, 8, 128, 14336, 128256)),
    # the 70B's draft is the 8B-shape int8 model over the target's vocabulary
    "llama2-70b": ((80, 8192, 64, 8, 128, 28672, 32000), (32, 4096, 32, 8, 128, 14336, 32000)),
}
# (target fmt, draft fmt, prompt, new tokens, gamma, temperature, seed, batch)
RUNS = {
    "tiny": ("i8_row", "i8_row", 32, 128, 4, 0.0, 0, 1),
    "tinyllama": ("q4_0", "q4_0", 512, 256, 5, 0.8, 7, 1),
    "llama3-8b": ("i8_row", "i8_row", 1024, 256, 4, 0.0, 0, 1),
    "llama3-8b-bs8": ("i8_row", "i8_row", 1024, 256, 4, 0.0, 0, 8),
    "llama2-70b": ("q4_0", "i8_row", 2048, 256, 4, 0.0, 0, 1),
}


@pytest.mark.parametrize("name", sorted(SHAPES))
def test_workload_matches_configuration(name):
    wl = bench.workloads()[name]
    assert (_shape(wl.target), _shape(wl.draft)) == SHAPES[name]
    assert (wl.fmt, wl.draft_fmt, wl.prompt_len, wl.new_tokens, wl.gamma, wl.temperature,
            wl.seed, wl.batch) == RUNS[name]
    assert wl.accept_mode == 0  # min(1, p/q) when stochastic


def test_rope_and_norm_constants():
    w = bench.workloads()
    assert w["llama3-8b"].target.rope_theta == 500000.0
    assert w["tinyllama"].target.rope_theta == 10000.0
    # the tiny model runs in the reference's own mode: heads = d / 64, eps 1e-6
    from modelc_b200.model import MODE_REFERENCE
    assert w["tiny"].target.mode == MODE_REFERENCE


def test_headline_is_the_default(monkeypatch):
    seen = {}
    monkeypatch.setattr(bench, "run_ours", lambda a: seen.setdefault("args", a))
    monkeypatch.setattr(sys, "argv", ["bench.py"])
    bench.main()
    a = seen["args"]
    assert (a.config, a.gpus, a.impl, a.replicas, a.tp_nccl) == ("llama3-8b", 1, "ours", False,
                                                                 False)
    assert a.warmup >= 3
    assert bench.workloads()[a.config].metric == bench.METRIC


def test_warmup_is_raised_to_three_and_multi_gpu_flags_parse(monkeypatch):
    seen = {}
    monkeypatch.setattr(bench, "run_ours", lambda a: seen.setdefault("args", a))
    monkeypatch.setattr(sys, "argv", ["bench.py", "--gpus", "8", "--steps", "2", "--warmup", "1",
                                      "--replicas", "--tp-nccl", "--config", "llama2-70b"])
    bench.main()
    a = seen["args"]
    assert (a.gpus, a.steps, a.warmup, a.replicas, a.tp_nccl, a.config) == (8, 2, 3, True, True,
                                                                          "llama2-70b")
