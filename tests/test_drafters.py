"""The reference's small drafters on the device, against the oracle.

MlpDraftModel (draft.rs:28-147): embedding row -> FC1 + bias -> ReLU -> FC2 +
bias -> argmax.  The device sums every output row in the reference's order
(bias, then j ascending, separate multiply and add), so its greedy drafts
equal the oracle's token for token, ties and all.  Temperature > 0 is not
offered: the reference samples from an unseeded generator there.

n-gram drafter (generate.rs:771-841): draft_tokens over build_ngram_index of
the token history, as speculative_generate calls it (the history is both the
index and the lookup context).  The reference breaks count ties by HashMap
iteration order; the device and the oracle both take the continuation seen
first, and the small-vocabulary cases below are full of such ties.
"""
import os
import sys

import numpy as np
import pytest

sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "oracle"))
import oracle as o  # noqa: E402

import modelc_b200 as mb  # noqa: E402

pytestmark = pytest.mark.gpu


def _mlp_tensors(V, d, dh, seed, embed_name="draft.embed.weight"):
    rng = np.random.default_rng(seed)
    f = lambda *s: rng.standard_normal(s, dtype=np.float32)  # noqa: E731
    return {embed_name: f(V, d), "draft.fc1.weight": f(dh, d) * np.float32(0.1),
            "draft.fc1.bias": f(dh) * np.float32(0.1), "draft.fc2.weight": f(V, dh),
            "draft.fc2.bias": f(V) * np.float32(0.1)}


def _oracle_mlp(t, embed_name="draft.embed.weight"):
    return o.OracleMlpDraft(t[embed_name], t["draft.fc1.weight"], t["draft.fc1.bias"],
                            t["draft.fc2.weight"], t["draft.fc2.bias"])


def test_mlp_draft_reference_kat():  # draft.rs:162-221 -> [2, 2, 2]
    t = {"draft.embed.weight": np.array([1, 0, 0, 1, 1, 1, 0, 0], np.float32).reshape(4, 2),
         "draft.fc1.weight": np.array([1, 0, 0, 1], np.float32).reshape(2, 2),
         "draft.fc1.bias": np.zeros(2, np.float32),
         "draft.fc2.weight": np.array([0, 0, 0, 0, 1, 0, 0, 0], np.float32).reshape(4, 2),
         "draft.fc2.bias": np.zeros(4, np.float32)}
    d = mb.MlpDraftModel(t)
    assert d.draft([0], 3) == [2, 2, 2]
    d.close()


@pytest.mark.parametrize("V,d,dh", [(300, 128, 64), (4096, 256, 64), (32000, 2048, 64),
                                    (1000, 100, 7)])
def test_mlp_draft_matches_oracle(V, d, dh):
    t = _mlp_tensors(V, d, dh, seed=V + d)
    dev, ref = mb.MlpDraftModel(t), _oracle_mlp(t)
    rng = np.random.default_rng(1)
    contexts = [[int(x)] for x in rng.integers(0, V, 6)] + [
        rng.integers(0, V, 20).tolist(), [], [V + 3], [V - 1]]
    for ctx in contexts:
        for gamma in (1, 4, 16):
            assert dev.draft(ctx, gamma) == ref.draft(ctx, gamma), (ctx[-1:], gamma)
    dev.close()


def test_mlp_draft_borrows_target_embedding_and_rejects_bad_input():
    t = _mlp_tensors(500, 64, 16, seed=3, embed_name="model.embed_tokens.weight")
    d = mb.MlpDraftModel(t)
    assert d.draft([7, 9], 5) == _oracle_mlp(t, "model.embed_tokens.weight").draft([7, 9], 5)
    with pytest.raises(mb.McError):  # at most 16 steps
        d.draft([1], 17)
    d.close()
    bad = dict(t)
    del bad["draft.fc2.bias"]
    with pytest.raises(mb.McError):
        mb.MlpDraftModel(bad)
    bad = dict(t)
    bad["draft.fc1.weight"] = bad["draft.fc1.weight"][:, :10]
    with pytest.raises(mb.McError):
        mb.MlpDraftModel(bad)


KAT_STREAMS = [
    [1, 2, 3, 1, 2, 4, 1, 2, 3],                  # generate.rs:1234-1240 pattern
    [1, 2, 3, 1, 2, 4, 1, 2, 3, 5, 1, 2, 3],      # generate.rs:1243-1250 pattern
    [1, 2, 3, 4, 9, 9, 9],                        # generate.rs:1253-1258: no match
    [7, 7, 7, 1, 7, 7, 7, 2, 7, 7, 7, 2, 7, 7, 7, 3, 7, 7, 7, 2, 7, 7, 7],  # most_frequent
]


@pytest.mark.parametrize("stream", KAT_STREAMS)
@pytest.mark.parametrize("n", [1, 2, 3])
def test_ngram_draft_reference_patterns(stream, n):
    d = mb.NgramDraftModel(n=n, max_tokens=256)
    for gamma in (1, 3, 8):
        assert d.draft(stream, gamma) == o.ngram_draft(stream, stream, gamma, n), gamma
    d.close()


@pytest.mark.parametrize("vocab,length", [(3, 40), (5, 300), (50, 2000), (4, 4096)])
@pytest.mark.parametrize("n", [1, 2, 3, 4])
def test_ngram_draft_matches_oracle_random(vocab, length, n):
    rng = np.random.default_rng(vocab * 1000 + length + n)
    d = mb.NgramDraftModel(n=n, max_tokens=4096)
    for trial in range(3):
        s = rng.integers(0, vocab, length).tolist()
        for gamma in (1, 4, 16):
            assert d.draft(s, gamma) == o.ngram_draft(s, s, gamma, n), (trial, gamma)
    assert d.draft([], 4) == []
    assert d.draft([1, 2], 4) == o.ngram_draft([1, 2], [1, 2], 4, n)
    with pytest.raises(mb.McError):  # history above max_tokens
        d.draft(list(range(4097)), 2)
    d.close()
