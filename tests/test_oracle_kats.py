"""The reference's own known-answer tests, run against the C oracle.

Each test cites the reference test it restates (paths inside yingkitw/modelc).
"""
import math
import os
import sys

import numpy as np
import pytest

sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(__file__)), "oracle"))
import oracle as o  # noqa: E402


def test_silu_known_values():  # transformer.rs:1042-1046
    s = o.silu([0.0, 1.0])
    assert abs(s[0]) < 1e-6
    assert abs(s[1] - (1.0 / (1.0 + math.exp(-1.0)))) < 1e-6


def test_rms_norm_positive():  # transformer.rs:1058-1064
    y = o.rms_norm([1.0, 2.0, 3.0, 4.0], [1.0] * 4, 1e-6)
    assert (y > 0).all()


def test_rope_at_zero_is_identity():  # transformer.rs:1067-1073
    x = np.arange(12, dtype=np.float32)
    y = o.rope(x, 0, 2)
    assert np.all(np.abs(x - y) < 1e-5)


def test_add_is_elementwise():  # transformer.rs:1076-1081
    assert o.add([1.0, 2.0, 3.0], [10.0, 20.0, 30.0]).tolist() == [11.0, 22.0, 33.0]


def test_attention_single_token_is_identity():  # transformer.rs:1084-1091
    out = o.attention_kv([1.0, 2.0], [1.0, 2.0], [0.5, 0.25], 1)
    assert out.tolist() == [0.5, 0.25]


def test_attention_two_tokens():  # transformer.rs:1094-1114
    out = o.attention_kv([0.0, 1.0], [1.0, 0.0, 0.0, 1.0], [1.0, 0.0, 0.0, 1.0], 1)
    assert 0.2 < out[0] < 0.4 and 0.6 < out[1] < 0.8


def test_attention_multi_head_finite():  # transformer.rs:1348-1364
    nh, hd, seq = 4, 8, 16
    q = np.arange(nh * hd, dtype=np.float32) * 0.1
    k = np.arange(seq * nh * hd, dtype=np.float32) * 0.05
    v = np.arange(seq * nh * hd, dtype=np.float32) * 0.03
    out = o.attention_kv(q, k, v, nh)
    assert out.shape == (nh * hd,) and np.isfinite(out).all()


def test_kv_cache_appends_and_reuses():  # transformer.rs:1117-1134
    m = o.OracleModel({}, 0, 2, 1, 1, mode=o.MODE_GENERAL, n_heads=1, n_kv_heads=1,
                      head_dim=2)
    kv = m.new_kv(4)
    assert len(kv) == 0


def test_softmax_inplace_matches_softmax():  # transformer.rs:1336-1345
    xs = [1.0, 2.0, 3.0, 4.0]
    a = o.softmax_inplace(xs)
    e = o.softmax(xs)
    assert np.all(np.abs(a - e) < 1e-6)


def test_argmax_picks_max():  # generate.rs:1131-1133
    assert o.argmax([1.0, 3.0, 2.0]) == 1


def test_argmax_first_of_ties_and_nan():  # generate.rs:1088-1098 rule
    assert o.argmax([2.0, 5.0, 5.0, 1.0]) == 1
    assert o.argmax([float("nan"), 1.0]) == 1
    assert o.argmax([float("nan")] * 3) == 0


def test_softmax_sums_to_one():  # generate.rs:1136-1140
    assert abs(float(np.sum(o.softmax([1.0, 2.0, 3.0]))) - 1.0) < 1e-5


def test_greedy_sample_picks_argmax():  # generate.rs:1143-1150
    assert o.sample([1.0, 5.0, 2.0], 0.0, 0, 0) == 1


def test_top_p_keeps_nucleus():  # generate.rs:1153-1162
    p = o.apply_top_p([0.5, 0.3, 0.15, 0.05], 0.8)
    assert abs(p[2]) < 1e-6 and abs(p[3]) < 1e-6
    assert abs(float(p.sum()) - 1.0) < 1e-5


def test_top_p_high_keeps_all():  # generate.rs:1165-1171
    p = o.apply_top_p([0.4, 0.3, 0.2, 0.1], 0.99)
    assert abs(float(p.sum()) - 1.0) < 1e-5 and (p > 0).all()


def test_min_p_drops_low():  # generate.rs:1174-1199
    p = o.apply_min_p([0.5, 0.2, 0.15, 0.15], 0.5)
    assert abs(p[1]) < 1e-6 and abs(p[2]) < 1e-6 and abs(p[3]) < 1e-6
    assert abs(float(p.sum()) - 1.0) < 1e-5


def test_min_p_keeps_above_threshold():  # generate.rs:1202-1222
    p = o.apply_min_p([0.4, 0.3, 0.2, 0.1], 0.5)
    assert p[0] > 0 and p[1] > 0 and p[2] > 0 and abs(p[3]) < 1e-6
    assert abs(float(p.sum()) - 1.0) < 1e-5


def test_min_p_zero_is_noop():  # generate.rs:1225-1231
    x = np.array([0.5, 0.3, 0.2], np.float32)
    assert (o.apply_min_p(x, 0.0) == x).all()


def test_ngram_index_trigrams():  # generate.rs:1234-1240 via draft_tokens
    t = [1, 2, 3, 1, 2, 4]
    assert o.ngram_draft(t, [1, 2, 3], 1) == [1]
    assert o.ngram_draft(t, [2, 3, 1], 1) == [2]
    assert o.ngram_draft(t, [3, 1, 2], 1) == [4]


def test_ngram_draft_continues():  # generate.rs:1243-1250
    t = [1, 2, 3, 1, 2, 4, 1, 2, 3, 5]
    assert len(o.ngram_draft(t, [1, 2, 3], 2)) > 0


def test_ngram_draft_stops_without_match():  # generate.rs:1253-1258
    assert o.ngram_draft([1, 2, 3, 4], [9, 9, 9], 3) == []


def test_ngram_most_frequent_mode():  # generate.rs:1261-1265 most_frequent
    # context [7,7,7] followed by 1,2,2,3,2 -> mode 2
    t = [7, 7, 7, 1, 7, 7, 7, 2, 7, 7, 7, 2, 7, 7, 7, 3, 7, 7, 7, 2]
    assert o.ngram_draft(t, [7, 7, 7], 1) == [2]


def test_multinomial_same_seed_deterministic():  # generate.rs:1345-1352
    p = [0.1, 0.2, 0.3, 0.4]
    assert o.multinomial(p, 0, 42) == o.multinomial(p, 0, 42)


def test_multinomial_different_step_differs():  # generate.rs:1355-1366
    p = [0.1, 0.2, 0.3, 0.4]
    assert o.multinomial(p, 0, 42) != o.multinomial(p, 1, 42)


def test_sample_with_seed_deterministic():  # generate.rs:1369-1382
    assert o.sample([1.0, 2.0, 3.0], 1.0, 0, 123) == o.sample([1.0, 2.0, 3.0], 1.0, 0, 123)


def test_chacha20_rfc8439_vectors():
    # The ChaCha core (rand_chacha 0.3.1 ChaCha12Rng uses it with 12 rounds):
    # RFC 8439 A.1 test vectors #1 and #2 (all-zero key and nonce).
    b0 = o.chacha_block([0] * 8, 0, 0, 20)
    assert [hex(x) for x in b0[:4]] == ["0xade0b876", "0x903df1a0", "0xe56a5d40", "0x28bd8653"]
    assert hex(b0[15]) == "0x8665eeb2"
    b1 = o.chacha_block([0] * 8, 1, 0, 20)
    assert hex(b1[0]) == "0xbee7079f"


def test_rand_f32_in_unit_interval():
    rs = [o.lib().oracle_rand_f32(s) for s in range(200)]
    assert all(0.0 <= r < 1.0 for r in rs)
    assert 0.35 < float(np.mean(rs)) < 0.65


def test_mlp_draft_greedy_kat():  # draft.rs:162-221 -> [2, 2, 2]
    emb = np.array([1, 0, 0, 1, 1, 1, 0, 0], np.float32).reshape(4, 2)
    w1 = np.array([1, 0, 0, 1], np.float32).reshape(2, 2)
    b1 = np.zeros(2, np.float32)
    w2 = np.array([0, 0, 0, 0, 1, 0, 0, 0], np.float32).reshape(4, 2)
    b2 = np.zeros(4, np.float32)
    d = o.OracleMlpDraft(emb, w1, b1, w2, b2)
    assert d.draft([0], 3) == [2, 2, 2]


def test_q4_0_length_and_values():  # runtime/serve.rs:187-205 + dequant.rs:23-46
    blk = np.zeros(18, np.uint8)
    blk[0:2] = np.frombuffer(np.float16(1.0).tobytes(), np.uint8)
    blk[2:] = 0x88
    y = o.dequant_q4_0(blk, 32)
    assert len(y) == 32 and (y == 0).all()
    blk[2] = 0x9F  # lo nibble 15 -> 7*d ; hi nibble 9 -> 1*d
    y = o.dequant_q4_0(blk, 32)
    assert y[0] == 7.0 and y[16] == 1.0


def test_q4_0_roundtrip_error_bound():
    x = np.random.default_rng(3).standard_normal(32 * 64).astype(np.float32)
    y = o.dequant_q4_0(o.quantize_q4_0(x), x.size)
    blocks = x.reshape(-1, 32)
    amax = np.abs(blocks).max(1, keepdims=True)
    # step = amax/8; the end opposite the largest magnitude clips at +7 steps
    assert (np.abs(y.reshape(-1, 32) - blocks) <= amax / 8 * 1.001).all()


def test_int8_tensor_quantizer_rule():  # compiler.rs:207-229
    x = np.array([0.5, -1.0, 0.25, 0.0], np.float32)
    q, s = o.quantize_int8_tensor(x)
    assert s == np.float32(1.0) / np.float32(127.0)
    assert q.tolist() == [64, -127, 32, 0]  # 63.5 rounds half away from zero
    z, s0 = o.quantize_int8_tensor(np.zeros(4, np.float32))
    assert s0 == 0.0 and (z == 0).all()


def test_f16_conversions():
    for v in (0.0, 1.0, -2.5, 65504.0, 6.1035156e-05):
        assert o.lib().oracle_f16_to_f32(o.lib().oracle_f32_to_f16(v)) == np.float32(v)
