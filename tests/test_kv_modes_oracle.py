"""The oracle's KvLayer variants and context shift against the reference's
own tests (CPU).

transformer.rs:1135-1336 test the FP32 / INT8 / MIXED layers: append,
k_all, shift and shift_anchored; the exact expectations are restated here
(a one-layer OracleKV with kv_dim 2 or 4), the tolerance ones with their
tolerances.  generate.rs:26-63 context_shift has no test of its own in the
reference; its arithmetic is checked on hand-worked cases.
"""
import os
import sys

import numpy as np

sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "oracle"))
import oracle as o  # noqa: E402


def _layer(mode, dim, window=64, cap=16):
    kv = o.OracleKV(None, cap, n_layers=1, kv_dim=dim)
    kv.set_mode(mode, window)
    return kv


def _k(kv):
    return kv.layer_k(0).ravel().tolist()


def _v(kv):
    return kv.layer_v(0).ravel().tolist()


def test_int8_roundtrip():  # transformer.rs:1136-1159
    kv = _layer(o.KV_INT8, 2)
    kv.append([0.5, -0.3], [1.2, -0.8])
    assert np.allclose(_k(kv), [0.5, -0.3], atol=0.02)
    assert np.allclose(_v(kv), [1.2, -0.8], atol=0.02)
    # q = round(x / (max|x| / 127)) * scale: the largest element is exact
    assert _k(kv)[0] == np.float32(0.5)


def test_int8_multiple_tokens():  # :1161-1172
    kv = _layer(o.KV_INT8, 2)
    kv.append([1.0, 0.0], [0.0, 1.0])
    kv.append([0.5, 0.5], [0.5, 0.5])
    assert len(kv) == 2 and len(_k(kv)) == 4 and len(_v(kv)) == 4


def test_fp32_shift_discards_oldest():  # :1174-1185
    kv = _layer(o.KV_FP32, 2)
    for k, v in (([1, 2], [3, 4]), ([5, 6], [7, 8]), ([9, 10], [11, 12])):
        kv.append(k, v)
    kv.shift(1)
    assert len(kv) == 2
    assert _k(kv) == [5.0, 6.0, 9.0, 10.0]
    assert _v(kv) == [7.0, 8.0, 11.0, 12.0]


def test_int8_shift_discards_oldest():  # :1187-1201
    kv = _layer(o.KV_INT8, 2)
    for k, v in (([1, 0], [0, 1]), ([0.5, 0.5], [0.5, 0.5]), ([0, 1], [1, 0])):
        kv.append(k, v)
    kv.shift(2)
    assert len(kv) == 1 and _k(kv) == [0.0, 1.0] and _v(kv) == [1.0, 0.0]


def test_cache_shift_syncs_all_layers():  # :1203-1217 (every layer shifts alike)
    kv = o.OracleKV(None, 8, n_layers=2, kv_dim=2)
    kv.append([1, 2], [3, 4])
    kv.append([5, 6], [7, 8])
    kv.shift(1)
    assert len(kv) == 1
    assert kv.layer_k(0).ravel().tolist() == [5.0, 6.0]
    assert kv.layer_k(1).ravel().tolist() == [5.0, 6.0]


def test_mixed_keeps_recent_in_fp32():  # :1219-1238
    kv = _layer(o.KV_MIXED, 2, window=2)
    for k, v in (([1, 0], [0, 1]), ([0.5, 0.5], [0.5, 0.5]), ([0, 1], [1, 0])):
        kv.append(k, v)
    k = _k(kv)
    assert len(kv) == 3 and len(k) == 6
    assert abs(k[0] - 1.0) < 0.02 and abs(k[1]) < 0.02
    assert k[2:] == [0.5, 0.5, 0.0, 1.0]


def test_mixed_matches_fp32_output():  # :1240-1259
    mixed, fp32 = _layer(o.KV_MIXED, 4, window=3), _layer(o.KV_FP32, 4)
    for i in range(8):
        for kv in (mixed, fp32):
            kv.append([float(i)] * 4, [float(i + 1)] * 4)
    assert len(mixed) == 8
    assert np.allclose(_k(mixed), _k(fp32), atol=0.05)
    # five cold tokens were quantized: a constant row is exact after int8
    assert _k(mixed) == _k(fp32)


def test_mixed_shift_discards_oldest():  # :1261-1274
    kv = _layer(o.KV_MIXED, 2, window=2)
    for k, v in (([1, 0], [0, 1]), ([0.5, 0.5], [0.5, 0.5]), ([0, 1], [1, 0]), ([2, 2], [3, 3])):
        kv.append(k, v)
    kv.shift(2)
    assert len(kv) == 2 and _k(kv) == [0.0, 1.0, 2.0, 2.0]


def test_fp32_shift_anchored_preserves_first():  # :1276-1287
    kv = _layer(o.KV_FP32, 2)
    for i in range(6):
        kv.append([i, i + 0.5], [i + 10.0, i + 10.5])
    kv.shift(2, anchor=2)
    assert len(kv) == 4
    assert _k(kv) == [0.0, 0.5, 1.0, 1.5, 4.0, 4.5, 5.0, 5.5]


def test_int8_shift_anchored_preserves_first():  # :1289-1303
    kv = _layer(o.KV_INT8, 2)
    for i in range(6):
        kv.append([i, i + 0.5], [i + 10.0, i + 10.5])
    kv.shift(2, anchor=2)
    k = _k(kv)
    assert len(kv) == 4
    for j, want in ((0, 0.0), (2, 1.0), (4, 4.0), (6, 5.0)):
        assert abs(k[j] - want) < 0.02


def test_mixed_shift_anchored_preserves_first():  # :1305-1322
    kv = _layer(o.KV_MIXED, 2, window=3)
    for i in range(8):
        kv.append([i, i + 0.5], [i + 10.0, i + 10.5])
    kv.shift(3, anchor=2)
    k = _k(kv)
    assert len(kv) == 5
    for j, want in ((0, 0.0), (2, 1.0), (4, 5.0), (6, 6.0), (8, 7.0)):
        assert abs(k[j] - want) < 0.02
    # re-appended: the last `window` tokens are the f32 suffix, exactly
    assert k[4:] == [5.0, 5.5, 6.0, 6.5, 7.0, 7.5]


def test_shift_anchored_falls_back_when_not_enough_tokens():  # :1324-1333
    kv = _layer(o.KV_FP32, 2)
    kv.append([1, 2], [3, 4])
    kv.append([5, 6], [7, 8])
    kv.shift(1, anchor=2)
    assert len(kv) == 1 and _k(kv) == [5.0, 6.0]


def test_qdq_rules():
    # scale = max|x| / 127; halves round away from zero; NaN codes are 0
    x = np.array([127.0, 0.5, -0.5, 1.5, -2.5], np.float32)
    assert o.kv_qdq(x).tolist() == [127.0, 1.0, -1.0, 2.0, -3.0]
    assert o.kv_qdq(np.zeros(3, np.float32)).tolist() == [0.0, 0.0, 0.0]
    y = o.kv_qdq(np.array([np.nan, 1.0], np.float32))
    assert y[0] == 0.0 and y[1] == 1.0


def test_context_shift_plain_and_anchored():
    toks = list(range(100, 120))  # 20 tokens, prompt 12
    # plain: overflow = 20 - 16 + 4 = 8 oldest tokens leave
    t, pl, ov, at = o.context_shift(toks, 12, 16, 0)
    assert (ov, at, pl) == (8, 0, 4) and t == toks[8:]
    # anchored: the 8 tokens after the first 3 leave
    t, pl, ov, at = o.context_shift(toks, 12, 16, 3)
    assert (ov, at) == (8, 3) and t == toks[:3] + toks[11:]
    assert pl == 3 + (12 - 3) - 8  # removed = min(overflow, prompt tokens past the anchor)
    # the anchored branch needs len > anchor + overflow; else the plain one
    t, pl, ov, at = o.context_shift(toks, 12, 16, 12)
    assert (ov, at) == (8, 0) and t == toks[8:]
    # prompt_len saturates at 0 in the plain branch
    t, pl, ov, at = o.context_shift(toks, 5, 16, 0)
    assert pl == 0
