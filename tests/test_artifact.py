"""The reference's artifact path: ``.modelc`` v2 container, ``quant_scale``
text, per-tensor int8 through the device loader.

CPU:
* write -> read round trips, raw and zstd-compressed (pack.rs:42-101,
  :148-236): the header JSON, sorted names and offsets; version-1 files
  (no flags word); the reference's error cases (bad magic, unknown version,
  a tensor past the blob, an unknown dtype);
* the scale text: Rust's ``f32::to_string`` digits (shortest round trip,
  positional) and ``str::parse::<f32>`` (one correct rounding, including a
  decimal just above an f32 midpoint, where parsing through f64 rounds
  twice and lands on the wrong neighbour);
* ``modelc pack --quantize int8`` (compiler.rs:207-229) applied to every f32
  tensor, norms and embeddings included, and the tensors the device loader
  receives equal the reference's dequantized values (model.rs:182-185); the
  int4 mode's nibble order (model.rs:163-178).

GPU: the tiny benchmark workload (4-layer d 256 target, seed 0; 1-layer
draft, seed 1; 32-id prompt, seed 2; gamma 4; 128 new tokens, greedy) packed
exactly as ``modelc pack --quantize int8`` packs it (the draft artifact
zstd-compressed), read back, loaded as MC_DTYPE_I8_TENSOR in reference mode
(heads = hidden / 64, theta 1e4, eps 1e-6): identical tokens and accepted
counts to the oracle running on the same artifact's dequantized weights.
"""
import json
import os
import struct
import sys

import numpy as np
import pytest

sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "oracle"))
import oracle as o  # noqa: E402

import modelc_b200 as mb  # noqa: E402
from modelc_b200 import artifact as A  # noqa: E402


def _art(seed=0):
    rng = np.random.default_rng(seed)
    art = A.Artifact("m", "llama", {"quant_scale.b": "0.5"}, {})
    art.tensors["b"] = A.ArtifactTensor([2, 3], "i8", rng.integers(-127, 128, 6, dtype=np.int8).tobytes())
    art.tensors["a"] = A.ArtifactTensor([4], "f32", rng.standard_normal(4).astype(np.float32).tobytes())
    art.tensors["c"] = A.ArtifactTensor([1, 32], "q4_0", bytes(range(18)))
    return art


@pytest.mark.parametrize("compress", [False, True])
def test_container_round_trip(tmp_path, compress):
    art = _art()
    p = tmp_path / "m.modelc"
    A.write_artifact(p, art, compress=compress)
    raw = p.read_bytes()
    assert raw[:6] == b"MODELC"
    version, flags, hlen = struct.unpack_from("<IIQ", raw, 6)
    assert (version, flags) == (2, 1 if compress else 0)
    header = json.loads(raw[22:22 + hlen])
    assert [t["name"] for t in header["tensors"]] == ["a", "b", "c"]  # sorted (pack.rs:53-55)
    assert [t["offset"] for t in header["tensors"]] == [0, 16, 22]
    back = A.read_artifact(p)
    assert back.name == "m" and back.metadata == art.metadata
    for n, t in art.tensors.items():
        assert back.tensors[n].data == t.data
        assert back.tensors[n].shape == t.shape and back.tensors[n].dtype == t.dtype


def test_version1_has_no_flags_word(tmp_path):
    art = _art(1)
    p = tmp_path / "v2.modelc"
    A.write_artifact(p, art)
    raw = p.read_bytes()
    _, _, hlen = struct.unpack_from("<IIQ", raw, 6)
    v1 = b"MODELC" + struct.pack("<IQ", 1, hlen) + raw[22:]
    q = tmp_path / "v1.modelc"
    q.write_bytes(v1)
    back = A.read_artifact(q)
    assert back.tensors["b"].data == art.tensors["b"].data


def test_container_errors(tmp_path):
    art = _art(2)
    p = tmp_path / "m.modelc"
    A.write_artifact(p, art)
    raw = p.read_bytes()
    bad = tmp_path / "bad.modelc"
    for blob, msg in [(b"MODELX" + raw[6:], "magic"), (raw[:6] + struct.pack("<I", 3) + raw[10:],
                                                        "version"),
                      (raw[:-5], "exceeds blob size"), (raw[:15], "too short")]:
        bad.write_bytes(blob)
        with pytest.raises(A.ArtifactError, match=msg):
            A.read_artifact(bad)
    art.tensors["d"] = A.ArtifactTensor([1], "f64", b"\0" * 8)
    A.write_artifact(p, art)
    with pytest.raises(A.ArtifactError, match="unknown dtype"):
        A.read_artifact(p)


def test_zstd_decodes_concatenated_frames():
    a, b = os.urandom(1000) + bytes(5000), bytes(range(256)) * 40
    assert A.zstd_decompress(A.zstd_compress(a) + A.zstd_compress(b)) == a + b
    with pytest.raises(A.ArtifactError):
        A.zstd_decompress(A.zstd_compress(a)[:-3])


def test_parse_f32_follows_rust():
    f = np.float32
    cases = {"0.5": f(0.5), "1": f(1.0), "+1.5": f(1.5), "-0": f(-0.0), ".25": f(0.25),
             "5.": f(5.0), "1e-3": f(1e-3), "2.5E2": f(250.0), "1e400": f(np.inf),
             "-1e400": f(-np.inf), "1e-50": f(0.0), "inf": f(np.inf), "-Infinity": f(-np.inf),
             "0.007874016": f(1.0) / f(127.0)}
    for s, want in cases.items():
        got = A.parse_f32(s)
        assert got is not None and got.dtype == np.float32, s
        assert got == want and np.signbit(got) == np.signbit(want), (s, got, want)
    assert np.isnan(A.parse_f32("NaN"))
    for s in ["", " 1", "1 ", "1_000", "1e", "e5", "0x10", "1.2.3", "+-1", "--1", "1e5e3", "."]:
        assert A.parse_f32(s) is None, s
    # just above the midpoint of 1 and its successor: one rounding goes up;
    # through f64 the text first becomes the exact midpoint, which rounds to 1
    s = "1.0000000596046447753906250000000001"
    assert A.parse_f32(s) == np.nextafter(np.float32(1.0), np.float32(2.0))
    assert np.float32(float(s)) == np.float32(1.0)
    assert A.parse_f32("1.000000059604644775390625") == np.float32(1.0)  # tie -> even
    # the smallest subnormal and the rounding into it
    assert A.parse_f32("1.401298464324817e-45") == np.float32(1.401298464324817e-45)
    assert A.parse_f32("7e-46") == np.float32(0.0)
    assert A.parse_f32("8e-46") == np.float32(1.401298464324817e-45)


def test_format_f32_shortest_positional_round_trip():
    f = np.float32
    assert A.format_f32(f(1.0)) == "1"
    assert A.format_f32(f(0.5)) == "0.5"
    assert A.format_f32(f(1e-7)) == "0.0000001"
    assert A.format_f32(f(1.0) / f(127.0)) == "0.007874016"
    assert A.format_f32(f(-0.0)) == "-0"
    rng = np.random.default_rng(0)
    xs = np.concatenate([rng.standard_normal(3000).astype(np.float32) * f(0.02) / f(127.0),
                         rng.integers(0, 2**31 - 1, 3000, dtype=np.uint32).view(np.float32)])
    for x in xs:
        if np.isfinite(x):
            assert A.parse_f32(A.format_f32(x)) == x, x


def test_pack_quantize_int8_rule_and_loader_values():
    rng = np.random.default_rng(4)
    w = (rng.standard_normal((8, 40)) * 0.02).astype(np.float32)
    norm = np.ones(40, np.float32)
    zero = np.zeros(40, np.float32)
    art = A.pack_quantized_int8({"w": w, "norm": norm, "z": zero})
    assert art.tensors["w"].dtype == "i8" and art.tensors["norm"].dtype == "i8"
    assert art.tensors["z"].dtype == "f32"  # max|x| == 0 stays f32 (compiler.rs:215)
    q, s = o.quantize_int8_tensor(w)
    assert art.tensors["w"].data == q.tobytes()
    assert A.parse_f32(art.metadata["quant_scale.w"]) == np.float32(s)
    ws = A.weights_from_artifact(art)
    assert ws["w"].dtype == "i8_tensor"
    ref = (q.astype(np.float32) * np.float32(s)).astype(np.float32)  # model.rs:182-185
    assert np.array_equal(ws["w"].dequant(), ref)
    assert np.array_equal(ws["norm"].dequant(),
                          (np.full(40, 127, np.float32) * (np.float32(1) / np.float32(127))))
    assert np.array_equal(ws["z"].dequant(), zero)


def test_int4_nibbles_and_unscaled_i8():
    art = A.Artifact("m", "llama", {"quant_scale.q": "0.25", "quant_mode.q": "int4"}, {})
    art.tensors["q"] = A.ArtifactTensor([3], "i8", bytes([0x0F, 0x80]))  # 3 nibbles
    art.tensors["raw"] = A.ArtifactTensor([2], "i8", bytes([0xFF, 0x05]))  # no scale
    art.metadata["quant_scale.bad"] = "0.5 "  # not parseable by Rust: raw codes
    art.tensors["bad"] = A.ArtifactTensor([1], "i8", bytes([3]))
    ws = A.weights_from_artifact(art)
    # high nibble first (model.rs:168-175): 0x0F -> -8, 7; 0x80 -> 0
    assert ws["q"].dequant().tolist() == [-2.0, 1.75, 0.0]
    assert ws["raw"].dequant().tolist() == [-1.0, 5.0]
    assert ws["bad"].dequant().tolist() == [3.0]


def _tiny_f32(cfg, seed):
    return {k: v.data for k, v in mb.synth_weights(cfg, seed=seed, fmt="f32").items()}


@pytest.mark.gpu
def test_reference_int8_artifact_spec_decode(tmp_path):
    cfg = mb.TINY
    tp, dp = tmp_path / "target.modelc", tmp_path / "draft.modelc"
    A.write_artifact(tp, A.pack_quantized_int8(_tiny_f32(cfg, 0)))
    A.write_artifact(dp, A.pack_quantized_int8(_tiny_f32(cfg.with_layers(1), 1)), compress=True)
    ta, da = A.read_artifact(tp), A.read_artifact(dp)
    tcfg, dcfg = A.llama_config_from_artifact(ta), A.llama_config_from_artifact(da)
    assert (tcfg.n_layers, tcfg.hidden, tcfg.n_heads, tcfg.ffn, tcfg.vocab) == (4, 256, 4, 688, 4096)
    assert dcfg.n_layers == 1
    tw, dw = A.weights_from_artifact(ta), A.weights_from_artifact(da)
    assert all(t.dtype == "i8_tensor" for t in tw.values())  # norms and embeddings too

    def om(ws, c):
        return o.OracleModel({k: v.dequant() for k, v in ws.items()}, c.n_layers, c.hidden,
                             c.vocab, c.ffn, mode=o.MODE_REFERENCE)
    prompt = np.random.default_rng(2).integers(0, cfg.vocab, 32).tolist()
    ref, racc = om(tw, tcfg).speculative_generate(prompt, 128, 4,
                                                  o.OracleLlamaDraft(om(dw, dcfg), 256))
    s = mb.Session(mb.Weights(tw, tcfg), mb.Weights(dw, dcfg), gamma=4, max_context=256)
    got, gacc = s.speculative_generate(prompt, 128)
    s.close()
    assert got == ref
    assert gacc == racc
