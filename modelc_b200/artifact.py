"""The reference's ``.modelc`` artifact container, read and written on the host.

Layout (version 2, pack.rs:1-22): the magic ``MODELC``, a u32 LE version, a
u32 LE flags word (version 2 only; bit 0 = the data blob is zstd-compressed),
a u64 LE header length, the header JSON ``{"name", "architecture",
"metadata": {str: str}, "tensors": [{"name", "shape", "dtype", "offset",
"length"}]}``, then the blob.  ``read_artifact`` follows ``unpack``
(pack.rs:148-236): versions 1 and 2, tensors cut from the (decompressed)
blob by offset and length, a tensor past the blob's end is an error.
``write_artifact`` follows ``pack`` (pack.rs:42-101): tensors in sorted name
order, offsets accumulated in that order, the blob compressed with zstd level
3 when asked.  zstd itself is the system ``libzstd`` (the reference links the
``zstd`` crate, which wraps the same library).

``weights_from_artifact`` turns an artifact into the device loader's tensors
the way ``modelc run`` materialises them (``Model::dequantize_in_place``,
model.rs:148-199, then ``Runtime::from_raw``, runtime/serve.rs:121-132):

* ``i8`` with metadata ``quant_scale.<name>`` whose text parses as an f32
  (the rule of Rust's ``str::parse::<f32>``: correctly rounded, no
  whitespace) is per-tensor int8, value ``q as f32 * scale``; with
  ``quant_mode.<name> == "int4"`` the bytes hold two signed nibbles each,
  high nibble first (model.rs:163-178), unpacked here to int8 codes with the
  same scale;
* ``i8`` without a parseable scale keeps its raw codes (scale 1.0), as
  ``bytes_to_f32_slice`` reads them;
* ``f32`` stays f32, ``f16``/``bf16`` convert exactly to f32, ``q4_0`` stays
  ggml blocks.
"""
from __future__ import annotations

import ctypes as C
import json
import struct
from dataclasses import dataclass, field
from fractions import Fraction

import numpy as np

from .model import QTensor, LlamaConfig, MODE_REFERENCE

MAGIC = b"MODELC"
VERSION = 2
FLAG_COMPRESSED = 1


class ArtifactError(ValueError):
    pass


@dataclass
class ArtifactTensor:
    shape: list
    dtype: str
    data: bytes


@dataclass
class Artifact:
    name: str = ""
    architecture: str = "llama"
    metadata: dict = field(default_factory=dict)
    tensors: dict = field(default_factory=dict)  # name -> ArtifactTensor


# ---------------------------------------------------------------- zstd
_zstd = None


def _libzstd():
    global _zstd
    if _zstd is None:
        try:
            L = C.CDLL("libzstd.so.1")
        except OSError as e:
            raise ArtifactError(f"zstd-compressed artifact but libzstd is unavailable: {e}")

        class Buf(C.Structure):
            _fields_ = [("ptr", C.c_void_p), ("size", C.c_size_t), ("pos", C.c_size_t)]
        L.ZSTD_createDStream.restype = C.c_void_p
        L.ZSTD_freeDStream.argtypes = [C.c_void_p]
        L.ZSTD_initDStream.argtypes = [C.c_void_p]
        L.ZSTD_decompressStream.restype = C.c_size_t
        L.ZSTD_decompressStream.argtypes = [C.c_void_p, C.POINTER(Buf), C.POINTER(Buf)]
        L.ZSTD_isError.argtypes = [C.c_size_t]
        L.ZSTD_getErrorName.restype = C.c_char_p
        L.ZSTD_getErrorName.argtypes = [C.c_size_t]
        L.ZSTD_compressBound.restype = C.c_size_t
        L.ZSTD_compressBound.argtypes = [C.c_size_t]
        L.ZSTD_compress.restype = C.c_size_t
        L.ZSTD_compress.argtypes = [C.c_void_p, C.c_size_t, C.c_void_p, C.c_size_t, C.c_int]
        L.Buf = Buf
        _zstd = L
    return _zstd


def zstd_decompress(data: bytes) -> bytes:
    """zstd::decode_all: every frame of data, streamed (frames need not
    record their content size)."""
    L = _libzstd()
    ds = L.ZSTD_createDStream()
    if not ds:
        raise ArtifactError("zstd: cannot create a decompression stream")
    try:
        L.ZSTD_initDStream(ds)
        src = C.create_string_buffer(bytes(data), len(data))
        inb = L.Buf(C.cast(src, C.c_void_p), len(data), 0)
        chunk = 1 << 22
        dst = C.create_string_buffer(chunk)
        out = bytearray()
        last = 0
        while True:
            outb = L.Buf(C.cast(dst, C.c_void_p), chunk, 0)
            last = L.ZSTD_decompressStream(ds, C.byref(outb), C.byref(inb))
            if L.ZSTD_isError(last):
                raise ArtifactError("failed to decompress artifact data: "
                                    + L.ZSTD_getErrorName(last).decode())
            out += dst.raw[:outb.pos]
            if inb.pos >= inb.size and outb.pos < chunk:
                break
        if last != 0:
            raise ArtifactError("failed to decompress artifact data: truncated zstd frame")
        return bytes(out)
    finally:
        L.ZSTD_freeDStream(ds)


def zstd_compress(data: bytes, level: int = 3) -> bytes:
    L = _libzstd()
    cap = L.ZSTD_compressBound(len(data))
    dst = C.create_string_buffer(cap)
    n = L.ZSTD_compress(dst, cap, bytes(data), len(data), level)
    if L.ZSTD_isError(n):
        raise ArtifactError("zstd compression failed: " + L.ZSTD_getErrorName(n).decode())
    return dst.raw[:n]


# ---------------------------------------------------------------- f32 text
def parse_f32(s: str):
    """Rust's ``str::parse::<f32>``: an optional sign, then ``inf``,
    ``infinity`` or ``nan`` (any case) or a decimal with an optional exponent,
    rounded once, to nearest-even, to f32.  Returns None where Rust returns
    Err (whitespace, empty text, stray characters)."""
    if not isinstance(s, str) or not s or s != s.strip():
        return None
    body = s[1:] if s[0] in "+-" else s
    neg = s[0] == "-"
    low = body.lower()
    if low in ("inf", "infinity"):
        return np.float32(-np.inf if neg else np.inf)
    if low == "nan":
        return np.float32(np.nan)
    mant, _, expo = low.partition("e")
    if "e" in low:
        if not expo or not (expo.lstrip("+-").isdigit() and expo.count("+") + expo.count("-") <= 1
                            and expo[0] in "+-0123456789"):
            return None
    ip, dot, fp = mant.partition(".")
    if not (ip + fp) or not (ip.isdigit() or ip == "") or not (fp.isdigit() or fp == ""):
        return None
    digits = (ip + fp).lstrip("0")
    e10 = (int(expo) if "e" in low else 0) - len(fp)
    if not digits:
        v = np.float32(0.0)
    elif len(digits) + e10 > 40:     # above 1e39: past the largest f32
        v = np.float32(np.inf)
    elif len(digits) + e10 < -47:    # below 1e-47: under half the smallest subnormal
        v = np.float32(0.0)
    else:
        v = _round_f32(Fraction(int(digits)) * Fraction(10) ** e10)
    return np.float32(-v) if neg else v


def _round_f32(x: Fraction):
    """The f32 nearest to x >= 0 (ties to even), inf above the largest."""
    if x == 0:
        return np.float32(0.0)
    fmax = Fraction(float(np.finfo(np.float32).max))
    half_ulp_top = Fraction(2) ** (127 - 24)
    if x >= fmax + half_ulp_top:
        return np.float32(np.inf)
    # exponent of x: 2^e <= x < 2^(e+1), f32 spacing 2^(max(e, -126) - 23)
    e = x.numerator.bit_length() - x.denominator.bit_length()
    if Fraction(2) ** e > x:
        e -= 1
    q = Fraction(2) ** (max(e, -126) - 23)
    n = x / q
    fl = n.numerator // n.denominator
    rem = n - fl
    if rem > Fraction(1, 2) or (rem == Fraction(1, 2) and fl % 2 == 1):
        fl += 1
    return np.float32(float(fl * q))


def format_f32(x) -> str:
    """Rust's ``Display`` for f32 (``f32::to_string``): the shortest digits that
    parse back to x, written positionally (no exponent), ``1`` for 1.0."""
    x = np.float32(x)
    if np.isnan(x):
        return "NaN"
    if np.isinf(x):
        return "inf" if x > 0 else "-inf"
    return np.format_float_positional(x, unique=True, trim="-")


# ---------------------------------------------------------------- container
def _parse_dtype(s):
    known = ("f32", "f16", "bf16", "i64", "i32", "i16", "i8", "u8", "bool", "q4_0", "q5_0",
             "q8_0", "q4_k", "q6_k")
    if s not in known:
        raise ArtifactError(f"unknown dtype '{s}' in artifact")
    return s


def read_artifact(path) -> Artifact:
    """pack.rs:148-236 unpack."""
    with open(path, "rb") as f:
        raw = f.read()
    if len(raw) < 6:
        raise ArtifactError("artifact file too short (magic)")
    if raw[:6] != MAGIC:
        raise ArtifactError("invalid artifact magic bytes (not a .modelc file)")
    pos = 6
    if len(raw) < pos + 4:
        raise ArtifactError("artifact file too short (version)")
    (version,) = struct.unpack_from("<I", raw, pos)
    pos += 4
    flags = 0
    if version >= 2:
        if len(raw) < pos + 4:
            raise ArtifactError("artifact file too short (flags)")
        (flags,) = struct.unpack_from("<I", raw, pos)
        pos += 4
    if version not in (1, 2):
        raise ArtifactError(f"unsupported artifact version {version} (expected 1 or 2)")
    if len(raw) < pos + 8:
        raise ArtifactError("artifact file too short (header length)")
    (hlen,) = struct.unpack_from("<Q", raw, pos)
    pos += 8
    if len(raw) < pos + hlen:
        raise ArtifactError("artifact file too short (header)")
    try:
        header = json.loads(raw[pos:pos + hlen].decode("utf-8"))
    except (UnicodeDecodeError, json.JSONDecodeError) as e:
        raise ArtifactError(f"failed to deserialize artifact header: {e}")
    blob = raw[pos + hlen:]
    if flags & FLAG_COMPRESSED:
        blob = zstd_decompress(blob)
    art = Artifact(header.get("name", ""), header.get("architecture", ""),
                   dict(header.get("metadata", {})), {})
    for t in header["tensors"]:
        start, length = int(t["offset"]), int(t["length"])
        if start + length > len(blob):
            raise ArtifactError(
                f"artifact corrupted: tensor {t['name']} claims offset {start} + length {length} "
                f"exceeds blob size {len(blob)}")
        art.tensors[t["name"]] = ArtifactTensor(list(t["shape"]), _parse_dtype(t["dtype"]),
                                                blob[start:start + length])
    return art


def write_artifact(path, art: Artifact, compress: bool = False) -> None:
    """pack.rs:42-101 pack: sorted tensor names, offsets in that order."""
    names = sorted(art.tensors)
    entries, blob, off = [], bytearray(), 0
    for n in names:
        t = art.tensors[n]
        entries.append({"name": n, "shape": [int(v) for v in t.shape], "dtype": t.dtype,
                        "offset": off, "length": len(t.data)})
        blob += t.data
        off += len(t.data)
    header = json.dumps({"name": art.name, "architecture": art.architecture,
                         "metadata": art.metadata, "tensors": entries},
                        separators=(",", ":")).encode()
    data = zstd_compress(bytes(blob), 3) if compress else bytes(blob)
    with open(path, "wb") as f:
        f.write(MAGIC)
        f.write(struct.pack("<IIQ", VERSION, FLAG_COMPRESSED if compress else 0, len(header)))
        f.write(header)
        f.write(data)


def pack_quantized_int8(tensors: dict, name: str = "model", architecture: str = "llama") -> Artifact:
    """What ``modelc pack --quantize int8`` writes for f32 tensors
    (compiler.rs:207-229): every tensor with max|x| > 0 becomes ``i8`` with
    scale max|x| / 127 stored as the text ``quant_scale.<name>``; all-zero
    tensors stay ``f32``.  tensors: name -> f32 numpy array."""
    from .model import quantize_int8_tensor
    art = Artifact(name, architecture, {}, {})
    for n, x in tensors.items():
        x = np.ascontiguousarray(x, np.float32)
        q, scale = quantize_int8_tensor(x)
        if scale > 0:
            art.tensors[n] = ArtifactTensor(list(x.shape), "i8", q.tobytes())
            art.metadata[f"quant_scale.{n}"] = format_f32(scale)
        else:
            art.tensors[n] = ArtifactTensor(list(x.shape), "f32", x.tobytes())
    return art


# ---------------------------------------------------------------- to the device loader
def _count(shape):
    n = 1
    for v in shape:
        n *= int(v)
    return n


def weights_from_artifact(art: Artifact) -> dict:
    """name -> QTensor for mc_weights_load, holding exactly the values that
    dequantize_in_place + Runtime::from_raw give the reference."""
    out = {}
    for n, t in art.tensors.items():
        shape = tuple(int(v) for v in t.shape)
        cnt = _count(shape)
        if t.dtype == "i8":
            sc = parse_f32(art.metadata.get(f"quant_scale.{n}")) \
                if f"quant_scale.{n}" in art.metadata else None
            buf = np.frombuffer(t.data, np.uint8)
            if sc is not None and art.metadata.get(f"quant_mode.{n}") == "int4":
                hi = ((buf >> 4) & 0x0F).astype(np.int16) - 8
                lo = (buf & 0x0F).astype(np.int16) - 8
                codes = np.stack([hi, lo], axis=1).reshape(-1)[:cnt].astype(np.int8)
            else:
                if len(buf) < cnt:
                    raise ArtifactError(f"{n}: {len(buf)} bytes for {cnt} int8 elements")
                codes = buf[:cnt].view(np.int8)
            scale = np.float32(1.0) if sc is None else np.float32(sc)
            out[n] = QTensor("i8_tensor", codes.reshape(shape).copy(), scale)
        elif t.dtype == "f32":
            out[n] = QTensor("f32", np.frombuffer(t.data, "<f4", cnt).reshape(shape).copy())
        elif t.dtype == "f16":
            out[n] = QTensor("f32", np.frombuffer(t.data, "<f2", cnt).astype(np.float32)
                             .reshape(shape))
        elif t.dtype == "bf16":
            b = np.frombuffer(t.data, "<u2", cnt).astype(np.uint32) << 16
            out[n] = QTensor("f32", b.view(np.float32).reshape(shape).copy())
        elif t.dtype == "q4_0":
            if len(shape) != 2 or shape[1] % 32:
                raise ArtifactError(f"{n}: q4_0 matrices need in_features % 32 == 0")
            out[n] = QTensor("q4_0", np.frombuffer(t.data, np.uint8).reshape(shape[0], -1).copy(),
                             None, shape)
        else:
            raise ArtifactError(f"{n}: dtype {t.dtype} is not on the device path")
    return out


def llama_config_from_artifact(art: Artifact, name: str = "artifact") -> LlamaConfig:
    """The reference runtime's view of a Llama artifact (arch.rs:29-137,
    generate.rs:865-881): layers counted from model.layers.{i}. names, hidden
    from q_proj's input width, FFN from gate_proj's rows, vocab from the
    embedding (or head) rows; heads = hidden / 64 in reference mode."""
    layers = set()
    for n in art.tensors:
        if n.startswith("model.layers."):
            layers.add(int(n.split(".")[2]))
    q = art.tensors["model.layers.0.self_attn.q_proj.weight"].shape
    g = art.tensors["model.layers.0.mlp.gate_proj.weight"].shape
    emb = art.tensors.get("model.embed_tokens.weight") or art.tensors.get("lm_head.weight")
    hidden = int(q[1])
    nh = max(hidden // 64, 1)
    return LlamaConfig(len(layers), hidden, nh, nh, hidden // nh, int(g[0]), int(emb.shape[0]),
                       10000.0, 1e-6, MODE_REFERENCE, name)
