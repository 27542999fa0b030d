"""Model configurations, synthetic weights, quantizers and device weights.

Tensor names and layouts follow the reference (``model.layers.{i}.self_attn.
q_proj.weight`` ..., matrices ``[out, in]``, transformer.rs:825).  The int8
quantization rule is the reference's pack-time rule (compiler.rs:207-229:
scale = max|x|/127, q = round(clamp(x/scale, -127, 127)), Rust ``round`` =
half away from zero) applied per output row.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, field, replace

import numpy as np

from . import _lib
from ._lib import check, lib

MODE_REFERENCE = _lib.MODE_REFERENCE
MODE_GENERAL = _lib.MODE_GENERAL


@dataclass(frozen=True)
class LlamaConfig:
    n_layers: int
    hidden: int
    n_heads: int
    n_kv_heads: int
    head_dim: int
    ffn: int
    vocab: int
    rope_theta: float = 10000.0
    eps: float = 1e-5
    mode: int = MODE_GENERAL
    name: str = "llama"

    def with_layers(self, n: int) -> "LlamaConfig":
        return replace(self, n_layers=n)

    def resolved(self) -> "LlamaConfig":
        """Head geometry as the runtime uses it (reference mode: hidden/64
        heads, MHA, theta 1e4, eps 1e-6; arch.rs:128-137)."""
        if self.mode != MODE_REFERENCE:
            return self
        nh = max(self.hidden // 64, 1)
        return replace(self, n_heads=nh, n_kv_heads=nh, head_dim=self.hidden // nh,
                       rope_theta=10000.0, eps=1e-6)

    def param_counts(self) -> dict:
        c = self.resolved()
        d, hd = c.hidden, c.head_dim
        attn = d * (c.n_heads * hd) * 2 + d * (c.n_kv_heads * hd) * 2
        mlp = 3 * d * c.ffn
        return {"layer": attn + mlp, "head": c.vocab * d, "embed": c.vocab * d}


# The workloads (shapes, seeds, run lengths) of the speculative-decoding
# benchmarks.  Reference-mode configs run exactly the reference's semantics.
TINY = LlamaConfig(4, 256, 4, 4, 64, 688, 4096, 10000.0, 1e-6, MODE_REFERENCE, "tiny-4L-d256")
TINYLLAMA = LlamaConfig(22, 2048, 32, 4, 64, 5632, 32000, 10000.0, 1e-5, MODE_GENERAL,
                        "tinyllama-1.1b")
LLAMA3_8B = LlamaConfig(32, 4096, 32, 8, 128, 14336, 128256, 500000.0, 1e-5, MODE_GENERAL,
                        "llama3-8b")
LLAMA2_70B = LlamaConfig(80, 8192, 64, 8, 128, 28672, 32000, 10000.0, 1e-5, MODE_GENERAL,
                         "llama2-70b")
PRESETS = {c.name: c for c in (TINY, TINYLLAMA, LLAMA3_8B, LLAMA2_70B)}


def tensor_names(cfg: LlamaConfig, tied: bool = False):
    names = ["model.embed_tokens.weight"]
    for i in range(cfg.n_layers):
        p = f"model.layers.{i}."
        names += [p + "input_layernorm.weight", p + "self_attn.q_proj.weight",
                  p + "self_attn.k_proj.weight", p + "self_attn.v_proj.weight",
                  p + "self_attn.o_proj.weight", p + "post_attention_layernorm.weight",
                  p + "mlp.gate_proj.weight", p + "mlp.up_proj.weight",
                  p + "mlp.down_proj.weight"]
    names.append("model.norm.weight")
    if not tied:
        names.append("lm_head.weight")
    return names


def tensor_shape(cfg: LlamaConfig, name: str):
    c = cfg.resolved()
    d, hd = c.hidden, c.head_dim
    if name.endswith("norm.weight"):
        return (d,)
    if name.endswith("q_proj.weight"):
        return (c.n_heads * hd, d)
    if name.endswith(("k_proj.weight", "v_proj.weight")):
        return (c.n_kv_heads * hd, d)
    if name.endswith("o_proj.weight"):
        return (d, c.n_heads * hd)
    if name.endswith(("gate_proj.weight", "up_proj.weight")):
        return (c.ffn, d)
    if name.endswith("down_proj.weight"):
        return (d, c.ffn)
    return (c.vocab, d)  # embed_tokens / lm_head


# ------------------------------------------------------------------ quantizers
def _round_half_away(v: np.ndarray) -> np.ndarray:
    """Rust f32::round (half away from zero), exact for f32 inputs."""
    v64 = v.astype(np.float64)
    return np.sign(v64) * np.floor(np.abs(v64) + 0.5)


def quantize_int8_rows(x: np.ndarray):
    """Per-row int8: the compiler.rs:207-229 rule applied to each output row.
    All-zero rows get scale 1.0 (transformer.rs:195-197)."""
    x = np.ascontiguousarray(x, np.float32)
    amax = np.max(np.abs(x), axis=1)
    scale = (amax / np.float32(127.0)).astype(np.float32)
    zero = ~(amax > 0)
    safe = np.where(zero, np.float32(1.0), scale).astype(np.float32)
    v = (x / safe[:, None]).astype(np.float32)
    v = np.clip(v, np.float32(-127.0), np.float32(127.0))
    q = _round_half_away(v).astype(np.int8)
    q[zero] = 0
    return q, safe


def quantize_int8_tensor(x: np.ndarray):
    """compiler.rs:207-229 per-tensor int8 (scale 0.0 = left unquantized)."""
    x = np.ascontiguousarray(x, np.float32)
    amax = np.float32(np.max(np.abs(x))) if x.size else np.float32(0)
    if not amax > 0:
        return np.zeros(x.shape, np.int8), np.float32(0.0)
    scale = np.float32(amax / np.float32(127.0))
    v = np.clip((x / scale).astype(np.float32), -127.0, 127.0)
    return _round_half_away(v).astype(np.int8), scale


def dequant_int8_rows(q: np.ndarray, scale: np.ndarray) -> np.ndarray:
    """model.rs:182-185: (q as f32) * scale."""
    return (q.astype(np.float32) * scale.astype(np.float32)[:, None]).astype(np.float32)


def quantize_q4_0(x: np.ndarray) -> np.ndarray:
    """ggml's q4_0 rule (the format parsers/gguf/dequant.rs:23-46 reads):
    per block of 32 consecutive weights, d = (the signed value of largest
    magnitude, first on ties) / -8, codes = trunc(x / d + 8.5) clamped to 15,
    d stored as fp16.  Returns uint8 [rows, cols/32 * 18] for [rows, cols]."""
    x = np.ascontiguousarray(x, np.float32)
    rows, cols = x.shape
    if cols % 32:
        raise ValueError("q4_0 needs cols % 32 == 0")
    b = x.reshape(rows, cols // 32, 32)
    idx = np.argmax(np.abs(b), axis=2)  # first index of the largest |x|
    mx = np.take_along_axis(b, idx[..., None], axis=2)[..., 0]
    d = (mx / np.float32(-8.0)).astype(np.float32)
    with np.errstate(divide="ignore"):
        inv = np.where(d != 0, np.float32(1.0) / d, np.float32(0.0)).astype(np.float32)
    v = (b * inv[..., None]).astype(np.float32) + np.float32(8.5)
    q = np.minimum(np.trunc(v).astype(np.int32), 15).astype(np.uint8)
    out = np.empty((rows, cols // 32, 18), np.uint8)
    out[..., 0:2] = d.astype(np.float16).view(np.uint8).reshape(rows, cols // 32, 2)
    out[..., 2:] = q[..., :16] | (q[..., 16:] << 4)
    return out.reshape(rows, cols // 32 * 18)


def dequant_q4_0(blocks: np.ndarray, rows: int, cols: int) -> np.ndarray:
    """dequant.rs:33-44: (code - 8) as f32 * d, low nibbles first."""
    b = np.ascontiguousarray(blocks, np.uint8).reshape(rows, cols // 32, 18)
    d = b[..., 0:2].copy().view(np.float16).astype(np.float32)  # [rows, nb, 1]
    qs = b[..., 2:].astype(np.int32)
    lo = (qs & 0x0F) - 8
    hi = (qs >> 4) - 8
    v = np.concatenate([lo, hi], axis=2).astype(np.float32) * d
    return v.reshape(rows, cols).astype(np.float32)


@dataclass
class QTensor:
    dtype: str                 # "f32" | "i8_row" | "i8_tensor" | "q4_0"
    data: np.ndarray
    scales: np.ndarray | None = None
    qshape: tuple | None = None  # logical [rows, cols] of q4_0 blocks

    @property
    def shape(self):
        return tuple(self.qshape) if self.qshape is not None else self.data.shape

    def dequant(self) -> np.ndarray:
        if self.dtype == "f32":
            return np.ascontiguousarray(self.data, np.float32)
        if self.dtype == "i8_row":
            return dequant_int8_rows(self.data, self.scales)
        if self.dtype == "i8_tensor":
            return (self.data.astype(np.float32) * np.float32(self.scales)).astype(np.float32)
        if self.dtype == "q4_0":
            return dequant_q4_0(self.data, *self.shape)
        raise ValueError(self.dtype)


def synth_weights(cfg: LlamaConfig, seed: int, std: float = 0.02, fmt: str = "i8_row",
                  tied: bool = False) -> dict:
    """Seeded synthetic weights: N(0, std) f32 (numpy PCG64, tensors drawn in
    tensor_names order), quantized per output row; norm weights 1.0."""
    rng = np.random.default_rng(seed)
    out = {}
    for name in tensor_names(cfg, tied):
        shape = tensor_shape(cfg, name)
        if len(shape) == 1:
            out[name] = QTensor("f32", np.ones(shape, np.float32))
            continue
        w = (rng.standard_normal(shape, dtype=np.float32) * np.float32(std)).astype(np.float32)
        if fmt == "i8_row":
            q, s = quantize_int8_rows(w)
            out[name] = QTensor("i8_row", q, s)
        elif fmt == "q4_0":
            out[name] = QTensor("q4_0", quantize_q4_0(w), None, shape)
        elif fmt == "f32":
            out[name] = QTensor("f32", w)
        else:
            raise ValueError(fmt)
    return out


def _q4_0_torch(w):
    """quantize_q4_0 in torch (same rule, f32 arithmetic) for device tensors."""
    import torch
    rows, cols = w.shape
    b = w.view(rows, cols // 32, 32)
    idx = b.abs().argmax(dim=2, keepdim=True)  # first maximal index
    mx = b.gather(2, idx)[..., 0]
    d = mx / -8.0
    inv = torch.where(d != 0, 1.0 / d, torch.zeros_like(d))
    v = b * inv[..., None] + 8.5
    q = v.trunc().to(torch.int32).clamp_(max=15).to(torch.uint8)
    out = torch.empty((rows, cols // 32, 18), dtype=torch.uint8, device=w.device)
    out[..., 0:2] = d.to(torch.float16).contiguous().view(torch.uint8).view(rows, cols // 32, 2)
    out[..., 2:] = q[..., :16] | (q[..., 16:] << 4)
    return out.view(rows, cols // 32 * 18)


def synth_weights_torch(cfg: LlamaConfig, seed: int, device, std: float = 0.02,
                        tied: bool = False, fmt: str = "i8_row") -> dict:
    """The same distribution generated on the GPU (for the multi-GB shapes):
    torch.randn per tensor from one seeded CUDA generator, then the per-row
    int8 rule (or q4_0) in f32 arithmetic.  Returns name -> (dtype, tensor,
    scales); q4_0 entries are ("q4_0", blocks, (rows, cols))."""
    import torch
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    out = {}
    for name in tensor_names(cfg, tied):
        shape = tensor_shape(cfg, name)
        if len(shape) == 1:
            out[name] = ("f32", torch.ones(shape, dtype=torch.float32, device=device), None)
            continue
        rows = shape[0]
        if fmt == "q4_0":
            blk = torch.empty((rows, shape[1] // 32 * 18), dtype=torch.uint8, device=device)
            step = max(1, (1 << 28) // shape[1])
            for r0 in range(0, rows, step):
                w = torch.randn((min(step, rows - r0), shape[1]), generator=g, device=device,
                                dtype=torch.float32) * std
                blk[r0:r0 + w.shape[0]] = _q4_0_torch(w)
                del w
            out[name] = ("q4_0", blk, tuple(shape))
            continue
        q = torch.empty(shape, dtype=torch.int8, device=device)
        sc = torch.empty(rows, dtype=torch.float32, device=device)
        step = max(1, (1 << 28) // shape[1])
        for r0 in range(0, rows, step):
            w = torch.randn((min(step, rows - r0), shape[1]), generator=g, device=device,
                            dtype=torch.float32) * std
            amax = w.abs().amax(dim=1)
            s = amax / 127.0
            s = torch.where(amax > 0, s, torch.ones_like(s))
            v = (w / s[:, None]).clamp_(-127.0, 127.0)
            a = v.abs()
            fl = a.floor()
            r = fl + ((a - fl) >= 0.5).to(torch.float32)
            q[r0:r0 + w.shape[0]] = (torch.sign(v) * r).to(torch.int8)
            sc[r0:r0 + w.shape[0]] = s
            del w, v, a, fl, r
        out[name] = ("i8_row", q, sc)
    return out


# ------------------------------------------------------------------ device weights
def _cfg_struct(cfg: LlamaConfig, tp_rank: int = 0, tp_world: int = 1) -> _lib.ModelCfg:
    return _lib.ModelCfg(cfg.mode, cfg.n_layers, cfg.hidden, cfg.n_heads, cfg.n_kv_heads,
                         cfg.head_dim, cfg.ffn, cfg.vocab, cfg.rope_theta, cfg.eps, tp_rank,
                         tp_world)


_DT = {"f32": _lib.DTYPE_F32, "i8_tensor": _lib.DTYPE_I8_TENSOR, "i8_row": _lib.DTYPE_I8_ROW,
       "q4_0": _lib.DTYPE_Q4_0}


def _desc_arrays(tensors: dict):
    """Build TensorDesc entries from numpy QTensors or torch (dtype, t, scales)."""
    keep, descs = [], []
    for name, t in tensors.items():
        if isinstance(t, QTensor):
            data = np.ascontiguousarray(t.data)
            sc = None
            if t.scales is not None:
                sc = np.ascontiguousarray(np.atleast_1d(np.asarray(t.scales, np.float32)))
            keep += [data, sc]
            shape = list(t.shape) + [0] * (2 - len(t.shape))
            descs.append(_lib.TensorDesc(name.encode(), _DT[t.dtype], _lib.MEM_HOST, len(t.shape),
                                         (C.c_int64 * 2)(*shape), data.ctypes.data,
                                         sc.ctypes.data if sc is not None else None))
        else:
            dt, ten, sc = t
            if dt == "q4_0":  # sc carries the logical (rows, cols)
                keep += [ten]
                descs.append(_lib.TensorDesc(name.encode(), _DT[dt], _lib.MEM_DEVICE, 2,
                                             (C.c_int64 * 2)(*sc), ten.data_ptr(), None))
                continue
            keep += [ten, sc]
            shape = list(ten.shape) + [0] * (2 - ten.dim())
            descs.append(_lib.TensorDesc(name.encode(), _DT[dt], _lib.MEM_DEVICE, ten.dim(),
                                         (C.c_int64 * 2)(*shape), ten.data_ptr(),
                                         sc.data_ptr() if sc is not None else None))
    arr = (_lib.TensorDesc * max(len(descs), 1))(*descs)
    return arr, len(descs), keep


class Weights:
    """Device-resident, repacked weights (the reference's Runtime,
    runtime/serve.rs:9-11, without the f32 dequantization)."""

    def __init__(self, tensors: dict, cfg: LlamaConfig, device: int = 0, tp_rank: int = 0,
                 tp_world: int = 1):
        """tp_world > 1 keeps this rank's tensor-parallel shard (Megatron:
        column-parallel q/k/v and gate/up, row-parallel o and down, vocab-
        parallel head) of the full tensors given."""
        self.cfg = cfg
        self.tp_rank, self.tp_world = tp_rank, tp_world
        arr, n, keep = _desc_arrays(tensors)
        h = C.c_void_p()
        c = _cfg_struct(cfg, tp_rank, tp_world)
        check(lib().mc_weights_load(arr, n, C.byref(c), device, C.byref(h)))
        del keep
        self.handle = h
        self.device = device

    @property
    def streamed_bytes(self) -> int:
        """Algorithmic weight bytes one forward streams (int8 codes + row scales)."""
        return int(lib().mc_weights_bytes(self.handle))

    def close(self):
        if getattr(self, "handle", None):
            lib().mc_weights_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Linear:
    """Standalone quantized projection y = x . dequant(W)^T (linear_with,
    transformer.rs:825-843) on device buffers."""

    def __init__(self, w: QTensor | tuple, device: int = 0):
        arr, n, keep = _desc_arrays({"w": w})
        h = C.c_void_p()
        check(lib().mc_linear_create(arr, device, C.byref(h)))
        self.handle = h
        self.out_features = int(arr[0].shape[0])
        self.in_features = int(arr[0].shape[1])

    @property
    def weight_bytes(self) -> int:
        return int(lib().mc_linear_weight_bytes(self.handle))

    def run_ptr(self, x_ptr: int, m: int, y_ptr: int, stream_ptr: int = 0):
        check(lib().mc_linear_run(self.handle, x_ptr, m, y_ptr, stream_ptr or None))

    def __call__(self, x):
        """x: torch CUDA f32 [m, in] -> torch CUDA f32 [m, out]."""
        import torch
        x = x.contiguous()
        y = torch.empty((x.shape[0], self.out_features), dtype=torch.float32, device=x.device)
        self.run_ptr(x.data_ptr(), x.shape[0], y.data_ptr(),
                     torch.cuda.current_stream(x.device).cuda_stream)
        return y

    def close(self):
        if getattr(self, "handle", None):
            lib().mc_linear_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
