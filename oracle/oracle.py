"""ctypes binding of the CPU parity oracle (``libmc_oracle.so``).

TEST INFRASTRUCTURE ONLY: the oracle is the checker.  Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / reference arm
import this module.  The CUDA product path never does.

The oracle restates modelc's Rust hot path (``src/runtime/transformer.rs``,
``src/generate.rs``, ``src/draft.rs``) in C; see ``mc_oracle.h``.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "libmc_oracle.so")

MODE_REFERENCE = 0
MODE_GENERAL = 1
DRAFT_NGRAM, DRAFT_LLAMA, DRAFT_MLP, DRAFT_NONE = 0, 1, 2, 3

_fp = C.POINTER(C.c_float)
_u32p = C.POINTER(C.c_uint32)


class Layer(C.Structure):
    _fields_ = [(n, _fp) for n in ("attn_norm", "wq", "wk", "wv", "wo",
                                    "mlp_norm", "wg", "wu", "wd")]


class Model(C.Structure):
    _fields_ = [("mode", C.c_int), ("n_layers", C.c_int), ("hidden", C.c_int),
                ("n_heads", C.c_int), ("n_kv_heads", C.c_int),
                ("head_dim", C.c_int), ("ffn", C.c_int), ("vocab", C.c_int),
                ("rope_base", C.c_float), ("eps", C.c_float),
                ("embed", _fp), ("final_norm", _fp), ("lm_head", _fp),
                ("layers", C.POINTER(Layer)), ("n_threads", C.c_int)]


class KV(C.Structure):
    _fields_ = [("n_layers", C.c_int), ("kv_dim", C.c_int), ("len", C.c_int),
                ("cap", C.c_int), ("k", _fp), ("v", _fp), ("mode", C.c_int),
                ("window", C.c_int), ("hot", C.c_int)]


KV_FP32, KV_INT8, KV_MIXED = 0, 1, 2  # KvLayer variants (transformer.rs:167-193)


class MlpDraft(C.Structure):
    _fields_ = [("vocab", C.c_int), ("hidden", C.c_int),
                ("draft_hidden", C.c_int), ("embed", _fp), ("w1", _fp),
                ("b1", _fp), ("w2", _fp), ("b2", _fp),
                ("temperature", C.c_float), ("top_p", C.c_float)]


class GenCfg(C.Structure):
    _fields_ = [("max_tokens", C.c_int), ("temperature", C.c_float),
                ("top_p", C.c_float), ("min_p", C.c_float), ("gamma", C.c_int),
                ("seed", C.c_uint64), ("tok_vocab", C.c_int),
                ("bonus", C.c_int), ("cancel", C.POINTER(C.c_int)),
                ("max_context", C.c_int), ("anchor_tokens", C.c_int), ("kv_mode", C.c_int)]


def build() -> str:
    """Compile the oracle with its Makefile (strict IEEE flags)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH) or (
                os.path.getmtime(_LIB_PATH) < os.path.getmtime(os.path.join(_HERE, "mc_oracle.c"))):
            build()
        L = C.CDLL(_LIB_PATH)
        L.oracle_argmax.restype = C.c_int
        L.oracle_rand_f32.restype = C.c_float
        L.oracle_rand_f32.argtypes = [C.c_uint64]
        L.oracle_multinomial.restype = C.c_uint32
        L.oracle_multinomial.argtypes = [_fp, C.c_int, C.c_uint64, C.c_uint64]
        L.oracle_sample.restype = C.c_uint32
        L.oracle_sample.argtypes = [_fp, C.c_int, C.c_float, C.c_float, C.c_float,
                                    C.c_uint64, C.c_uint64]
        L.oracle_chacha_block.argtypes = [_u32p, C.c_uint64, C.c_uint64, C.c_int, _u32p]
        L.oracle_f16_to_f32.restype = C.c_float
        L.oracle_f16_to_f32.argtypes = [C.c_uint16]
        L.oracle_f32_to_f16.restype = C.c_uint16
        L.oracle_f32_to_f16.argtypes = [C.c_float]
        L.oracle_kv_new.restype = C.POINTER(KV)
        L.oracle_kv_new.argtypes = [C.c_int, C.c_int, C.c_int]
        L.oracle_kv_free.argtypes = [C.POINTER(KV)]
        L.oracle_kv_truncate.argtypes = [C.POINTER(KV), C.c_int]
        L.oracle_kv_len.argtypes = [C.POINTER(KV)]
        L.oracle_kv_set_mode.argtypes = [C.POINTER(KV), C.c_int, C.c_int]
        L.oracle_kv_qdq.argtypes = [_fp, C.c_int]
        L.oracle_kv_shift.argtypes = [C.POINTER(KV), C.c_int, C.c_int]
        L.oracle_context_shift.restype = C.c_int
        L.oracle_context_shift.argtypes = [_u32p, C.POINTER(C.c_int), C.POINTER(C.c_int),
                                           C.POINTER(KV), C.c_int, C.c_int,
                                           C.POINTER(C.c_int)]
        L.oracle_model_resolve.argtypes = [C.POINTER(Model)]
        L.oracle_forward.argtypes = [C.POINTER(Model), _fp, C.POINTER(KV), _fp]
        L.oracle_forward_ids.argtypes = [C.POINTER(Model), _u32p, C.c_int,
                                         C.POINTER(KV), _fp]
        L.oracle_llama_draft_new.restype = C.c_void_p
        L.oracle_llama_draft_new.argtypes = [C.POINTER(Model), C.c_int]
        L.oracle_llama_draft_free.argtypes = [C.c_void_p]
        L.oracle_llama_draft_run.argtypes = [C.c_void_p, _u32p, C.c_int, C.c_int, _u32p]
        L.oracle_mlp_draft_run.argtypes = [C.POINTER(MlpDraft), _u32p, C.c_int,
                                           C.c_int, _u32p]
        L.oracle_ngram_draft.argtypes = [_u32p, C.c_int, _u32p, C.c_int, C.c_int,
                                         C.c_int, _u32p]
        L.oracle_generate_core.argtypes = [C.POINTER(Model), _u32p, C.c_int,
                                           C.POINTER(GenCfg), _u32p, C.c_int]
        L.oracle_speculative_generate.argtypes = [
            C.POINTER(Model), C.c_int, C.c_void_p, _u32p, C.c_int,
            C.POINTER(GenCfg), _u32p, C.c_int, C.POINTER(C.c_int),
            C.POINTER(C.c_int), C.c_int]
        L.oracle_speculative_generate_kv.argtypes = [
            C.POINTER(Model), C.c_int, C.c_void_p, _u32p, C.c_int,
            C.POINTER(GenCfg), _u32p, C.c_int, C.POINTER(C.c_int),
            C.POINTER(C.c_int), C.c_int, C.POINTER(KV), C.c_int]
        L.oracle_philox4x32_10.argtypes = [_u32p, _u32p, _u32p]
        L.oracle_philox_uniform.restype = C.c_float
        L.oracle_philox_uniform.argtypes = [C.c_uint64, C.c_uint32, C.c_uint32]
        L.oracle_filtered_weights.restype = C.c_float
        L.oracle_filtered_weights.argtypes = [_fp, C.c_int, C.c_float, C.c_float, C.c_float,
                                              _fp]
        L.oracle_sample_philox.restype = C.c_uint32
        L.oracle_sample_philox.argtypes = [_fp, C.c_int, C.c_float, C.c_float, C.c_float,
                                           C.c_uint64, C.c_uint32, C.c_uint32]
        L.oracle_speculative_sample.argtypes = [
            C.POINTER(Model), C.c_void_p, _u32p, C.c_int, C.POINTER(GenCfg), C.c_int, _u32p,
            C.c_int, C.POINTER(C.c_int), C.POINTER(C.c_int), C.c_int]
        _lib = L
    return _lib


def fptr(a: np.ndarray | None):
    if a is None:
        return None
    assert a.dtype == np.float32 and a.flags.c_contiguous
    return a.ctypes.data_as(_fp)


def u32ptr(a: np.ndarray):
    assert a.dtype == np.uint32 and a.flags.c_contiguous
    return a.ctypes.data_as(_u32p)


def f32(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.float32))


# ---------------------------------------------------------------- numerics
def linear(w, x, bias=None):
    w, x = f32(w), f32(x)
    out = np.empty(w.shape[0], np.float32)
    lib().oracle_linear(fptr(w), w.shape[0], w.shape[1],
                        fptr(f32(bias)) if bias is not None else None, fptr(x), fptr(out))
    return out


def linear_par(w, x, n_threads=8):
    w, x = f32(w), f32(x)
    out = np.empty(w.shape[0], np.float32)
    lib().oracle_linear_par(fptr(w), w.shape[0], w.shape[1], fptr(x), fptr(out), n_threads)
    return out


def rms_norm(x, w, eps):
    x, w = f32(x), f32(w)
    out = np.empty_like(x)
    lib().oracle_rms_norm(fptr(x), len(x), fptr(w), len(w), C.c_float(eps), fptr(out))
    return out


def silu(x):
    x = f32(x)
    out = np.empty_like(x)
    lib().oracle_silu(fptr(x), len(x), fptr(out))
    return out


def add(a, b):
    a, b = f32(a), f32(b)
    out = np.empty(max(len(a), len(b)), np.float32)
    lib().oracle_add(fptr(a), len(a), fptr(b), len(b), fptr(out))
    return out


def rope(x, pos, n_heads, base=10000.0):
    x = f32(x)
    out = np.empty_like(x)
    lib().oracle_rope(fptr(x), len(x), pos, n_heads, C.c_float(base), fptr(out))
    return out


def rope_table(max_pos, head_dim, base):
    half = head_dim // 2
    c = np.empty((max_pos, half), np.float32)
    s = np.empty((max_pos, half), np.float32)
    lib().oracle_rope_table(max_pos, head_dim, C.c_float(base), fptr(c), fptr(s))
    return c, s


def attention_kv(q, k_all, v_all, n_heads, n_kv_heads=None):
    q, k_all, v_all = f32(q), f32(k_all), f32(v_all)
    n_kv = n_heads if n_kv_heads is None else n_kv_heads
    hd = max(len(q) // max(n_heads, 1), 1)
    seq = len(k_all) // max(n_kv * hd, 1)
    out = np.empty(len(q), np.float32)
    lib().oracle_attention_kv(fptr(q), len(q), fptr(k_all), fptr(v_all), seq,
                              n_heads, n_kv, fptr(out))
    return out


def softmax_inplace(x):
    x = f32(x).copy()
    lib().oracle_softmax_inplace(fptr(x), len(x))
    return x


def argmax(x):
    x = f32(x)
    return lib().oracle_argmax(fptr(x), len(x))


def softmax(x):
    x = f32(x)
    out = np.empty_like(x)
    lib().oracle_softmax(fptr(x), len(x), fptr(out))
    return out


def apply_top_p(p, top_p):
    p = f32(p).copy()
    lib().oracle_apply_top_p(fptr(p), len(p), C.c_float(top_p))
    return p


def apply_min_p(p, min_p):
    p = f32(p).copy()
    lib().oracle_apply_min_p(fptr(p), len(p), C.c_float(min_p))
    return p


def multinomial(p, step, seed):
    p = f32(p)
    return lib().oracle_multinomial(fptr(p), len(p), step, seed)


def sample(logits, temperature, step, seed, top_p=0.0, min_p=0.0):
    logits = f32(logits)
    return lib().oracle_sample(fptr(logits), len(logits), temperature, top_p,
                               min_p, step, seed)


def chacha_block(key, counter=0, nonce=0, rounds=20):
    k = np.ascontiguousarray(np.asarray(key, np.uint32))
    out = np.empty(16, np.uint32)
    lib().oracle_chacha_block(u32ptr(k), counter, nonce, rounds, u32ptr(out))
    return out


# ---------------------------------------------------------------- weights
def quantize_int8_tensor(x):
    x = f32(x)
    q = np.empty(x.shape, np.int8)
    s = C.c_float()
    lib().oracle_quantize_int8_tensor(fptr(x), C.c_size_t(x.size),
                                      q.ctypes.data_as(C.c_void_p), C.byref(s))
    return q, s.value


def quantize_int8_rows(x):
    x = f32(x)
    q = np.empty(x.shape, np.int8)
    s = np.empty(x.shape[0], np.float32)
    lib().oracle_quantize_int8_rows(fptr(x), x.shape[0], x.shape[1],
                                    q.ctypes.data_as(C.c_void_p), fptr(s))
    return q, s


def dequant_int8_rows(q, scales):
    q = np.ascontiguousarray(q, np.int8)
    scales = f32(scales)
    out = np.empty(q.shape, np.float32)
    lib().oracle_dequant_int8_rows(q.ctypes.data_as(C.c_void_p), fptr(scales),
                                   q.shape[0], q.shape[1], fptr(out))
    return out


def quantize_q4_0(x):
    x = f32(x)
    blocks = np.empty(x.size // 32 * 18, np.uint8)
    rc = lib().oracle_quantize_q4_0(fptr(x), C.c_size_t(x.size),
                                    blocks.ctypes.data_as(C.c_void_p))
    assert rc == 0
    return blocks


def dequant_q4_0(blocks, n):
    blocks = np.ascontiguousarray(blocks, np.uint8)
    out = np.empty(n, np.float32)
    rc = lib().oracle_dequant_q4_0(blocks.ctypes.data_as(C.c_void_p), C.c_size_t(n), fptr(out))
    assert rc == 0
    return out


# ---------------------------------------------------------------- model
class OracleModel:
    """An oracle model over dequantized f32 numpy weights.

    ``weights`` maps reference tensor names (``model.layers.{i}.self_attn.
    q_proj.weight`` ...) to f32 arrays; missing tensors follow the reference's
    Option semantics (no norm -> identity, no head -> no logits).
    """

    def __init__(self, weights: dict, n_layers, hidden, vocab, ffn, *,
                 mode=MODE_REFERENCE, n_heads=0, n_kv_heads=0, head_dim=0,
                 rope_base=10000.0, eps=1e-6, n_threads=1):
        self._keep = []
        g = lambda k: self._arr(weights.get(k))
        layers = (Layer * max(n_layers, 1))()
        for i in range(n_layers):
            p = f"model.layers.{i}."
            layers[i] = Layer(
                g(p + "input_layernorm.weight"), g(p + "self_attn.q_proj.weight"),
                g(p + "self_attn.k_proj.weight"), g(p + "self_attn.v_proj.weight"),
                g(p + "self_attn.o_proj.weight"), g(p + "post_attention_layernorm.weight"),
                g(p + "mlp.gate_proj.weight"), g(p + "mlp.up_proj.weight"),
                g(p + "mlp.down_proj.weight"))
        self._layers = layers
        self.m = Model(mode, n_layers, hidden, n_heads, n_kv_heads, head_dim, ffn,
                       vocab, rope_base, eps, g("model.embed_tokens.weight"),
                       g("model.norm.weight"), g("lm_head.weight"), layers, n_threads)
        rc = lib().oracle_model_resolve(C.byref(self.m))
        if rc != 0:
            raise ValueError("oracle: unsupported head geometry for this mode")

    def _arr(self, a):
        if a is None:
            return None
        a = f32(a)
        self._keep.append(a)
        return fptr(a)

    @property
    def kv_dim(self):
        return self.m.n_kv_heads * self.m.head_dim

    def new_kv(self, cap):
        return OracleKV(self, cap)

    def forward_ids(self, ids, kv=None):
        ids = np.ascontiguousarray(np.asarray(ids, np.uint32))
        out = np.empty((len(ids), self.m.vocab), np.float32)
        have = lib().oracle_forward_ids(C.byref(self.m), u32ptr(ids), len(ids),
                                        kv.ptr if kv is not None else None, fptr(out))
        return out if have else None

    def forward_embedding(self, x, kv=None):
        x = f32(x)
        out = np.empty(self.m.vocab, np.float32)
        have = lib().oracle_forward(C.byref(self.m), fptr(x),
                                    kv.ptr if kv is not None else None, fptr(out))
        return out if have else None

    def _cfg(self, max_tokens, temperature, gamma, seed, top_p, min_p, tok_vocab, bonus,
             max_context=0, anchor_tokens=0, kv_mode=KV_FP32):
        return GenCfg(max_tokens, temperature, top_p, min_p, gamma, seed, tok_vocab,
                      bonus, None, max_context, anchor_tokens, kv_mode)

    def generate_core(self, prompt, max_tokens, temperature=0.0, seed=0,
                      top_p=0.0, min_p=0.0, tok_vocab=0):
        prompt = np.ascontiguousarray(np.asarray(prompt, np.uint32))
        cfg = self._cfg(max_tokens, temperature, 0, seed, top_p, min_p, tok_vocab, 0)
        out = np.zeros(max_tokens + 1, np.uint32)
        n = lib().oracle_generate_core(C.byref(self.m), u32ptr(prompt), len(prompt),
                                       C.byref(cfg), u32ptr(out), len(out))
        return out[:n].tolist()

    def speculative_generate(self, prompt, max_tokens, gamma, draft=None,
                             temperature=0.0, seed=0, top_p=0.0, min_p=0.0,
                             tok_vocab=0, bonus=False, max_context=0, anchor_tokens=0,
                             kv_mode=KV_FP32, rounds_cap=None, kv=None, matched_len=0):
        """Returns (tokens, accepted-per-round).  max_context / anchor_tokens:
        the context shift (0: none); kv_mode: KV_FP32, KV_INT8 or KV_MIXED.
        kv (an OracleKV, its mode set): the cache holding the first
        matched_len prompt tokens' K/V (a prefix-cache hit), which ends the
        run holding the final cache."""
        prompt = np.ascontiguousarray(np.asarray(prompt, np.uint32))
        cfg = self._cfg(max_tokens, temperature, gamma, seed, top_p, min_p,
                        tok_vocab, int(bonus), max_context, anchor_tokens, kv_mode)
        cap = max_tokens + gamma + 2
        out = np.zeros(cap, np.uint32)
        rounds_cap = rounds_cap or cap + 1
        acc = (C.c_int * rounds_cap)()
        nr = C.c_int()
        if draft is None:
            kind, ptr = DRAFT_NGRAM, None
        else:
            kind, ptr = draft.kind, draft.handle
        n = lib().oracle_speculative_generate_kv(C.byref(self.m), kind, ptr, u32ptr(prompt),
                                                 len(prompt), C.byref(cfg), u32ptr(out), cap,
                                                 acc, C.byref(nr), rounds_cap,
                                                 kv.ptr if kv is not None else None,
                                                 matched_len)
        return out[:n].tolist(), [acc[i] for i in range(min(nr.value, rounds_cap))]


    def speculative_sample(self, prompt, max_tokens, gamma, draft, temperature, seed,
                           accept_mode=0, bonus=False, top_p=0.0, min_p=0.0):
        """Stochastic speculative decoding with a sampling transformer draft
        (accept_mode 0: min(1, p/q) with residual resampling; 1: the
        reference's target-sample == draft rule), every distribution after
        top-p and min-p as filtered_weights states them.  Returns (tokens,
        accepted)."""
        prompt = np.ascontiguousarray(np.asarray(prompt, np.uint32))
        cfg = self._cfg(max_tokens, temperature, gamma, seed, top_p, min_p, 0, int(bonus))
        cap = max_tokens + gamma + 2
        out = np.zeros(cap, np.uint32)
        acc = (C.c_int * (cap + 1))()
        nr = C.c_int()
        n = lib().oracle_speculative_sample(C.byref(self.m), draft.handle, u32ptr(prompt),
                                            len(prompt), C.byref(cfg), accept_mode,
                                            u32ptr(out), cap, acc, C.byref(nr), cap + 1)
        return out[:n].tolist(), [acc[i] for i in range(min(nr.value, cap + 1))]


def philox4x32_10(ctr, key):
    c = np.ascontiguousarray(np.asarray(ctr, np.uint32))
    k = np.ascontiguousarray(np.asarray(key, np.uint32))
    o = np.zeros(4, np.uint32)
    lib().oracle_philox4x32_10(u32ptr(c), u32ptr(k), u32ptr(o))
    return o.tolist()


def philox_uniform(seed, rnd, slot):
    return float(lib().oracle_philox_uniform(seed, rnd, slot))


def filtered_weights(logits, temperature, top_p=0.0, min_p=0.0):
    """exp((l - max) / T) with the top-p and min-p filters applied
    (mc_oracle.c oracle_filtered_weights); returns (weights, their sum)."""
    logits = np.ascontiguousarray(logits, dtype=np.float32)
    w = np.empty_like(logits)
    s = lib().oracle_filtered_weights(fptr(logits), len(logits), temperature, top_p, min_p,
                                      fptr(w))
    return w, float(s)


def kv_qdq(x):
    """A token's K or V as an int8 KvLayer returns it (quantize_scale, quantize,
    then q * scale)."""
    x = np.array(f32(x), copy=True)
    lib().oracle_kv_qdq(fptr(x), len(x))
    return x


def context_shift(tokens, prompt_len, max_ctx, anchor, kv=None):
    """generate.rs:26-63 on a token list (and optionally an OracleKV):
    returns (tokens, prompt_len, overflow, removed_at)."""
    t = np.ascontiguousarray(np.asarray(tokens, np.uint32)).copy()
    n, pl, at = C.c_int(len(t)), C.c_int(prompt_len), C.c_int(0)
    ov = lib().oracle_context_shift(u32ptr(t), C.byref(n), C.byref(pl),
                                    kv.ptr if kv is not None else None, max_ctx, anchor,
                                    C.byref(at))
    return t[:n.value].tolist(), pl.value, ov, at.value


def sample_philox(logits, temperature, seed, rnd, slot, top_p=0.0, min_p=0.0):
    """One token of logits after the filters, with the Philox uniform of
    (seed, rnd, slot); greedy at temperature <= 0."""
    logits = np.ascontiguousarray(logits, dtype=np.float32)
    return int(lib().oracle_sample_philox(fptr(logits), len(logits), temperature, top_p,
                                          min_p, seed, rnd, slot))


class OracleKV:
    def __init__(self, model: OracleModel | None, cap: int, n_layers=None, kv_dim=None):
        self.ptr = lib().oracle_kv_new(model.m.n_layers if model else n_layers,
                                       model.kv_dim if model else kv_dim, cap)
        self._model = model

    def __len__(self):
        return lib().oracle_kv_len(self.ptr)

    def truncate(self, n):
        lib().oracle_kv_truncate(self.ptr, n)

    def set_mode(self, mode, window=64):
        """The KvLayer variant of every layer (KV_FP32 / KV_INT8 / KV_MIXED)."""
        lib().oracle_kv_set_mode(self.ptr, mode, window)

    def append(self, k, v):
        """KvLayer::append of one token's k and v (kv_dim values each) to every
        layer: the slot is written, then quantized as the variant does."""
        kv = self.ptr.contents
        assert kv.len < kv.cap
        ka = np.ctypeslib.as_array(kv.k, shape=(kv.n_layers * kv.cap * kv.kv_dim,))
        va = np.ctypeslib.as_array(kv.v, shape=(kv.n_layers * kv.cap * kv.kv_dim,))
        pos = kv.len
        # the token an INT8 layer quantizes now, or the one a MIXED layer moves cold
        quantized = []
        if kv.mode == KV_INT8:
            quantized = [pos]
        elif kv.mode == KV_MIXED and kv.hot + 1 > kv.window:
            quantized = [pos - kv.window]
        for layer in range(kv.n_layers):
            base = (layer * kv.cap + pos) * kv.kv_dim
            ka[base: base + kv.kv_dim] = f32(k)
            va[base: base + kv.kv_dim] = f32(v)
            for p in quantized:
                o = (layer * kv.cap + p) * kv.kv_dim
                for a in (ka, va):
                    a[o: o + kv.kv_dim] = kv_qdq(a[o: o + kv.kv_dim])
        kv.len = pos + 1
        if kv.mode == KV_MIXED and kv.hot < kv.window:
            kv.hot += 1

    def shift(self, n, anchor=0):
        """KvCache::shift (anchor 0) / shift_anchored."""
        lib().oracle_kv_shift(self.ptr, n, anchor)

    def layer_k(self, layer):
        kv = self.ptr.contents
        base = layer * kv.cap * kv.kv_dim
        return np.ctypeslib.as_array(kv.k, shape=(kv.n_layers * kv.cap * kv.kv_dim,))[
            base: base + kv.len * kv.kv_dim].reshape(kv.len, kv.kv_dim).copy()

    def layer_v(self, layer):
        kv = self.ptr.contents
        base = layer * kv.cap * kv.kv_dim
        return np.ctypeslib.as_array(kv.v, shape=(kv.n_layers * kv.cap * kv.kv_dim,))[
            base: base + kv.len * kv.kv_dim].reshape(kv.len, kv.kv_dim).copy()

    def __del__(self):
        try:
            lib().oracle_kv_free(self.ptr)
        except Exception:
            pass


class OracleLlamaDraft:
    kind = DRAFT_LLAMA

    def __init__(self, model: OracleModel, cap: int):
        self.model = model
        self.handle = lib().oracle_llama_draft_new(C.byref(model.m), cap)

    def draft(self, context, gamma):
        ctx = np.ascontiguousarray(np.asarray(context, np.uint32))
        out = np.zeros(max(gamma, 1), np.uint32)
        n = lib().oracle_llama_draft_run(self.handle, u32ptr(ctx), len(ctx), gamma, u32ptr(out))
        return out[:n].tolist()

    def __del__(self):
        try:
            lib().oracle_llama_draft_free(self.handle)
        except Exception:
            pass


class OracleMlpDraft:
    kind = DRAFT_MLP

    def __init__(self, embed, w1, b1, w2, b2, temperature=0.0, top_p=0.0):
        self._keep = [f32(a) for a in (embed, w1, b1, w2, b2)]
        e, a1, c1, a2, c2 = self._keep
        self.s = MlpDraft(a2.shape[0], e.shape[1], a1.shape[0], fptr(e), fptr(a1),
                          fptr(c1), fptr(a2), fptr(c2), temperature, top_p)
        self.handle = C.cast(C.pointer(self.s), C.c_void_p)

    def draft(self, context, gamma):
        ctx = np.ascontiguousarray(np.asarray(context, np.uint32))
        out = np.zeros(max(gamma, 1), np.uint32)
        n = lib().oracle_mlp_draft_run(C.byref(self.s), u32ptr(ctx), len(ctx), gamma, u32ptr(out))
        return out[:n].tolist()


class OracleNoDraft:
    kind = DRAFT_NONE
    handle = None


def ngram_draft(tokens, context, gamma, n=3):
    t = np.ascontiguousarray(np.asarray(tokens, np.uint32))
    c = np.ascontiguousarray(np.asarray(context, np.uint32))
    out = np.zeros(max(gamma, 1), np.uint32)
    k = lib().oracle_ngram_draft(u32ptr(t), len(t), u32ptr(c), len(c), n, gamma, u32ptr(out))
    return out[:k].tolist()
