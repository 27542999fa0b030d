"""Shared test fixtures: reference test models and a float64 cross-check.

The Llama fixture restates the reference's own test model
(tests/common/mod.rs:188-196 fp32_matrix / fp32_vector, :278-358
create_llama_test_model): one layer, hidden 12, FFN 48, vocab 10, matrix
entries (i % 7) - 3, norm weights 1.0.
"""
from __future__ import annotations

import numpy as np

LLAMA_HIDDEN, LLAMA_INTER, LLAMA_VOCAB = 12, 48, 10


def fp32_matrix(rows, cols):
    """tests/common/mod.rs:188-192: element i = (i as f32 % 7.0) - 3.0."""
    i = np.arange(rows * cols, dtype=np.float32)
    return (np.fmod(i, np.float32(7.0)) - np.float32(3.0)).reshape(rows, cols)


def fp32_vector(n, fill):
    return np.full(n, fill, np.float32)


def reference_llama_fixture():
    """tests/common/mod.rs:278-358 create_llama_test_model (f32 tensors)."""
    h, f, v = LLAMA_HIDDEN, LLAMA_INTER, LLAMA_VOCAB
    w = {
        "model.layers.0.input_layernorm.weight": fp32_vector(h, 1.0),
        "model.layers.0.self_attn.q_proj.weight": fp32_matrix(h, h),
        "model.layers.0.self_attn.k_proj.weight": fp32_matrix(h, h),
        "model.layers.0.self_attn.v_proj.weight": fp32_matrix(h, h),
        "model.layers.0.self_attn.o_proj.weight": fp32_matrix(h, h),
        "model.layers.0.post_attention_layernorm.weight": fp32_vector(h, 1.0),
        "model.layers.0.mlp.gate_proj.weight": fp32_matrix(f, h),
        "model.layers.0.mlp.up_proj.weight": fp32_matrix(f, h),
        "model.layers.0.mlp.down_proj.weight": fp32_matrix(h, f),
        "model.embed_tokens.weight": fp32_matrix(v, h),
        "model.norm.weight": fp32_vector(h, 1.0),
        "lm_head.weight": fp32_matrix(v, h),
    }
    return w


def f64_forward_seq(w, ids, n_layers, n_heads, n_kv, head_dim, base, eps):
    """Float64 restatement of transformer.rs:64-96 over a token sequence
    (causal attention, RoPE at each position).  Returns logits [n, vocab]."""
    d = w["model.embed_tokens.weight"].shape[1]
    x = np.stack([w["model.embed_tokens.weight"][i].astype(np.float64) for i in ids])
    n = len(ids)
    half = head_dim // 2
    pos = np.arange(n, dtype=np.float64)[:, None]
    inv = base ** (-(np.arange(half, dtype=np.float64)) / half)
    ang = pos * inv[None, :]
    cos, sin = np.cos(ang), np.sin(ang)

    def rms(h, wt):
        return h / np.sqrt((h * h).mean(-1, keepdims=True) + eps) * wt

    def rope(t, nh):
        t = t.reshape(n, nh, head_dim).copy()
        a, b = t[..., :half].copy(), t[..., half:2 * half].copy()
        t[..., :half] = a * cos[:, None, :] - b * sin[:, None, :]
        t[..., half:2 * half] = a * sin[:, None, :] + b * cos[:, None, :]
        return t

    for l in range(n_layers):
        p = f"model.layers.{l}."
        g = lambda k: w[p + k].astype(np.float64)
        hn = rms(x, g("input_layernorm.weight"))
        q = rope(hn @ g("self_attn.q_proj.weight").T, n_heads)
        k = rope(hn @ g("self_attn.k_proj.weight").T, n_kv)
        v = (hn @ g("self_attn.v_proj.weight").T).reshape(n, n_kv, head_dim)
        grp = n_heads // n_kv
        o = np.zeros((n, n_heads, head_dim))
        for hh in range(n_heads):
            s = q[:, hh] @ k[:, hh // grp].T / np.sqrt(head_dim)
            s = s + np.triu(np.full((n, n), -np.inf), 1)
            s = np.exp(s - s.max(-1, keepdims=True))
            s = s / s.sum(-1, keepdims=True)
            o[:, hh] = s @ v[:, hh // grp]
        x = x + o.reshape(n, -1) @ g("self_attn.o_proj.weight").T
        hn = rms(x, g("post_attention_layernorm.weight"))
        gt = hn @ g("mlp.gate_proj.weight").T
        up = hn @ g("mlp.up_proj.weight").T
        x = x + (gt / (1 + np.exp(-gt)) * up) @ g("mlp.down_proj.weight").T
    x = rms(x, w["model.norm.weight"].astype(np.float64))
    head = w.get("lm_head.weight", w["model.embed_tokens.weight"]).astype(np.float64)
    return x @ head.T
