"""Host API mirroring modelc's generation interface over the C ABI.

Names follow the reference: ``GenerationConfig`` (generate.rs:65-167),
``speculative_generate`` (generate.rs:598-767), ``forward_llama_cached``
(transformer.rs:64-96, batched here), ``DraftModel.draft`` (draft.rs:18-21).
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np

from . import _lib
from ._lib import check, lib
from .model import Weights


@dataclass
class GenerationConfig:
    """The speculative-path subset of generate.rs:65-167 (defaults :146-167)."""
    max_tokens: int = 128
    temperature: float = 0.0
    gamma: int = 0
    seed: int = 0
    bonus: bool = False   # False: the reference verify (no bonus token)
    accept_mode: int = 0  # temperature > 0: 0 = min(1, p/q), 1 = sample == draft
    top_p: float = 0.0    # temperature > 0: applied when in (0, 1) (generate.rs:961-963)
    min_p: float = 0.0    # temperature > 0: applied when in (0, 1) (generate.rs:964-966)
    max_context: int = 0  # the context shift's threshold (None = 0)
    anchor_tokens: int = 0
    use_int8_kv: bool = False
    use_mixed_kv: bool = False


# target KV variants (make_kv_cache, generate.rs:17-24)
KV_FP32, KV_INT8, KV_MIXED = 0, 1, 2


def _u32(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.uint32))


class Session:
    """Device state of n_requests concurrent requests (default one): target
    KV, draft KV and speculative state per request.  ``draft`` is the
    drafter of the rounds: a transformer draft (Weights), an MlpDraftModel,
    or None for the reference's trigram n-gram drafter.

    Mirrors the reference's per-request ``Option<KvCache>`` (generate.rs:
    617-627) plus the draft model's cache; a batched session decodes its
    requests in lock step, each exactly as it would decode alone.
    ``max_context`` is the KV capacity; ``shift_context`` / ``anchor_tokens``
    are GenerationConfig::max_context / anchor_tokens (the context shift,
    generate.rs:26-63); ``kv_mode`` the target cache variant (KV_FP32,
    KV_INT8 or KV_MIXED)."""

    def __init__(self, target: Weights, draft=None, gamma: int = 4,
                 max_context: int = 2048, bonus: bool = False, temperature: float = 0.0,
                 seed: int = 0, accept_mode: int = 0, n_requests: int = 1,
                 top_p: float = 0.0, min_p: float = 0.0, shift_context: int = 0,
                 anchor_tokens: int = 0, kv_mode: int = KV_FP32):
        self.target, self.draft = target, draft
        self.gamma = gamma
        self.n_requests = n_requests
        self._cancel = C.c_int32(0)
        cfg = _lib.SpecCfg(gamma, max_context, int(bonus), temperature, seed,
                           C.pointer(self._cancel), accept_mode, n_requests, top_p, min_p,
                           shift_context, anchor_tokens, kv_mode)
        h = C.c_void_p()
        if isinstance(draft, MlpDraftModel):  # MlpDraftModel drives the rounds
            check(lib().mc_session_create_mlp(target.handle, draft.handle, C.byref(cfg),
                                              C.byref(h)))
        else:  # a transformer draft, or None: the reference's trigram drafter
            check(lib().mc_session_create(target.handle, draft.handle if draft else None,
                                          C.byref(cfg), C.byref(h)))
        self.handle = h

    # -- forward_llama_cached (batched) ------------------------------------
    def forward(self, ids, logits: bool = True):
        """Forward ids at the current KV length; returns [n, vocab] logits."""
        ids = _u32(ids)
        out = np.empty((len(ids), self.target.cfg.vocab), np.float32) if logits else None
        check(lib().mc_forward(self.handle, ids.ctypes.data_as(C.POINTER(C.c_uint32)), len(ids),
                               out.ctypes.data_as(C.POINTER(C.c_float)) if logits else None))
        return out

    def draft_forward(self, ids, logits: bool = True):
        ids = _u32(ids)
        out = np.empty((len(ids), self.draft.cfg.vocab), np.float32) if logits else None
        check(lib().mc_draft_forward(self.handle, ids.ctypes.data_as(C.POINTER(C.c_uint32)),
                                     len(ids),
                                     out.ctypes.data_as(C.POINTER(C.c_float)) if logits else None))
        return out

    def kv_len(self) -> int:
        return int(lib().mc_kv_len(self.handle))

    def kv_truncate(self, n: int):
        check(lib().mc_kv_truncate(self.handle, n))

    # -- DraftModel::draft ---------------------------------------------------
    def draft_tokens(self, context, gamma: int):
        ctx = _u32(context)
        out = np.zeros(max(gamma, 1), np.uint32)
        n = C.c_int32()
        check(lib().mc_draft(self.handle, ctx.ctypes.data_as(C.POINTER(C.c_uint32)), len(ctx),
                             gamma, out.ctypes.data_as(C.POINTER(C.c_uint32)), C.byref(n)))
        return out[: n.value].tolist()

    # -- speculative_generate ------------------------------------------------
    def speculative_generate(self, prompt, max_tokens: int):
        """Returns (generated ids, accepted-draft count per round)."""
        p = _u32(prompt)
        cap = max_tokens + self.gamma + 2
        out = np.zeros(cap, np.uint32)
        acc = np.zeros(cap + 1, np.int32)
        n_out, n_rounds = C.c_int32(), C.c_int32()
        check(lib().mc_speculative_generate(
            self.handle, p.ctypes.data_as(C.POINTER(C.c_uint32)), len(p), max_tokens,
            out.ctypes.data_as(C.POINTER(C.c_uint32)), cap, C.byref(n_out),
            acc.ctypes.data_as(C.POINTER(C.c_int32)), len(acc), C.byref(n_rounds)))
        return out[: n_out.value].tolist(), acc[: min(n_rounds.value, len(acc))].tolist()

    def speculative_generate_batch(self, prompts, max_tokens: int):
        """Batched speculative_generate over this session's n_requests
        prompts; returns one (generated ids, accepted per round) per prompt."""
        p = _u32(np.concatenate([_u32(x) for x in prompts]))
        lens = np.ascontiguousarray([len(x) for x in prompts], dtype=np.int32)
        B = len(prompts)
        stride = max_tokens + self.gamma + 2
        out = np.zeros((B, stride), np.uint32)
        acc = np.zeros((B, stride + 1), np.int32)
        n_out = np.zeros(B, np.int32)
        n_rounds = np.zeros(B, np.int32)
        i32p = C.POINTER(C.c_int32)
        check(lib().mc_speculative_generate_batch(
            self.handle, p.ctypes.data_as(C.POINTER(C.c_uint32)), lens.ctypes.data_as(i32p), B,
            max_tokens, out.ctypes.data_as(C.POINTER(C.c_uint32)), stride,
            n_out.ctypes.data_as(i32p), acc.ctypes.data_as(i32p), stride + 1,
            n_rounds.ctypes.data_as(i32p)))
        return [(out[z, : n_out[z]].tolist(), acc[z, : min(n_rounds[z], stride + 1)].tolist())
                for z in range(B)]

    def prime(self, prompt):
        p = _u32(prompt)
        check(lib().mc_spec_prime(self.handle, p.ctypes.data_as(C.POINTER(C.c_uint32)), len(p)))

    def prime_cached(self, snapshot: "KvSnapshot", prompt):
        """prime() for a prompt that starts with the snapshot's tokens: their
        K/V are restored, the rest forwarded (generate.rs:617-636)."""
        p = _u32(prompt)
        check(lib().mc_spec_prime_cached(self.handle, snapshot.handle,
                                         p.ctypes.data_as(C.POINTER(C.c_uint32)), len(p)))

    def snapshot(self, request: int = 0) -> "KvSnapshot":
        """The request's context tokens and target K/V as they stand."""
        return KvSnapshot(self, request)

    def prime_batch(self, prompts):
        """Prime one prompt per request (n_requests of them)."""
        p = _u32(np.concatenate([_u32(x) for x in prompts]))
        lens = np.ascontiguousarray([len(x) for x in prompts], dtype=np.int32)
        check(lib().mc_spec_prime_batch(self.handle, p.ctypes.data_as(C.POINTER(C.c_uint32)),
                                        lens.ctypes.data_as(C.POINTER(C.c_int32)), len(prompts)))

    def decode(self, max_tokens: int) -> int:
        n = C.c_int32()
        check(lib().mc_spec_decode(self.handle, max_tokens, C.byref(n)))
        return n.value

    def read(self, cap: int = 1 << 16, request: int = 0):
        """(generated ids, accepted per round) of one request."""
        out = np.zeros(cap, np.uint32)
        acc = np.zeros(cap, np.int32)
        n_out, n_rounds = C.c_int32(), C.c_int32()
        check(lib().mc_spec_read_request(self.handle, request,
                                         out.ctypes.data_as(C.POINTER(C.c_uint32)), cap,
                                         C.byref(n_out), acc.ctypes.data_as(C.POINTER(C.c_int32)),
                                         cap, C.byref(n_rounds)))
        return out[: n_out.value].tolist(), acc[: min(n_rounds.value, cap)].tolist()

    def rewind(self):
        """Back to the primed prompt (its KV kept)."""
        check(lib().mc_spec_rewind(self.handle))

    def tp_init(self, unique_id: bytes, rank: int, world: int):
        """Join the tensor-parallel group (target weights loaded with the
        same tp_rank / tp_world); unique_id comes from tp_unique_id() on one
        rank, shared by the host."""
        check(lib().mc_session_tp_init(self.handle, bytes(unique_id), rank, world))

    def tp_ipc_handle(self) -> bytes:
        """64-byte IPC handle of this rank's reduce buffer (fused reduction)."""
        buf = C.create_string_buffer(64)
        check(lib().mc_session_tp_ipc_handle(self.handle, buf))
        return buf.raw

    def tp_open_peers(self, handles):
        """Open every rank's reduce buffer (handles in rank order); switches the
        row-parallel reductions from NCCL to the fused NVLink path."""
        blob = b"".join(bytes(h) for h in handles)
        check(lib().mc_session_tp_open_peers(self.handle, blob))

    def set_wait_timeout(self, ms: int):
        """Limit of every bounded device wait (a tensor-parallel peer's flag)."""
        check(lib().mc_session_set_wait_timeout(self.handle, ms))

    def set_seed(self, seed: int):
        """Seed of the stochastic rounds from the next round on."""
        check(lib().mc_spec_set_seed(self.handle, seed))

    def verify_launch(self, n: int):
        """Enqueue n verify forwards on the session stream (timing only)."""
        check(lib().mc_spec_verify_launch(self.handle, n))

    @property
    def stream_ptr(self) -> int:
        return int(lib().mc_session_stream(self.handle) or 0)

    @property
    def round_launches(self) -> int:
        return int(lib().mc_session_round_launches(self.handle))

    def cancel(self):
        """Raise the cancel flag: a running or later decode returns
        MC_E_CANCELLED at its next look (at most every 64 rounds)."""
        self._cancel.value = 1

    def uncancel(self):
        self._cancel.value = 0

    def close(self):
        if getattr(self, "handle", None):
            lib().mc_session_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def tp_unique_id() -> bytes:
    """128-byte id of a new tensor-parallel communicator (one rank calls it;
    the host distributes it)."""
    buf = C.create_string_buffer(128)
    check(lib().mc_tp_unique_id(buf))
    return buf.raw


class LlamaDraftModel:
    """A transformer drafter behind the reference's DraftModel trait
    (draft.rs:18-21): ``draft(context, gamma) -> list of ids``."""

    def __init__(self, target: Weights, draft: Weights, max_context: int = 2048):
        self.session = Session(target, draft, gamma=1, max_context=max_context)

    def draft(self, context, gamma: int):
        return self.session.draft_tokens(context, gamma)


class MlpDraftModel:
    """MlpDraftModel (draft.rs:28-147) on the device, greedy: ``tensors``
    maps the names MlpDraftModel::from_runtime looks up (draft.fc1.weight,
    draft.fc1.bias, draft.fc2.weight, draft.fc2.bias and draft.embed.weight or
    model.embed_tokens.weight) to f32 numpy arrays.  ``draft(context, gamma)``
    returns the reference's tokens bit for bit."""

    def __init__(self, tensors: dict, device: int = 0):
        from .model import QTensor, _desc_arrays
        qt = {k: QTensor("f32", np.ascontiguousarray(np.asarray(v, np.float32)))
              for k, v in tensors.items()}
        arr, n, self._keep = _desc_arrays(qt)
        h = C.c_void_p()
        check(lib().mc_mlp_draft_create(arr, n, device, C.byref(h)))
        self.handle = h

    def draft(self, context, gamma: int):
        ctx = _u32(context)
        out = np.zeros(max(gamma, 1), np.uint32)
        n = C.c_int32()
        check(lib().mc_mlp_draft(self.handle, ctx.ctypes.data_as(C.POINTER(C.c_uint32)),
                                 len(ctx), gamma, out.ctypes.data_as(C.POINTER(C.c_uint32)),
                                 C.byref(n)))
        return out[: n.value].tolist()

    def close(self):
        if getattr(self, "handle", None):
            lib().mc_mlp_draft_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class NgramDraftModel:
    """The n-gram drafter of speculative_generate (generate.rs:771-841) on
    the device: ``draft(tokens, gamma)`` drafts from the index of ``tokens``'
    windows of ``n`` tokens (ties: the continuation seen first)."""

    def __init__(self, n: int = 3, max_tokens: int = 1 << 16, device: int = 0):
        h = C.c_void_p()
        check(lib().mc_ngram_draft_create(n, max_tokens, device, C.byref(h)))
        self.handle = h

    def draft(self, tokens, gamma: int):
        t = _u32(tokens)
        out = np.zeros(max(gamma, 1), np.uint32)
        n = C.c_int32()
        check(lib().mc_ngram_draft(self.handle, t.ctypes.data_as(C.POINTER(C.c_uint32)), len(t),
                                   gamma, out.ctypes.data_as(C.POINTER(C.c_uint32)),
                                   C.byref(n)))
        return out[: n.value].tolist()

    def close(self):
        if getattr(self, "handle", None):
            lib().mc_ngram_draft_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class KvSnapshot:
    """A device copy of one request's context tokens and target K/V
    (CachedPrefix, prefix_cache.rs:14-24; last_logits are not kept)."""

    def __init__(self, session: Session, request: int = 0):
        h = C.c_void_p()
        check(lib().mc_kv_snapshot_take(session.handle, request, C.byref(h)))
        self.handle = h
        n = lib().mc_kv_snapshot_tokens(h, None, 0)
        out = np.zeros(max(n, 1), np.uint32)
        lib().mc_kv_snapshot_tokens(h, out.ctypes.data_as(C.POINTER(C.c_uint32)), n)
        self.tokens = out[:n].tolist()

    def close(self):
        if getattr(self, "handle", None):
            lib().mc_kv_snapshot_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


@dataclass
class CacheLookup:
    """prefix_cache.rs:26-37: tokens covered by the match and the entry."""
    matched_len: int
    kv: object


class PrefixCache:
    """Bounded LRU cache of prompt-prefix K/V snapshots (prefix_cache.rs:
    39-110): ``lookup`` returns the longest cached sequence that is a prefix
    of the query (ties: the most recently used entry), ``insert`` puts an
    entry first (replacing an equal key) and evicts from the tail beyond
    ``max_entries`` (at least 1).  Values are any objects -- KvSnapshot in a
    serving loop -- and are closed when evicted if they have ``close``."""

    def __init__(self, max_entries: int):
        self.entries: list[tuple[tuple[int, ...], object]] = []
        self.max_entries = max(max_entries, 1)

    def lookup(self, tokens) -> CacheLookup | None:
        t = tuple(int(x) for x in tokens)
        best = None
        for seq, kv in self.entries:  # most recently used first
            if t[:len(seq)] == seq and (best is None or len(seq) > len(best[0])):
                best = (seq, kv)
        return None if best is None else CacheLookup(len(best[0]), best[1])

    def insert(self, tokens, kv):
        key = tuple(int(x) for x in tokens)
        for i, (seq, old) in enumerate(self.entries):
            if seq == key:
                del self.entries[i]
                if old is not kv and hasattr(old, "close"):
                    old.close()
                break
        self.entries.insert(0, (key, kv))
        while len(self.entries) > self.max_entries:
            _, old = self.entries.pop()
            if hasattr(old, "close"):
                old.close()

    def __len__(self):
        return len(self.entries)

    def is_empty(self) -> bool:
        return not self.entries

    def capacity(self) -> int:
        return self.max_entries


def speculative_generate(target: Weights, draft: Weights, prompt, config: GenerationConfig,
                         max_context: int | None = None):
    """generate.rs:598-767 with a transformer draft; returns (ids, accepted)."""
    cap = max_context or (len(prompt) + config.max_tokens + config.gamma + 8)
    s = Session(target, draft, gamma=config.gamma, max_context=cap, bonus=config.bonus,
                temperature=config.temperature, seed=config.seed,
                accept_mode=config.accept_mode, top_p=config.top_p, min_p=config.min_p,
                shift_context=config.max_context, anchor_tokens=config.anchor_tokens,
                kv_mode=(KV_MIXED if config.use_mixed_kv else
                         KV_INT8 if config.use_int8_kv else KV_FP32))
    try:
        return s.speculative_generate(prompt, config.max_tokens)
    finally:
        s.close()


def sample_rows(logits, temperature: float = 0.0, top_p: float = 0.0, min_p: float = 0.0,
                seed: int = 0, round: int = 0):
    """generate.rs:948-969 sample, one token per row of a CUDA f32 tensor
    [rows, vocab]: argmax at temperature <= 0, else softmax(l / T) after
    top-p and min-p with the Philox uniform of (seed, round, row).  Returns a
    CUDA int32 tensor of token ids (uint32 values below 2^31)."""
    import torch
    x = logits.contiguous()
    if x.dim() == 1:
        x = x.unsqueeze(0)
    out = torch.empty(x.shape[0], dtype=torch.int32, device=x.device)
    check(lib().mc_sample_rows(x.data_ptr(), x.shape[0], x.shape[1], temperature, top_p, min_p,
                               seed, round, out.data_ptr(),
                               torch.cuda.current_stream(x.device).cuda_stream))
    return out


def forward_llama_cached(session: Session, ids):
    """Batched transformer.rs:64-96: logits for each id, KV appended."""
    return session.forward(ids)
