#!/usr/bin/env python
"""Speculative-decoding throughput on B200: Llama-3-8B-shape int8 target, batch 1.

Workload (one "step"): decode 256 new tokens greedily with speculative decoding
(gamma = 4 draft tokens per round from a 2-layer draft of the same width,
one batched verify forward per round, acceptance on the device) after a
primed 1024-token prompt.  Weights: N(0, 0.02) random init, per-row int8
(target seed 0, draft seed 1), prompt ids uniform from seed 2, generated on
the GPU.  Inputs (7.5 GB of weights) exceed the 126 MB L2 on every step.

  value   decode tokens/s with weights, prompt KV and state resident in HBM
  e2e     the same metric through the C ABI call a user makes
          (mc_speculative_generate: host prompt in, host ids out, prime
          included), host<->device copies inside the timed region
  roofline  verify forward (the dominant kernel set): algorithmic bytes
          (int8 weights + row scales + KV read) / CUDA-event time
  cpu_baseline  the CPU oracle (C restatement of the reference's Rust path)
          timed on this host on a bounded sample, extrapolated per token

``--impl reference`` times the reference's CPU algorithm (the oracle's
bit-identical row-parallel linear on all host cores) on the same workload.
Multi-GPU (torchrun, N ranks): the workload's requests with the target
Megatron tensor-parallel over the N GPUs (column-parallel QKV and gate/up,
row-parallel O and down followed by the fused NVLink reduction, or NCCL
all-reduces with --tp-nccl; vocab-parallel LM head; the draft replicated);
strong scaling, value = the requests' tokens / max-over-ranks time.
--replicas instead runs N independent copies of the workload, one per GPU,
with nothing crossing NVLink (weak scaling); value = all ranks' tokens /
max-over-ranks time.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
METRIC = "spec-decode tokens/s, 8B-shape int8 bs1; verify-kernel HBM GB/s vs 8 TB/s"
PROMPT_LEN, NEW_TOKENS, GAMMA = 1024, 256, 4
WORKLOAD = "llama3-8b-shape int8-row target + 2-layer int8 draft, bs1, prompt 1024, gamma 4, greedy, 256 new"


class Workload:
    """One speculative-decoding benchmark configuration (shapes, formats,
    seeds and run lengths of the reference's benchmark table)."""

    def __init__(self, name, metric, desc, target, draft, fmt, draft_fmt, prompt_len, new_tokens,
                 gamma, temperature=0.0, seed=0, accept_mode=0, batch=1):
        self.name, self.metric, self.desc = name, metric, desc
        self.target, self.draft = target, draft
        self.fmt, self.draft_fmt = fmt, draft_fmt
        self.prompt_len, self.new_tokens, self.gamma = prompt_len, new_tokens, gamma
        self.temperature, self.seed, self.accept_mode = temperature, seed, accept_mode
        self.batch = batch  # concurrent requests


def workloads():
    from dataclasses import replace
    import modelc_b200 as mb
    return {
        "tiny": Workload(
            "tiny", "spec-decode tokens/s, tiny 4-layer d256 int8 bs1 (L2-resident, latency-bound)",
            "tiny-4l-d256 int8-row target (reference-exact: heads = d/64, eps 1e-6, theta 1e4) + "
            "1-layer draft, bs1, prompt 32, gamma 4, greedy, 128 new",
            mb.TINY, mb.TINY.with_layers(1), "i8_row", "i8_row", 32, 128, 4),
        "llama3-8b": Workload("llama3-8b", METRIC, WORKLOAD, mb.LLAMA3_8B,
                              mb.LLAMA3_8B.with_layers(2), "i8_row", "i8_row", PROMPT_LEN,
                              NEW_TOKENS, GAMMA),
        "llama3-8b-bs8": Workload(
            "llama3-8b-bs8", "spec-decode tokens/s, 8B-shape int8 bs8 (8 concurrent requests)",
            "llama3-8b-shape int8-row target + 2-layer int8 draft, 8 concurrent requests, "
            "prompts 1024, gamma 4, greedy, 256 new each",
            mb.LLAMA3_8B, mb.LLAMA3_8B.with_layers(2), "i8_row", "i8_row", PROMPT_LEN, NEW_TOKENS,
            GAMMA, batch=8),
        "tinyllama": Workload(
            "tinyllama", "spec-decode tokens/s, TinyLlama-1.1B-shape q4_0 bs1, stochastic T=0.8",
            "tinyllama-1.1b-shape q4_0 target + 2-layer q4_0 draft, bs1, prompt 512, gamma 5, "
            "min(1,p/q) acceptance at T=0.8 (top-p off, Philox seed 7), 256 new",
            mb.TINYLLAMA, mb.TINYLLAMA.with_layers(2), "q4_0", "q4_0", 512, 256, 5,
            temperature=0.8, seed=7),
        "llama2-70b": Workload(
            "llama2-70b", "spec-decode tokens/s, 70B-shape q4_0 bs1",
            "llama2-70b-shape q4_0 target + llama3-8b-shape int8 draft (vocab 32000), bs1, "
            "prompt 2048, gamma 4, greedy, 256 new",
            mb.LLAMA2_70B, replace(mb.LLAMA3_8B, vocab=32000), "q4_0", "i8_row", 2048, 256, 4),
    }


def dist_env():
    return (int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)),
            int(os.environ.get("LOCAL_RANK", 0)))


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def profile_traffic(workload, parallelism):
    """Per-launch DRAM bytes of the verify forward from the committed ncu
    summary, or None when that capture was of another workload."""
    p = os.path.join(ROOT, "profiles", "verify_traffic.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        if d.get("workload") == workload and d.get("parallelism") == parallelism:
            return d.get("verify_forward_dram_bytes")
    return None


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.samples = []
        self._stop = threading.Event()
        self._t = None

    def _run(self):
        while not self._stop.is_set():
            try:
                out = subprocess.run(["nvidia-smi", "-i", str(self.gpu), "--query-gpu=" + self.FIELDS,
                                      "--format=csv,noheader,nounits"], capture_output=True,
                                     text=True, timeout=5).stdout.strip()
                if out:
                    self.samples.append([x.strip() for x in out.split(",")])
            except Exception:
                pass
            self._stop.wait(0.2)

    def __enter__(self):
        self._t = threading.Thread(target=self._run, daemon=True)
        self._t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        self._t.join(timeout=10)

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        sm = [float(s[1]) for s in self.samples if s[1].replace(".", "").isdigit()]
        mx = [float(s[2]) for s in self.samples if s[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for s in self.samples for i in range(4)
                          if len(s) > 5 + i and s[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
                "samples": len(self.samples)}


# ---------------------------------------------------------------------- CPU
def cpu_sample(n_threads: int, kv_len: int = 1100, cfg=None):
    """Time the CPU oracle on a bounded sample of the workload: one decoder
    layer of `cfg` and its LM head (f32 dequantized weights, as the reference
    holds them) for a single-token forward at KV length kv_len, repeated.
    Per-token cost extrapolates to the target's layers + head per verify
    forward plus gamma draft forwards per round."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as o
    if cfg is None:
        from modelc_b200.model import LLAMA3_8B as cfg
    rng = np.random.default_rng(0)
    d, f, v = cfg.hidden, cfg.ffn, cfg.vocab
    hd, nh, nkv = cfg.head_dim, cfg.n_heads, cfg.n_kv_heads

    def mat(r, c):
        return (rng.standard_normal((r, c), dtype=np.float32) * np.float32(0.02))

    p = "model.layers.0."
    w = {p + "input_layernorm.weight": np.ones(d, np.float32),
         p + "self_attn.q_proj.weight": mat(nh * hd, d), p + "self_attn.k_proj.weight": mat(nkv * hd, d),
         p + "self_attn.v_proj.weight": mat(nkv * hd, d), p + "self_attn.o_proj.weight": mat(d, nh * hd),
         p + "post_attention_layernorm.weight": np.ones(d, np.float32),
         p + "mlp.gate_proj.weight": mat(f, d), p + "mlp.up_proj.weight": mat(f, d),
         p + "mlp.down_proj.weight": mat(d, f), "model.norm.weight": np.ones(d, np.float32)}
    layer = o.OracleModel(w, 1, d, v, f, mode=o.MODE_GENERAL, n_heads=nh, n_kv_heads=nkv,
                          head_dim=hd, rope_base=cfg.rope_theta, eps=cfg.eps, n_threads=n_threads)
    kv = layer.new_kv(kv_len + 8)
    kvs = kv.ptr.contents
    kvs.len = kv_len  # attend over kv_len cached positions (zeros)
    x = rng.standard_normal(d, dtype=np.float32)
    head = mat(v, d)
    # layer: attention + MLP for one token (no head in this model)
    reps_l, t0 = 0, time.perf_counter()
    while reps_l < 3 or time.perf_counter() - t0 < 4.0:
        kvs.len = kv_len
        layer.forward_embedding(x, kv)  # includes a head-less final norm
        reps_l += 1
    t_layer = (time.perf_counter() - t0) / reps_l
    reps_h, t0 = 0, time.perf_counter()
    while reps_h < 2 or time.perf_counter() - t0 < 4.0:
        if n_threads > 1:
            o.linear_par(head, x, n_threads)
        else:
            o.linear(head, x)
        reps_h += 1
    t_head = (time.perf_counter() - t0) / reps_h
    return t_layer, t_head, reps_l, reps_h


def cpu_tokens_per_s(t_layer, t_head, rounds, tokens, accepted, gamma=GAMMA, target_layers=32,
                     draft_layers=2, t_draft_layer=None, t_draft_head=None):
    """Reference cost model: per round gamma draft forwards (draft layers +
    head) and the sequential verify's target forwards (min(a+1, gamma) per
    round, generate.rs:695-726); tokens = emitted tokens."""
    t_draft = draft_layers * (t_draft_layer if t_draft_layer is not None else t_layer) + (
        t_draft_head if t_draft_head is not None else t_head)
    t_target = target_layers * t_layer + t_head
    target_fwd = sum(min(a + 1, gamma) for a in accepted) if accepted else rounds
    total = rounds * gamma * t_draft + target_fwd * t_target
    return tokens / total


def _dequant_q4_0_torch(blk, rows, cols):
    """dequant.rs:33-44 on the device: (code - 8) as f32 * d, low nibbles first."""
    import torch
    b = blk.view(rows, cols // 32, 18)
    d = b[..., 0:2].contiguous().view(torch.float16).float()  # [rows, nb, 1]
    qs = b[..., 2:].to(torch.int32)
    v = torch.cat([(qs & 0x0F) - 8, (qs >> 4) - 8], dim=2).float() * d
    return v.reshape(rows, cols)


def host_f32_model(cfg, seed, fmt, device, n_threads, keep=None):
    """The oracle over f32 host copies of the seeded weights build_models
    loads on the GPU (the same draw, dequantized on the device exactly as the
    reference dequantizes at load: int8 rows q * scale, q4_0 (code - 8) * d),
    so the CPU runs the very model the GPU runs.  keep: a dict that receives
    the arrays (the oracle model holds pointers into them)."""
    import torch
    import modelc_b200 as mb
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as o
    tt = mb.synth_weights_torch(cfg, seed=seed, device=device, fmt=fmt)
    w = {} if keep is None else keep
    for name in list(tt):
        dt, t, extra = tt.pop(name)
        if dt == "f32":
            f = t
        elif dt == "i8_row":
            f = t.float() * extra[:, None]
        else:
            f = _dequant_q4_0_torch(t, *extra)
        w[name] = f.cpu().numpy()
        del t, extra, f
    torch.cuda.empty_cache()
    c = cfg.resolved()
    return o.OracleModel(w, c.n_layers, c.hidden, c.vocab, c.ffn, mode=cfg.mode,
                         n_heads=c.n_heads, n_kv_heads=c.n_kv_heads, head_dim=c.head_dim,
                         rope_base=c.rope_theta, eps=c.eps, n_threads=n_threads)


def cpu_forward_time(model, kv_len, min_s, min_reps=1):
    """Seconds per single-token forward of a whole oracle model
    (forward_llama_cached: every layer, the final norm and the LM head) at
    KV length kv_len, averaged over at least min_s seconds."""
    rng = np.random.default_rng(0)
    x = rng.standard_normal(model.m.hidden).astype(np.float32)
    kv = model.new_kv(kv_len + 8)
    reps, t0 = 0, time.perf_counter()
    while reps < min_reps or time.perf_counter() - t0 < min_s:
        kv.ptr.contents.len = kv_len  # attend over kv_len cached positions
        model.forward_embedding(x, kv)
        reps += 1
    return (time.perf_counter() - t0) / reps, reps


def cpu_round_tokens_per_s(t_target, t_draft, rounds, tokens, accepted, gamma):
    """The reference's cost of this run's rounds, from whole-forward times:
    per round gamma draft forwards and the sequential verify's target
    forwards, min(a + 1, gamma) of them after a accepted drafts
    (generate.rs:641-726); tokens = emitted tokens."""
    target_fwd = sum(min(a + 1, gamma) for a in accepted) if accepted else rounds
    total = rounds * gamma * t_draft + target_fwd * t_target
    return tokens / total


def host_bytes_f32(cfg):
    pc = cfg.param_counts()
    return 4 * (cfg.n_layers * pc["layer"] + pc["head"] + pc["embed"])


def host_fits(*cfgs):
    """Whether f32 copies of these models fit comfortably in host memory."""
    try:
        import psutil
        avail = psutil.virtual_memory().available
    except Exception:
        return False
    return sum(host_bytes_f32(c) for c in cfgs) < 0.6 * avail


def cpu_baseline_full(wl, cfg, device_index, rounds, tokens, accepted):
    """The reference's CPU path on this host over the very models the GPU
    ran (f32 copies of the same seeded weights): whole single-token forwards
    of the target and the draft at KV length prompt + 76, timed (a) on every
    host thread with the bit-identical row-parallel linear and (b) on one
    thread with the reference-faithful scalar linear (linear_with has no
    threading, transformer.rs:825-843), then composed into this run's rounds
    (cpu_round_tokens_per_s).  Models too large for host memory (the 70B
    shape) fall back to one timed layer plus the head, extrapolated."""
    import torch
    nthr = os.cpu_count() or 1
    kvl = wl.prompt_len + 76
    if not host_fits(cfg, wl.draft):
        t_layer, t_head, rl, rh = cpu_sample(nthr, kvl, cfg)
        same = (wl.draft.hidden, wl.draft.ffn, wl.draft.vocab) == (cfg.hidden, cfg.ffn, cfg.vocab)
        tdl, tdh = (t_layer, t_head) if same else cpu_sample(nthr, kvl, wl.draft)[:2]
        v = cpu_tokens_per_s(t_layer, t_head, rounds, tokens, accepted, wl.gamma, cfg.n_layers,
                             wl.draft.n_layers, tdl, tdh)
        return {"value": round(v, 5), "unit": "tokens/s", "cores": nthr, "kind": "port",
                "sample": (f"f32 weights of this shape exceed host memory: oracle row-parallel "
                           f"forward of 1 target layer at KV {kvl} ({t_layer * 1e3:.1f} ms, {rl} "
                           f"reps) + LM head ({t_head * 1e3:.1f} ms, {rh} reps), extrapolated to "
                           f"{cfg.n_layers} layers + head and {wl.gamma} drafts per round with "
                           f"this run's acceptance")}
    dev = torch.device("cuda", device_index)
    keep_t, keep_d = {}, {}
    om_t = host_f32_model(cfg, 0, wl.fmt, dev, nthr, keep_t)
    om_d = host_f32_model(wl.draft, 1, wl.draft_fmt, dev, nthr, keep_d)
    tt, nt = cpu_forward_time(om_t, kvl, 8.0, 2)
    td, nd = cpu_forward_time(om_d, kvl, 3.0, 3)
    v = cpu_round_tokens_per_s(tt, td, rounds, tokens, accepted, wl.gamma)
    om_t.m.n_threads = 1
    om_d.m.n_threads = 1
    tt1, _ = cpu_forward_time(om_t, kvl, 0.0, 1)
    td1, _ = cpu_forward_time(om_d, kvl, 0.0, 1)
    v1 = cpu_round_tokens_per_s(tt1, td1, rounds, tokens, accepted, wl.gamma)
    return {"value": round(v, 5), "unit": "tokens/s", "cores": nthr, "kind": "port",
            "sample": (f"oracle over f32 copies of this run's models: whole {cfg.n_layers}-layer "
                       f"target forward at KV {kvl} {tt * 1e3:.1f} ms ({nt} reps), whole "
                       f"{wl.draft.n_layers}-layer draft forward {td * 1e3:.1f} ms ({nd} reps), "
                       f"row-parallel on {nthr} threads, composed into this run's {rounds} "
                       f"rounds ({wl.gamma} draft forwards + min(a+1, gamma) target forwards "
                       f"each)"),
            "single_thread": {"value": round(v1, 6), "unit": "tokens/s", "cores": 1,
                              "sample": (f"the same with the reference-faithful scalar linear on "
                                         f"one thread: target forward {tt1:.2f} s, draft forward "
                                         f"{td1:.2f} s")}}


# ---------------------------------------------------------------------- GPU
def build_models(device_index: int, layers: int | None = None, wl: Workload | None = None,
                 tp: tuple = (0, 1), draft_layers: int | None = None):
    """Random-init weights N(0, 0.02) generated on the GPU (target seed 0,
    draft seed 1) and a uniform prompt (seed 2).  tp = (rank, world) keeps
    this rank's tensor-parallel shard of the target; the draft is replicated."""
    import torch
    import modelc_b200 as mb
    wl = wl or workloads()["llama3-8b"]
    dev = torch.device("cuda", device_index)
    cfg = wl.target if not layers else wl.target.with_layers(layers)
    dcfg = wl.draft if not draft_layers else wl.draft.with_layers(draft_layers)
    tt = mb.synth_weights_torch(cfg, seed=0, device=dev, fmt=wl.fmt)
    target = mb.Weights(tt, cfg, device=device_index, tp_rank=tp[0], tp_world=tp[1])
    del tt
    torch.cuda.empty_cache()
    dt = mb.synth_weights_torch(dcfg, seed=1, device=dev, fmt=wl.draft_fmt)
    draft = mb.Weights(dt, dcfg, device=device_index)
    del dt
    torch.cuda.empty_cache()
    g = torch.Generator(device="cpu")
    g.manual_seed(2)
    prompts = [torch.randint(0, cfg.vocab, (wl.prompt_len,), generator=g).numpy().astype(np.uint32)
               for _ in range(wl.batch)]
    return cfg, target, draft, prompts[0] if wl.batch == 1 else prompts


def run_ours(args):
    import torch
    import modelc_b200 as mb
    wl = workloads()[args.config]
    PROMPT_LEN, NEW_TOKENS, GAMMA = wl.prompt_len, wl.new_tokens, wl.gamma
    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    # N > 1: the target tensor-parallel over the N GPUs (strong scaling);
    # --replicas: N independent copies of the workload (weak scaling)
    tp = world > 1 and not args.replicas
    if world > 1:
        import datetime
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=300))
    cfg, target, draft, prompt = build_models(local, wl=wl, tp=(rank, world) if tp else (0, 1))
    B = wl.batch
    prompts = prompt if B > 1 else [prompt]
    max_ctx = PROMPT_LEN + NEW_TOKENS + 2 * GAMMA + 8
    sess = mb.Session(target, draft, gamma=GAMMA, max_context=max_ctx,
                      temperature=wl.temperature, seed=wl.seed, accept_mode=wl.accept_mode,
                      n_requests=B)
    if tp:
        uid = torch.zeros(128, dtype=torch.uint8, device="cuda")
        if rank == 0:
            uid.copy_(torch.frombuffer(bytearray(mb.tp_unique_id()), dtype=torch.uint8))
        torch.distributed.broadcast(uid, 0)
        sess.tp_init(bytes(uid.cpu().numpy().tobytes()), rank, world)
        if not args.tp_nccl:  # fused NVLink reduction of the row-parallel projections
            handles = [None] * world
            torch.distributed.all_gather_object(handles, sess.tp_ipc_handle())
            sess.tp_open_peers(handles)
    stream = torch.cuda.ExternalStream(sess.stream_ptr, device=torch.device("cuda", local))

    def barrier():
        torch.cuda.synchronize()
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize()

    # ---- device-resident decode: prime once, each step decodes 256 tokens
    # (per request)
    sess.prime_batch(prompts)
    for _ in range(args.warmup):
        sess.rewind()
        sess.decode(NEW_TOKENS)
    barrier()
    tokens = 0
    rounds = 0
    accepted = []
    ev = []
    # weights smaller than L2: flush it (write 512 MB) before every timed step
    l2_flush = (torch.empty(512 << 20, dtype=torch.uint8, device="cuda")
                if target.streamed_bytes < (256 << 20) else None)
    with ClockSampler(local) as clk:
        for _ in range(args.steps):
            sess.rewind()
            if l2_flush is not None:
                l2_flush.fill_(1)
                torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            sess.decode(NEW_TOKENS)
            e1.record(stream)
            ev.append((e0, e1))
            step_rounds = 0
            for z in range(B):
                toks, acc = sess.read(request=z)
                tokens += len(toks)
                accepted += acc
                step_rounds = max(step_rounds, len(acc))
            rounds += step_rounds  # rounds run (every request takes part in each)
    barrier()
    ms = sum(a.elapsed_time(b) for a, b in ev)
    t_local = torch.tensor([ms / 1e3], device="cuda")
    n_local = torch.tensor([float(tokens)], device="cuda")
    if world > 1:
        torch.distributed.all_reduce(t_local, op=torch.distributed.ReduceOp.MAX)
        if not tp:  # replicas: every rank's tokens; TP: one request's tokens
            torch.distributed.all_reduce(n_local, op=torch.distributed.ReduceOp.SUM)
    t_total, tok_total = float(t_local.item()), float(n_local.item())
    value = tok_total / t_total
    ms_per_step = t_total * 1e3 / args.steps
    launches = rounds * sess.round_launches
    req_rounds = len(accepted)  # request-rounds (the CPU reference runs each)

    # ---- verify-forward roofline (dominant kernel set), stream events
    sess.rewind()
    sess.decode(8)
    vm = GAMMA
    kv_len = PROMPT_LEN + 8
    sess.verify_launch(3)
    torch.cuda.synchronize()
    n_ver = 20
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    sess.verify_launch(n_ver)
    e1.record(stream)
    torch.cuda.synchronize()
    t_ver = e0.elapsed_time(e1) / 1e3 / n_ver
    shards = world if tp else 1  # bytes this GPU reads
    kv_bytes = B * 2 * cfg.n_layers * (kv_len + vm) * cfg.n_kv_heads * cfg.head_dim * 4 // shards
    act_bytes = B * 2 * cfg.n_layers * vm * (3 * cfg.hidden + 2 * cfg.ffn // shards) * 4
    algo = target.streamed_bytes + kv_bytes + act_bytes
    peak, peak_kind = measured_peaks()
    achieved = algo / t_ver / 1e9
    parallelism = (((f"tp{world}" + ("-nccl" if args.tp_nccl else "-nvlink"))
                    if tp else f"replicas{world}") if world > 1 else "single")
    # each replica runs the single-GPU forward, so the single-GPU capture holds
    traffic = profile_traffic(args.config, "single" if not tp else parallelism)
    roof = {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
            "frac": round(achieved / peak, 4), "traffic": traffic,
            "peak_source": peak_kind, "kernel": "verify forward (k_gemv + fused kernels)",
            "algorithmic_bytes": algo, "ms": round(t_ver * 1e3, 4)}

    # ---- end to end through the C ABI (host buffers, prime included)
    e2e_ms = []
    h2d = B * PROMPT_LEN * 4
    for i in range(max(1, min(args.steps, 3)) + 1):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        if B == 1:
            res = [sess.speculative_generate(prompt, NEW_TOKENS)]
        else:
            res = sess.speculative_generate_batch(prompts, NEW_TOKENS)
        e1.record(stream)
        torch.cuda.synchronize()
        if i > 0:
            e2e_ms.append(e0.elapsed_time(e1))
    e2e_tokens = sum(len(t) for t, _ in res)
    d2h = sum(len(t) + len(a) for t, a in res) * 4
    e2e_local = torch.tensor([statistics.mean(e2e_ms) / 1e3], device="cuda")
    if world > 1:
        torch.distributed.all_reduce(e2e_local, op=torch.distributed.ReduceOp.MAX)
    e2e_value = e2e_tokens * (1 if tp else world) / float(e2e_local.item())

    line = None
    wbytes = target.streamed_bytes
    if rank == 0:
        cpu = None
        if not args.no_cpu and world == 1:
            sess.close()  # free the device before the CPU legs
            del target, draft
            torch.cuda.empty_cache()
            cpu = cpu_baseline_full(wl, cfg, local, req_rounds, tokens, accepted)
        clocks = clk.summary()
        line = {
            "metric": wl.metric, "value": round(value, 3), "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_per_step, 3),
            "higher_is_better": True, "scaling": "strong" if tp else "weak", "vs_baseline": None,
            "dtype": "int8" if wl.fmt == "i8_row" else "q4_0",
            "data": "synthetic (random-init weights N(0,0.02), uniform prompt ids)",
            "config": {"workload": wl.desc, "target": cfg.name, "draft_layers": wl.draft.n_layers,
                       "prompt_len": PROMPT_LEN, "new_tokens": NEW_TOKENS, "gamma": GAMMA,
                       "temperature": wl.temperature, "batch": B,
                       "parallelism": parallelism,
                       "l2": (f"inputs larger than L2 ({wbytes / 1e9:.2f} GB of weights per verify)"
                              if l2_flush is None else
                              f"L2 flushed (512 MB write) before each timed step; "
                              f"{wbytes / 1e6:.2f} MB of weights per verify stay L2-resident "
                              f"within a step")},
            "us_per_round": round(t_total * 1e6 / max(rounds, 1), 2),
            "roofline": roof, "cpu_baseline": cpu,
            "e2e": {"value": round(e2e_value, 3), "unit": "tokens/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h,
                    "includes": f"prime ({PROMPT_LEN}-token prefill) + decode"},
            "clocks": clocks, "gpu_launches": int(launches * world),
            "roofline_scope": "per GPU (this rank's weight shard)" if tp else "one GPU",
            "acceptance": {"rounds": rounds, "request_rounds": req_rounds, "tokens": tokens,
                           "mean_accepted": round(float(np.mean(accepted)) if accepted else 0.0, 4)},
        }
    if world > 1:
        torch.distributed.barrier()  # peers may still write into this rank's buffers
    sess.close()  # (already closed before a CPU leg; closing twice is harmless)
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()
    if line:
        print(json.dumps(line), flush=True)


def run_profile(args):
    """Short run for ncu launch lists: prime the 1024-token prompt, 2
    speculative rounds (their launch count is printed), 3 verify forwards,
    one more inside the NVTX range "verify" (select it with ncu --nvtx
    --nvtx-include verify/), and 2 more rounds."""
    import torch
    import modelc_b200 as mb
    torch.cuda.set_device(0)
    wl = workloads()[args.config]
    cfg, target, draft, prompt = build_models(0, args.layers, wl=wl,
                                              draft_layers=args.draft_layers)
    sess = mb.Session(target, draft, gamma=wl.gamma,
                      max_context=wl.prompt_len + wl.new_tokens + 2 * wl.gamma + 8,
                      temperature=wl.temperature, seed=wl.seed, accept_mode=wl.accept_mode)
    sess.prime(prompt)
    sess.decode(2)  # captures the round graph
    torch.cuda.synchronize()
    print(json.dumps({"round_launches": sess.round_launches}), flush=True)
    sess.verify_launch(3)
    torch.cuda.synchronize()
    torch.cuda.nvtx.range_push("verify")
    sess.verify_launch(1)
    torch.cuda.synchronize()
    torch.cuda.nvtx.range_pop()
    sess.decode(2)
    torch.cuda.synchronize()
    sess.close()


def run_timeline(args):
    """In-situ timeline of one verify forward (MC_TRACE build of the library):
    per launch the first CTA's start, its release from griddepcontrol.wait and
    the last CTA's end (%globaltimer), summed per kernel kind; plus per-phase
    times (thread 0 of each CTA) of the attention and the tcgen05 GEMMs.
    --config selects the workload (batch included).  Under torchrun with N
    ranks: the target tensor-parallel over them with the fused NVLink
    reduction, rank 0's timeline printed."""
    import ctypes as C
    import torch
    import modelc_b200 as mb
    import modelc_b200._lib as L
    L.use_trace_library()
    lib = L.lib()
    wl = workloads()[args.config]
    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=300))
    cfg, target, draft, prompt = build_models(local, wl=wl, tp=(rank, world))
    B = wl.batch
    prompts = prompt if B > 1 else [prompt]
    sess = mb.Session(target, draft, gamma=wl.gamma,
                      max_context=wl.prompt_len + wl.new_tokens + 2 * wl.gamma + 8, n_requests=B)
    if world > 1:
        uid = torch.zeros(128, dtype=torch.uint8, device="cuda")
        if rank == 0:
            uid.copy_(torch.frombuffer(bytearray(mb.tp_unique_id()), dtype=torch.uint8))
        torch.distributed.broadcast(uid, 0)
        sess.tp_init(bytes(uid.cpu().numpy().tobytes()), rank, world)
        handles = [None] * world
        torch.distributed.all_gather_object(handles, sess.tp_ipc_handle())
        sess.tp_open_peers(handles)
    sess.prime_batch(prompts)
    sess.decode(8)
    sess.verify_launch(3)
    torch.cuda.synchronize()
    # with encoding tails (one token group) the norm and SwiGLU-output
    # encoders run inside the GEMV before them: o, gu and down then include
    # the encoder of the next projection
    # (the attention too, when its query rows fit one m-tile and its grid one
    # wave: then it encodes the O projection's input)
    M = B * wl.gamma
    mask = int(os.environ.get("MODELC_CUDA_ENCODER_TAILS", "0"))
    tails = M <= 16 and bool(mask & 1)
    c = cfg.resolved()
    G = c.n_heads // c.n_kv_heads
    max_ctx = wl.prompt_len + wl.new_tokens + 2 * wl.gamma + 8
    att_tail = (bool(mask & 2) and G * min(wl.gamma, max(1, 64 // G)) <= 16
                and c.n_kv_heads * -(-max_ctx // 64) * B <= 2 * 148)
    att = ["attention+enc"] if att_tail else ["attention", "quant_o"]
    names = ["embed"]
    for l in range(cfg.n_layers):
        if world > 1:  # row-parallel GEMVs store partial rows; a reduce follows each
            names += ["quant_attn", "qkv"] + att + ["o", "o_reduce", "quant_mlp", "gu",
                                                    "quant_act", "down", "down_reduce"]
        elif tails:
            names += (["quant_attn"] if l == 0 else []) + ["qkv"] + att + ["o+enc", "gu+enc",
                                                                          "down+enc"]
        else:
            names += ["quant_attn", "qkv"] + att + ["o", "quant_mlp", "gu", "quant_act", "down"]
    names += ["head"] if tails and world == 1 else ["quant_final", "head"]
    n = len(names)
    for _ in range(3):  # the last of three repetitions
        if world > 1:
            torch.distributed.barrier()
        L.check(lib.mc_trace_reset())
        if world > 1:
            torch.distributed.barrier()
        sess.verify_launch(1)
        torch.cuda.synchronize()
        buf = (C.c_ulonglong * (19 * (n + 1)))()
        L.check(lib.mc_trace_read(buf, n + 1))
    # the launch list must be the forward's: slot n unused, slot n - 1 used
    if buf[3 * n] != 2 ** 64 - 1 or buf[3 * (n - 1)] == 2 ** 64 - 1:
        raise RuntimeError(f"timeline names do not match the forward's {n} launches")
    raw = np.array(buf, dtype=np.float64)[:19 * (n + 1)]
    raw = np.r_[raw[:3 * n], raw[3 * (n + 1): 3 * (n + 1) + 16 * n]]
    if world > 1:  # the peers still read this rank's exchange buffers until all are done
        torch.distributed.barrier()
        if rank != 0:
            sess.close()
            torch.distributed.barrier()
            torch.distributed.destroy_process_group()
            return
    a = raw[:3 * n].reshape(n, 3)
    ph = raw[3 * n:].reshape(n, 16)
    a = (a - a[0, 0]) / 1e3  # us
    exe = a[:, 2] - a[:, 1]
    gap = np.r_[0.0, a[1:, 1] - a[:-1, 2]]
    print(f"workload: {wl.desc}")
    print(f"verify forward critical path {a[-1, 2]:.1f} us over {n} launches")
    print(f"{'kind':12s} {'n':>4s} {'exec avg':>9s} {'gap avg':>8s} {'exec sum':>9s} {'gap sum':>8s}")
    kinds = {}
    for i, nm in enumerate(names):
        k = kinds.setdefault(nm, [0, 0.0, 0.0])
        k[0] += 1
        k[1] += exe[i]
        k[2] += gap[i]
    for nm, (c, e, g) in kinds.items():
        print(f"{nm:12s} {c:4d} {e / c:9.2f} {g / c:8.2f} {e:9.1f} {g:8.1f}")
    gemm_ph = ["launch->wait", "weights issued", "mma done", "cluster: all mma done",
               "tmem read + push", "pushes landed", "sums + epilogue", "end barrier"]
    attn_ph = ["launch->wait", "load K/V/q", "scores + softmax", "P.V", "partials out",
               "arrive", "-", "combine (last CTA)"]
    quant_ph = ["launch->wait", "producer stats in", "barrier", "encode + stores", "-", "-",
                "-", "-"]
    for kind in ["qkv", "o", "gu", "down", "head", "attention", "quant_attn", "quant_o",
                 "quant_mlp", "quant_act"]:  # GEMVs with a tail record no phases
        idx = [i for i, nm in enumerate(names) if nm == kind]
        sums, cnts = ph[idx, :8].sum(0), ph[idx, 8:].sum(0)
        if cnts.sum() == 0:
            continue
        labels = (attn_ph if kind == "attention" else
                  quant_ph if kind.startswith("quant") else gemm_ph)
        print(f"{kind} phases (avg us per CTA reaching it; CTAs per launch):")
        for k in range(8):
            if cnts[k]:
                print(f"  {k} {labels[k]:22s} {sums[k] / cnts[k] / 1e3:7.2f}   "
                      f"{cnts[k] / len(idx):7.1f}")
    sess.close()
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


def run_sweep(args):
    """Isolated verify-step projection Y = X . dequant(W)^T through the public
    mc_linear_run: X is M x 4096 N(0, 1), W is N x 4096 N(0, 0.02) as per-row
    int8 or q4_0.  Enough weight copies rotate (at least 4, more than L2) that
    every call streams W from HBM.  Achieved GB/s counts the weight codes and
    scales once per call plus X and Y; TFLOP/s = 2 M N K / time."""
    import torch
    import modelc_b200 as mb
    from modelc_b200.model import _q4_0_torch
    torch.cuda.set_device(0)
    peak, peak_kind = measured_peaks()
    K = 4096
    ms_list = [args.sweep_m] if args.sweep_m else [1, 5, 8, 16, 40, 64]
    for fmt in ((args.sweep_fmt,) if args.sweep_fmt else ("i8_row", "q4_0")):
        for n in ((args.sweep_n,) if args.sweep_n else (4096, 14336, 128256)):
            g = torch.Generator(device="cuda")
            g.manual_seed(n)
            wb = n * K // 32 * 18 if fmt == "q4_0" else n * K + 4 * n
            copies = max(4, -(-300_000_000 // wb))
            lins = []
            for c in range(copies):
                w = torch.randn((n, K), generator=g, device="cuda") * 0.02
                if fmt == "q4_0":
                    t = ("q4_0", _q4_0_torch(w), (n, K))
                else:
                    amax = w.abs().amax(dim=1)
                    sc = torch.where(amax > 0, amax / 127.0, torch.ones_like(amax))
                    q = torch.round(w / sc[:, None]).clamp_(-127, 127).to(torch.int8)
                    t = ("i8_row", q, sc)
                lins.append(mb.Linear(t))
                del w, t
            torch.cuda.empty_cache()
            for m in ms_list:
                x = torch.randn((m, K), generator=g, device="cuda")
                y = torch.empty((m, n), device="cuda")
                st = torch.cuda.current_stream().cuda_stream
                for l in lins:
                    l.run_ptr(x.data_ptr(), m, y.data_ptr(), st)
                reps = 4 * copies
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                for r in range(reps):
                    lins[r % copies].run_ptr(x.data_ptr(), m, y.data_ptr(), st)
                e1.record()
                torch.cuda.synchronize()
                us = e0.elapsed_time(e1) * 1e3 / reps
                algo = wb + 4 * m * K + 4 * m * n
                print(json.dumps({"sweep": "projection", "fmt": fmt, "M": m, "N": n, "K": K,
                                  "us": round(us, 2), "GB_s": round(algo / us / 1e3, 1),
                                  "hbm_frac": round(algo / us / 1e3 / peak, 3),
                                  "TFLOP_s": round(2 * m * n * K / us / 1e6, 2),
                                  "peak_gbs": peak, "peak_source": peak_kind,
                                  "copies": copies}), flush=True)
            for l in lins:
                l.close()
            del lins
            torch.cuda.empty_cache()


def run_reference(args):
    """The reference's CPU path (the oracle's restatement of
    speculative_generate's rounds) on this host's cores, on the workload's
    own models: each step is one round at acceptance 0 (unrelated random-init
    target and draft: the first draft token is rejected, generate.rs:695-726),
    i.e. gamma whole draft forwards and one whole target forward at KV length
    prompt + 76, on every host thread with the bit-identical row-parallel
    linear.  One token per round."""
    rank, world, local = dist_env()
    if rank != 0:
        return
    import torch
    wl = workloads()[args.config]
    nthr = os.cpu_count() or 1
    kvl = wl.prompt_len + 76
    t_start = time.time()
    if host_fits(wl.target, wl.draft):
        dev = torch.device("cuda", local)
        keep_t, keep_d = {}, {}
        om_t = host_f32_model(wl.target, 0, wl.fmt, dev, nthr, keep_t)
        om_d = host_f32_model(wl.draft, 1, wl.draft_fmt, dev, nthr, keep_d)
        rng = np.random.default_rng(0)
        xt = rng.standard_normal(om_t.m.hidden).astype(np.float32)
        xd = rng.standard_normal(om_d.m.hidden).astype(np.float32)
        kvt, kvd = om_t.new_kv(kvl + 8), om_d.new_kv(kvl + 8)
        times = []
        t0 = time.time()
        for i in range(args.warmup + args.steps):
            t1 = time.perf_counter()
            for _ in range(wl.gamma):
                kvd.ptr.contents.len = kvl
                om_d.forward_embedding(xd, kvd)
            kvt.ptr.contents.len = kvl
            om_t.forward_embedding(xt, kvt)
            if i >= args.warmup:
                times.append(time.perf_counter() - t1)
        v = 1.0 / statistics.mean(times)
        ms_step = (time.time() - t0) * 1e3 / (args.warmup + args.steps)
        sample = (f"per step one round: {wl.gamma} whole {wl.draft.n_layers}-layer draft forwards "
                  f"+ one whole {wl.target.n_layers}-layer target forward at KV {kvl} (f32 copies of "
                  f"the workload's seeded models), row-parallel on {nthr} threads; one token")
    else:
        vals = []
        for i in range(args.warmup + args.steps):
            t_layer, t_head, rl, rh = cpu_sample(nthr, kvl, wl.target)
            if i >= args.warmup:
                vals.append(cpu_tokens_per_s(t_layer, t_head, 1, 1, [0], wl.gamma,
                                             wl.target.n_layers, wl.draft.n_layers))
        v = statistics.mean(vals)
        ms_step = (time.time() - t_start) * 1e3 / (args.warmup + args.steps)
        sample = (f"f32 weights of this shape exceed host memory: per step 1 target layer at KV "
                  f"{kvl} + LM head, extrapolated to one round emitting one token")
    line = {"impl": "reference", "metric": wl.metric, "value": round(v, 5), "unit": "tokens/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms_step, 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "config": {"workload": wl.desc, "target": wl.target.name},
            "cpu_baseline": {"value": round(v, 5), "unit": "tokens/s", "cores": nthr, "kind": "port",
                             "sample": sample},
            "e2e": {"value": round(v, 5), "unit": "tokens/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline sample")
    ap.add_argument("--profile", action="store_true", help="short run for ncu launch lists")
    ap.add_argument("--layers", type=int, default=None,
                    help="--profile only: target layers (fewer = smaller device footprint)")
    ap.add_argument("--draft-layers", type=int, default=None,
                    help="--profile only: draft layers")
    ap.add_argument("--config", default="llama3-8b",
                    choices=["tiny", "llama3-8b", "llama3-8b-bs8", "tinyllama", "llama2-70b"],
                    help="workload (default: the headline 8B int8 batch-1 configuration)")
    ap.add_argument("--replicas", action="store_true",
                    help="N > 1: N independent copies of the workload, one per GPU, instead "
                         "of the target tensor-parallel over the N GPUs")
    ap.add_argument("--tp-nccl", action="store_true",
                    help="N > 1: NCCL all-reduces instead of the fused NVLink reduction")
    ap.add_argument("--timeline", action="store_true",
                    help="in-situ per-kernel timeline of one verify forward (MC_TRACE build)")
    ap.add_argument("--sweep", action="store_true",
                    help="isolated quantized-projection sweep (one JSON line per point)")
    ap.add_argument("--sweep-fmt", default=None, choices=["i8_row", "q4_0"],
                    help="--sweep: this weight format only")
    ap.add_argument("--sweep-n", type=int, default=None, help="--sweep: this N only")
    ap.add_argument("--sweep-m", type=int, default=None, help="--sweep: this M only")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.sweep:
        run_sweep(args)
    elif args.timeline:
        run_timeline(args)
    elif args.profile:
        run_profile(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
