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
Multi-GPU (torchrun): independent replicas, one request per GPU (weak
scaling); value = tokens of all ranks / max-over-ranks time.
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


def profile_traffic():
    """Per-launch DRAM bytes of the verify forward from the committed ncu summary."""
    p = os.path.join(ROOT, "profiles", "verify_traffic.json")
    if os.path.exists(p):
        with open(p) as f:
            return json.load(f).get("verify_forward_dram_bytes")
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
def cpu_sample(n_threads: int, kv_len: int = 1100):
    """Time the CPU oracle on a bounded sample of the workload: one target
    decoder layer and the LM head (f32 dequantized weights, as the reference
    holds them) for a single-token forward at KV length ~1100, repeated.
    Per-token cost extrapolates to 32 target layers + head per verify
    forward plus gamma 2-layer+head draft forwards per round."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as o
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


def cpu_tokens_per_s(t_layer, t_head, rounds, tokens, accepted):
    """Reference cost model: per round gamma draft forwards (2 layers + head)
    and the sequential verify's target forwards (min(a+1, gamma) per round,
    generate.rs:695-726); tokens = emitted tokens."""
    t_draft = 2 * t_layer + t_head
    t_target = 32 * t_layer + t_head
    target_fwd = sum(min(a + 1, GAMMA) for a in accepted) if accepted else rounds
    total = rounds * GAMMA * t_draft + target_fwd * t_target
    return tokens / total


# ---------------------------------------------------------------------- GPU
def build_models(device_index: int, layers: int | None = None):
    import torch
    import modelc_b200 as mb
    dev = torch.device("cuda", device_index)
    cfg = mb.LLAMA3_8B if not layers else mb.LLAMA3_8B.with_layers(layers)
    dcfg = cfg.with_layers(2)
    tt = mb.synth_weights_torch(cfg, seed=0, device=dev)
    target = mb.Weights(tt, cfg, device=device_index)
    del tt
    dt = mb.synth_weights_torch(dcfg, seed=1, device=dev)
    draft = mb.Weights(dt, dcfg, device=device_index)
    del dt
    torch.cuda.empty_cache()
    g = torch.Generator(device="cpu")
    g.manual_seed(2)
    prompt = torch.randint(0, cfg.vocab, (PROMPT_LEN,), generator=g).numpy().astype(np.uint32)
    return cfg, target, draft, prompt


def run_ours(args):
    import torch
    import modelc_b200 as mb
    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=300))
    cfg, target, draft, prompt = build_models(local)
    max_ctx = PROMPT_LEN + NEW_TOKENS + 2 * GAMMA + 8
    sess = mb.Session(target, draft, gamma=GAMMA, max_context=max_ctx)
    stream = torch.cuda.ExternalStream(sess.stream_ptr, device=torch.device("cuda", local))

    def barrier():
        torch.cuda.synchronize()
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize()

    # ---- device-resident decode: prime once, each step decodes 256 tokens
    sess.prime(prompt)
    for _ in range(args.warmup):
        sess.rewind()
        sess.decode(NEW_TOKENS)
    barrier()
    tokens = 0
    rounds = 0
    accepted = []
    ev = []
    with ClockSampler(local) as clk:
        for _ in range(args.steps):
            sess.rewind()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            n = sess.decode(NEW_TOKENS)
            e1.record(stream)
            ev.append((e0, e1))
            toks, acc = sess.read()
            tokens += len(toks)
            rounds += len(acc)
            accepted += acc
    barrier()
    ms = sum(a.elapsed_time(b) for a, b in ev)
    t_local = torch.tensor([ms / 1e3], device="cuda")
    n_local = torch.tensor([float(tokens)], device="cuda")
    if world > 1:
        torch.distributed.all_reduce(t_local, op=torch.distributed.ReduceOp.MAX)
        torch.distributed.all_reduce(n_local, op=torch.distributed.ReduceOp.SUM)
    t_total, tok_total = float(t_local.item()), float(n_local.item())
    value = tok_total / t_total
    ms_per_step = t_total * 1e3 / args.steps
    launches = rounds * sess.round_launches

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
    kv_bytes = 2 * cfg.n_layers * (kv_len + vm) * cfg.n_kv_heads * cfg.head_dim * 4
    act_bytes = 2 * cfg.n_layers * vm * (3 * cfg.hidden + 2 * cfg.ffn) * 4
    algo = target.streamed_bytes + kv_bytes + act_bytes
    peak, peak_kind = measured_peaks()
    achieved = algo / t_ver / 1e9
    traffic = profile_traffic()
    roof = {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
            "frac": round(achieved / peak, 4), "traffic": traffic,
            "peak_source": peak_kind, "kernel": "verify forward (k_gemv + fused kernels, 291 launches)",
            "algorithmic_bytes": algo, "ms": round(t_ver * 1e3, 4)}

    # ---- end to end through the C ABI (host buffers, prime included)
    e2e_ms = []
    h2d = PROMPT_LEN * 4
    for i in range(max(1, min(args.steps, 3)) + 1):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        toks, acc = sess.speculative_generate(prompt, NEW_TOKENS)
        e1.record(stream)
        torch.cuda.synchronize()
        if i > 0:
            e2e_ms.append(e0.elapsed_time(e1))
    d2h = (len(toks) + len(acc)) * 4
    e2e_local = torch.tensor([statistics.mean(e2e_ms) / 1e3], device="cuda")
    if world > 1:
        torch.distributed.all_reduce(e2e_local, op=torch.distributed.ReduceOp.MAX)
    e2e_value = len(toks) * world / float(e2e_local.item())

    line = None
    if rank == 0:
        cpu = None
        if not args.no_cpu:
            nthr = os.cpu_count() or 1
            t_layer, t_head, rl, rh = cpu_sample(nthr)
            cpu = {"value": round(cpu_tokens_per_s(t_layer, t_head, rounds, tokens, accepted), 5),
                   "unit": "tokens/s", "cores": nthr, "kind": "port",
                   "sample": (f"oracle row-parallel f32 forward of 1 target layer at KV 1100 "
                              f"({t_layer * 1e3:.1f} ms, {rl} reps) + LM head ({t_head * 1e3:.1f} ms, "
                              f"{rh} reps), extrapolated to 32 layers + head per target forward and "
                              f"{GAMMA} 2-layer drafts per round with this run's acceptance")}
        clocks = clk.summary()
        line = {
            "metric": METRIC, "value": round(value, 3), "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_per_step, 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8",
            "data": "synthetic (random-init weights N(0,0.02), uniform prompt ids)",
            "config": {"workload": WORKLOAD, "target": cfg.name, "draft_layers": 2,
                       "prompt_len": PROMPT_LEN, "new_tokens": NEW_TOKENS, "gamma": GAMMA,
                       "batch": 1, "parallelism": f"replicas{world}" if world > 1 else "single",
                       "l2": "inputs larger than L2 (7.5 GB int8 weights per verify)"},
            "roofline": roof, "cpu_baseline": cpu,
            "e2e": {"value": round(e2e_value, 3), "unit": "tokens/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "includes": "prime (1024-token prefill) + decode"},
            "clocks": clocks, "gpu_launches": int(launches * world),
            "acceptance": {"rounds": rounds, "tokens": tokens,
                           "mean_accepted": round(float(np.mean(accepted)) if accepted else 0.0, 4)},
        }
    sess.close()
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()
    if line:
        print(json.dumps(line), flush=True)


def run_profile(args):
    """Short run for ncu launch lists: prime the 1024-token prompt, then
    3 verify forwards and 2 speculative rounds.  Launch counts before the
    verify forwards are printed so a capture can skip exactly to them."""
    import torch
    import modelc_b200 as mb
    torch.cuda.set_device(0)
    cfg, target, draft, prompt = build_models(0, args.layers)
    sess = mb.Session(target, draft, gamma=GAMMA,
                      max_context=PROMPT_LEN + NEW_TOKENS + 2 * GAMMA + 8)
    sess.prime(prompt)
    torch.cuda.synchronize()
    chunks_t = -(-PROMPT_LEN // 16)
    chunks_d = -(-(PROMPT_LEN - 1) // 16)
    per_t = (sess.round_launches - 1 - GAMMA * 21)
    print(json.dumps({"prime_launches": chunks_t * (1 + per_t) + chunks_d * (1 + 21),
                      "verify_launches": per_t, "round_launches": sess.round_launches}),
          flush=True)
    sess.verify_launch(3)
    torch.cuda.synchronize()
    sess.decode(2)
    torch.cuda.synchronize()
    sess.close()


def run_reference(args):
    rank, world, _ = dist_env()
    if rank != 0:
        return
    nthr = os.cpu_count() or 1
    vals = []
    t0 = time.time()
    # acceptance of unrelated random-init target/draft models is ~1/vocab:
    # every round emits one token after one target forward
    for i in range(args.warmup + args.steps):
        t_layer, t_head, rl, rh = cpu_sample(nthr)
        if i >= args.warmup:
            vals.append(cpu_tokens_per_s(t_layer, t_head, 1, 1, [0]))
    v = statistics.mean(vals)
    sample = (f"per step: oracle row-parallel f32 forward of 1 target layer at KV 1100 + LM head, "
              f"extrapolated to one round (32-layer verify forward + {GAMMA} 2-layer draft "
              f"forwards) emitting one token")
    line = {"impl": "reference", "metric": METRIC, "value": round(v, 5), "unit": "tokens/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round((time.time() - t0) * 1e3 / (args.warmup + args.steps), 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "config": {"workload": WORKLOAD, "target": "llama3-8b"},
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
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.profile:
        run_profile(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
