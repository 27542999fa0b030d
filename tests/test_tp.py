"""Tensor parallelism (Megatron) for the verify forward.

CPU, world size 2 over gloo: the sharding the library applies, done here
with numpy on the oracle's f32 weights, reproduces the unsharded results:
column-parallel q/k/v (by heads) and gate/up (by FFN rows), row-parallel o
and down (partial sums + one all-reduce), and the vocab-parallel LM head
whose per-rank argmax keys merge with a MAX all-reduce into the global
first-index argmax (generate.rs:1088-1098 tie rule).

GPU (2, 4 and 8 ranks, each skipped without that many devices): every rank
holds its shard of the target and a replicated draft and decodes greedily -
with NCCL all-reduces in the round graph; with the fused NVLink exchange
(partial rows stored into every rank's buffer by the GEMV, argmax keys
merged over peer memory) next to an NCCL communicator; and with the fused
exchange alone, no NCCL at all - and produces exactly the oracle's tokens and
accepted counts.  Two ranks also run as two host threads of one process,
whose exchange buffers open each other directly.
"""
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "oracle"))


def _argmax_key(v, idx):
    b = np.float32(v).view(np.uint32).item()
    o = (~b) & 0xFFFFFFFF if b & 0x80000000 else b | 0x80000000
    return (o << 32) | ((~idx) & 0xFFFFFFFF)


def _key_index(k):
    return (~k) & 0xFFFFFFFF


def _tp_worker(rank, world, port, q):
    import torch
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        rng = np.random.default_rng(5)
        d, H, Hkv, hd, F, V = 64, 4, 2, 16, 96, 50
        x = rng.standard_normal(d).astype(np.float32)
        wq = rng.standard_normal((H * hd, d)).astype(np.float32)
        wk = rng.standard_normal((Hkv * hd, d)).astype(np.float32)
        wo = rng.standard_normal((d, H * hd)).astype(np.float32)
        wg = rng.standard_normal((F, d)).astype(np.float32)
        wd = rng.standard_normal((d, F)).astype(np.float32)
        wh = rng.standard_normal((V, d)).astype(np.float32)
        wh[7] = wh[31] = 3.0 * x  # the maximum, tied across the two shards: 7 must win
        hl, kl, fl, vl = H // world, Hkv // world, F // world, V // world
        # column-parallel: this rank's heads / FFN rows
        q_loc = wq[rank * hl * hd:(rank + 1) * hl * hd] @ x
        k_loc = wk[rank * kl * hd:(rank + 1) * kl * hd] @ x
        g_loc = wg[rank * fl:(rank + 1) * fl] @ x
        assert np.allclose(q_loc, (wq @ x)[rank * hl * hd:(rank + 1) * hl * hd])
        assert np.allclose(k_loc, (wk @ x)[rank * kl * hd:(rank + 1) * kl * hd])
        # row-parallel: partial sums of this rank's input slice + all-reduce
        a_full = rng.standard_normal(H * hd).astype(np.float32)
        f_full = rng.standard_normal(F).astype(np.float32)
        po = torch.from_numpy(wo[:, rank * hl * hd:(rank + 1) * hl * hd] @
                              a_full[rank * hl * hd:(rank + 1) * hl * hd])
        pd = torch.from_numpy(wd[:, rank * fl:(rank + 1) * fl] @ f_full[rank * fl:(rank + 1) * fl])
        dist.all_reduce(po)
        dist.all_reduce(pd)
        ok_o = np.allclose(po.numpy(), wo @ a_full, rtol=1e-5, atol=1e-4)
        ok_d = np.allclose(pd.numpy(), wd @ f_full, rtol=1e-5, atol=1e-4)
        # vocab-parallel head: local keys with global indices, MAX all-reduce
        logits = wh[rank * vl:(rank + 1) * vl] @ x
        best = max(_argmax_key(v, rank * vl + i) for i, v in enumerate(logits))
        kt = torch.tensor([best >> 1, best & 1], dtype=torch.int64)  # 63-bit safe split
        kts = [torch.zeros_like(kt) for _ in range(world)]
        dist.all_gather(kts, kt)
        merged = max((int(t[0]) << 1) | int(t[1]) for t in kts)
        full = wh @ x
        ok_h = _key_index(merged) == int(np.argmax(full))
        q.put((rank, ok_o and ok_d and ok_h, _key_index(merged), g_loc.shape[0] == fl))
    finally:
        dist.destroy_process_group()


def test_megatron_sharding_reproduces_unsharded_gloo():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29500 + (os.getpid() % 2000)
    procs = [ctx.Process(target=_tp_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert all(ok for _, ok, _, _ in res), res
    assert all(idx == 7 for _, _, idx, _ in res)
    assert all(shape for *_, shape in res)


def _gpu_rank(rank, world, uid, cfg_args, prompt, gamma, fused, port, q):
    import torch
    import torch.distributed as dist
    import modelc_b200 as mb
    from modelc_b200.model import LlamaConfig
    torch.cuda.set_device(rank)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        cfg = LlamaConfig(*cfg_args)
        tw = mb.synth_weights(cfg, seed=0)
        dw = mb.synth_weights(cfg.with_layers(1), seed=1)
        W = mb.Weights(tw, cfg, device=rank, tp_rank=rank, tp_world=world)
        D = mb.Weights(dw, cfg.with_layers(1), device=rank)
        s = mb.Session(W, D, gamma=gamma, max_context=128)
        if fused != "fused-only":
            s.tp_init(uid, rank, world)
        if fused:
            handles = [None] * world
            dist.all_gather_object(handles, s.tp_ipc_handle())
            s.tp_open_peers(handles)
        toks, acc = s.speculative_generate(prompt, 24)
        dist.barrier()  # no rank frees its reduce buffer while a peer may write it
        s.close()
        q.put((rank, toks, acc))
    finally:
        dist.destroy_process_group()


# per world size: a GQA shape whose heads, KV heads and FFN rows divide
# evenly (8 ranks: one KV head each; vocab shards of uneven stripe counts)
TP_CFGS = {2: (2, 128, 4, 2, 32, 192, 260), 4: (2, 256, 8, 4, 32, 384, 520),
           8: (2, 256, 8, 8, 32, 512, 1032)}


def _tp_reference(world):
    import oracle as o
    import modelc_b200 as mb
    from modelc_b200.model import LlamaConfig, MODE_GENERAL
    cfg = LlamaConfig(*TP_CFGS[world], 500000.0, 1e-5, MODE_GENERAL, f"tp{world}-gqa")
    prompt = np.random.default_rng(11).integers(0, cfg.vocab, 13).tolist()
    tw = mb.synth_weights(cfg, seed=0)
    dw = mb.synth_weights(cfg.with_layers(1), seed=1)

    def om(ws, c):
        return o.OracleModel({k: v.dequant() for k, v in ws.items()}, c.n_layers, c.hidden,
                             c.vocab, c.ffn, mode=c.mode, n_heads=c.n_heads,
                             n_kv_heads=c.n_kv_heads, head_dim=c.head_dim,
                             rope_base=c.rope_theta, eps=c.eps)
    ref, racc = om(tw, cfg).speculative_generate(
        prompt, 24, 4, o.OracleLlamaDraft(om(dw, cfg.with_layers(1)), 128))
    return cfg, tw, dw, prompt, ref, racc


@pytest.mark.gpu
@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("fused", [False, True, "fused-only"],
                         ids=["nccl", "fused-nvlink", "fused-only"])
def test_tp_spec_decode_matches_oracle(world, fused):
    import torch
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp
    import modelc_b200 as mb
    cfg, tw, dw, prompt, ref, racc = _tp_reference(world)
    uid = mb.tp_unique_id()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    args = (cfg.n_layers, cfg.hidden, cfg.n_heads, cfg.n_kv_heads, cfg.head_dim, cfg.ffn,
            cfg.vocab, cfg.rope_theta, cfg.eps, cfg.mode, cfg.name)
    port = 31000 + (os.getpid() % 2000) + {False: 0, True: 7, "fused-only": 3}[fused] + 13 * world
    procs = [ctx.Process(target=_gpu_rank, args=(r, world, uid, args, prompt, 4, fused, port, q))
             for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for _, toks, acc in res:
        assert toks == ref
        assert acc == racc


@pytest.mark.gpu
def test_tp_ranks_as_threads_of_one_process():
    """Two ranks as two host threads of this process (one GPU each): their
    exchange buffers open each other directly (CUDA IPC cannot map an
    allocation into the process that made it), no NCCL."""
    import threading
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import modelc_b200 as mb
    cfg, tw, dw, prompt, ref, racc = _tp_reference(2)
    sessions, handles, out = [None, None], [None, None], [None, None]
    errors = []
    bar = threading.Barrier(2, timeout=120)

    def rank(r):
        try:
            W = mb.Weights(tw, cfg, device=r, tp_rank=r, tp_world=2)
            D = mb.Weights(dw, cfg.with_layers(1), device=r)
            s = mb.Session(W, D, gamma=4, max_context=128)
            sessions[r] = (W, D, s)
            handles[r] = s.tp_ipc_handle()
            bar.wait()
            s.tp_open_peers(handles)
            bar.wait()
            out[r] = s.speculative_generate(prompt, 24)
        except Exception as e:  # reported below; the barrier frees the peer
            errors.append(repr(e))
            bar.abort()
        finally:
            try:
                bar.wait()  # no rank frees its buffer while the peer may write it
            except threading.BrokenBarrierError:
                pass

    th = [threading.Thread(target=rank, args=(r,)) for r in range(2)]
    for t in th:
        t.start()
    for t in th:
        t.join(timeout=300)
    for trio in sessions:
        if trio:
            trio[2].close()
            trio[0].close()
            trio[1].close()
    assert not errors, errors
    for toks, acc in out:
        assert toks == ref
        assert acc == racc
