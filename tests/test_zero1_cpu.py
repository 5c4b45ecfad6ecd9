"""Optimizer sharding's exchange, on CPU with two gloo ranks.

The library's plan (midman_shard_plan: each rank's range of the flat parameter
vector and the gradient buckets, the numbers a sharded trainer uses) drives the
exchange a sharded step makes, here with torch.distributed on CPU and the
oracle's gradients: each bucket reduced to the ranks owning its parts, the
global norm from the ranks' shares of the fixed 1,184-block sum-of-squares grid,
an AdamW update of the own range, the owners' parts broadcast. The result must be
the replicated step's bit for bit: the reduced gradients, the norm's partials and
the updated parameters (the update is AdamW of crates/midman-optim/src/adamw.rs:
141-217 with the clip of clip.rs:29-59, restated elementwise in numpy here).
"""
import os
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent


def _plan_checks(plan, total):
    ranges, buckets = plan["ranges"], plan["buckets"]
    assert ranges[0][0] == 0 and ranges[-1][1] == total
    assert all(a[1] == b[0] for a, b in zip(ranges, ranges[1:]))
    assert all(r[0] % plan["norm_block"] == 0 for r in ranges)
    assert buckets[0][0] == 0 and buckets[-1][1] == total
    assert all(a[1] == b[0] for a, b in zip(buckets, buckets[1:]))


def test_the_plan_tiles_the_vector(mm):
    import oracle as orc
    for cfg in (orc.config_array(64, 32, 2, 4, 2, 48, 16), orc.preset("large")):
        total = orc.param_breakdown(cfg)["total"]
        for world in (1, 2, 3, 8):
            plan = mm.shard_plan(cfg, world)
            assert plan["params"] == total and len(plan["ranges"]) == world
            _plan_checks(plan, total)
            assert len(plan["buckets"]) == int(cfg[2]) + 2
    with pytest.raises(mm.MidmanError):
        mm.shard_plan(orc.config_array(64, 32, 2, 4, 3, 48, 16), 2)  # heads not a multiple of kv heads


def _partials(vec, lo, hi, per, nb):
    n = vec.size
    out = np.zeros(nb)
    for b in range(nb):
        beg, end = b * per, min((b + 1) * per, n)
        if beg < end and beg >= lo and end <= hi:
            out[b] = np.sum(vec[beg:end].astype(np.float64) ** 2)
    return out


def _adamw(p, g, m, v, decay, factor, lr, step, b1=0.9, b2=0.95, eps=1e-8, wd=0.1):
    f32 = np.float32
    gr = (g * f32(factor)).astype(f32)
    x = np.where(decay, p * f32(1.0 - lr * wd), p).astype(f32)
    m2 = (f32(b1) * m + f32(1 - b1) * gr).astype(f32)
    v2 = (f32(b2) * v + f32(1 - b2) * gr * gr).astype(f32)
    bias1 = f32(1.0 - b1 ** step)
    bias2_sqrt = f32(np.sqrt(1.0 - b2 ** step))
    x = (x - f32(lr / bias1) * m2 / (np.sqrt(v2) / bias2_sqrt + f32(eps))).astype(f32)
    return x, m2, v2


def _rank(rank, world, port, q):
    sys.path[:0] = [str(ROOT / "midman-ai_b200"), str(ROOT / "oracle")]
    import torch
    import torch.distributed as dist
    import midman_b200 as mm
    import oracle as orc
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        cfg = orc.config_array(64, 32, 2, 4, 2, 48, 16)
        B, T = 2, 16
        plan = mm.shard_plan(cfg, world)
        model = orc.Model(cfg, seed=3, init_std=0.1)
        params = model.params.astype(np.float32)
        n = params.size
        decay = np.zeros(n, bool)
        for _name, shape, off, cnt in model.tensors():
            decay[off:off + cnt] = len(shape) >= 2
        r = orc.Rng(5)
        ids = np.array([r.below(64) for _ in range(world * B * (T + 1))], np.int32).reshape(world * B, T + 1)
        x = ids[rank * B:(rank + 1) * B, :T].ravel().copy()
        y = ids[rank * B:(rank + 1) * B, 1:].ravel().copy()
        _loss, g = model.loss(x, y, B, T, grads=True)
        g = np.asarray(g, np.float32)
        # replicated: every rank averages the whole gradient
        g_rep = torch.from_numpy(g.copy())
        dist.all_reduce(g_rep)
        g_rep = (g_rep / world).numpy()
        # sharded: each bucket's parts reduced to their owners
        g_sh = g.copy()
        for b0, b1 in plan["buckets"]:
            for owner, (lo, hi) in enumerate(plan["ranges"]):
                a, b = max(b0, lo), min(b1, hi)
                if a < b:
                    piece = torch.from_numpy(g_sh[a:b].copy())
                    dist.reduce(piece, dst=owner)
                    if rank == owner:
                        g_sh[a:b] = (piece / world).numpy()
        lo, hi = plan["ranges"][rank]
        same_grads = bool(np.array_equal(g_sh[lo:hi].view(np.uint32), g_rep[lo:hi].view(np.uint32)))
        # the norm from the ranks' shares of the fixed grid
        per, nb = plan["norm_block"], plan["norm_blocks"]
        full = _partials(g_rep, 0, n, per, nb)
        mine = torch.from_numpy(_partials(g_sh, lo, hi, per, nb))
        dist.all_reduce(mine)
        same_partials = bool(np.array_equal(mine.numpy(), full))
        norm = np.float32(np.sqrt(np.sum(full)))
        factor = 1.0 / (norm + 1e-6) if norm > 1.0 else 1.0
        zeros = np.zeros(n, np.float32)
        p_rep, _, _ = _adamw(params, g_rep, zeros, zeros, decay, factor, 0.01, 1)
        p_sh = params.copy()
        p_sh[lo:hi], _, _ = _adamw(params[lo:hi], g_sh[lo:hi], zeros[lo:hi], zeros[lo:hi], decay[lo:hi], factor,
                                   0.01, 1)
        for b0, b1 in plan["buckets"]:
            for owner, (olo, ohi) in enumerate(plan["ranges"]):
                a, b = max(b0, olo), min(b1, ohi)
                if a < b:
                    t = torch.from_numpy(p_sh[a:b].copy())
                    dist.broadcast(t, src=owner)
                    p_sh[a:b] = t.numpy()
        same_params = bool(np.array_equal(p_sh.view(np.uint32), p_rep.view(np.uint32)))
        q.put((rank, (same_grads, same_partials, same_params, bool(np.any(p_rep != params)))))
    finally:
        dist.destroy_process_group()


def test_the_sharded_exchange_equals_the_replicated_step():
    import multiprocessing as mp
    import socket
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=180) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert results == {0: (True, True, True, True), 1: (True, True, True, True)}
