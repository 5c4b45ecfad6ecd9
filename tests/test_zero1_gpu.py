"""Optimizer-state sharding (midman_train_shard_optimizer) on 2 GPUs.

A sharded run (each rank keeps the AdamW moments of its range; gradients reduced
to their owners, the owners' updates broadcast) against the unsharded data-parallel
run of the same batches: the same steps to rounding, identical parameters on both
ranks, moments gathered through the collective read, a state file written by rank
0 that a fresh sharded run resumes bit-for-bit, and the moments gathered back when
sharding is turned off. The AdamW update it shards is adamw.rs:141-217 with the
global-norm clip of clip.rs:29-59. Needs two GPUs; skipped on one.
"""
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

HYPER = dict(max_lr=0.02, min_lr=0.002, warmup=2, total=40, weight_decay=0.1, clip_norm=1.0, beta1=0.9, beta2=0.95)


def _worker(rank, world, port, cfg, B, T, data, params, path, q):
    import sys
    from pathlib import Path
    root = Path(__file__).resolve().parent.parent
    sys.path.insert(0, str(root / "midman-ai_b200"))
    import torch
    import torch.distributed as dist
    import midman_b200 as mm
    torch.cuda.set_device(rank)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    dist.init_process_group("gloo", rank=rank, world_size=world)
    ids = [mm.nccl_unique_id() if rank == 0 else None for _ in range(3)]
    dist.broadcast_object_list(ids, src=0)

    def trainer(k):
        t = mm.Trainer(cfg, mm.hyper_array(**HYPER), seed=0, batch=B, seq=T, precision=1, world=world, rank=rank,
                       nccl_id=ids[k])
        t.load_params(params)
        return t

    out = {}
    plain, zero = trainer(0), trainer(1)
    out["sharding"] = zero.shard_optimizer(True)
    sl = slice(rank * B * T, (rank + 1) * B * T)
    recs_p, recs_z = [], []
    for x, y in data[:4]:
        recs_p.append(plain.step(x[sl], y[sl]))
        recs_z.append(zero.step(x[sl], y[sl]))
    out["recs"] = (recs_p, recs_z)
    out["params"] = (plain.params(), zero.params())
    out["moments"] = ((plain.read(2), plain.read(3)), (zero.read(2), zero.read(3)))
    try:
        zero.grads()
        out["grads_refused"] = False
    except mm.MidmanError:
        out["grads_refused"] = True
    zero.save(path, data_seed=5, epoch=0, position=4)  # collective; rank 0 writes
    dist.barrier()
    resumed = trainer(2)
    resumed.shard_optimizer(True)
    out["progress"] = resumed.restore(path, data_seed=5)
    x, y = data[4]
    out["next"] = (zero.step(x[sl], y[sl]), resumed.step(x[sl], y[sl]))
    out["after_next"] = (zero.params(), resumed.params())
    gathered = zero.shard_optimizer(False)
    out["unsharded"] = (gathered["optimizer"], zero.read(2), zero.read(3))
    for t in (plain, zero, resumed):
        t.close()
    dist.barrier()
    dist.destroy_process_group()
    q.put((rank, out))


def test_sharded_adamw_matches_the_replicated_step(mm, tmp_path):
    torch = pytest.importorskip("torch")
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import multiprocessing as mp
    import socket
    import oracle as orc
    cfg = orc.config_array(64, 32, 2, 4, 2, 48, 16)
    B, T = 2, 16
    model = orc.Model(cfg, seed=11, init_std=0.1)
    r = orc.Rng(13)
    data = []
    for _ in range(5):
        ids = np.array([r.below(64) for _ in range(2 * B * (T + 1))], np.int32).reshape(2 * B, T + 1)
        data.append((ids[:, :T].ravel().copy(), ids[:, 1:].ravel().copy()))
    path = tmp_path / "zero.safetensors"
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    procs = [ctx.Process(target=_worker, args=(k, 2, port, cfg, B, T, data, model.params, str(path), q))
             for k in range(2)]
    for p in procs:
        p.start()
    out = dict(q.get(timeout=600) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    total = model.params.size
    # the ranges tile the vector and end on blocks of the fixed 1184-block norm grid
    per = ((total + 1183) // 1184 + 3) & ~3
    ranges = out[0]["sharding"]["ranges"]
    assert out[0]["sharding"]["optimizer"] and ranges == out[1]["sharding"]["ranges"]
    assert ranges[0][0] == 0 and ranges[0][1] == ranges[1][0] and ranges[1][1] == total
    assert ranges[0][1] == min(total, per * 592)
    for rank in (0, 1):
        o = out[rank]
        recs_p, recs_z = o["recs"]
        for (rp, sp), (rz, sz) in zip(recs_p, recs_z):
            assert sp == sz == 0
            assert abs(rz[0] - rp[0]) <= 1e-6 * abs(rp[0]) and abs(rz[1] - rp[1]) <= 1e-5 * abs(rp[1])
        pp, pz = o["params"]
        assert np.max(np.abs(pz - pp)) <= 1e-6
        (mp_, vp), (mz, vz) = o["moments"]
        assert np.linalg.norm(mz - mp_) <= 1e-5 * np.linalg.norm(mp_)
        assert np.linalg.norm(vz - vp) <= 1e-5 * np.linalg.norm(vp)
        assert o["grads_refused"]
        assert o["progress"] == {"step": 4, "epoch": 0, "position": 4}
        (rz, sz), (rr, sr) = o["next"]
        assert sz == sr == 0 and np.array_equal(rz, rr)  # the resumed sharded run continues bit for bit
        assert np.array_equal(o["after_next"][0], o["after_next"][1])
        on, m_all, v_all = o["unsharded"]
        assert not on and np.all(np.isfinite(m_all)) and np.all(v_all >= 0)
    # the ranks agree exactly
    assert np.array_equal(out[0]["params"][1], out[1]["params"][1])
    assert np.array_equal(out[0]["moments"][1][0], out[1]["moments"][1][0])
    assert np.array_equal(out[0]["unsharded"][1], out[1]["unsharded"][1])
    assert path.exists()
