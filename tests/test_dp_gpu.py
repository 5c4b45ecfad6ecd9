"""Data parallelism on 2 GPUs: a step on two ranks (each its half of the batch, gradients
averaged by NCCL inside the library) equals a one-GPU step on the whole batch.

This is the parity check of the one exchange step of the hot path (the bucketed gradient
allreduce); it needs two GPUs and is skipped on one.
"""
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _worker(rank, world, port, cfg, B, T, inputs, targets, params, q):
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
    obj = [mm.nccl_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(obj, src=0)
    t = mm.Trainer(cfg, mm.hyper_array(), seed=0, batch=B, seq=T, precision=1, world=world, rank=rank,
                   nccl_id=obj[0])
    t.load_params(params)
    sl = slice(rank * B * T, (rank + 1) * B * T)
    loss = t.loss_and_grads(inputs[sl], targets[sl])
    grads = t.grads()
    rec, status = t.step(inputs[sl], targets[sl])
    after = t.params()
    t.close()
    dist.barrier()
    dist.destroy_process_group()
    q.put((rank, loss, grads, status, rec, after))


def test_two_rank_step_equals_the_one_gpu_step(mm):
    torch = pytest.importorskip("torch")
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import multiprocessing as mp
    import socket
    import oracle as orc
    cfg = orc.config_array(64, 32, 2, 4, 2, 48, 16)
    B, T = 2, 16
    model = orc.Model(cfg, seed=11, init_std=0.3)
    r = orc.Rng(12)
    inputs = np.array([r.below(64) for _ in range(2 * B * T)], np.int32)
    targets = np.array([r.below(64) for _ in range(2 * B * T)], np.int32)
    params = model.params
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    procs = [ctx.Process(target=_worker, args=(k, 2, port, cfg, B, T, inputs, targets, params, q)) for k in range(2)]
    for p in procs:
        p.start()
    out = dict((x[0], x[1:]) for x in (q.get(timeout=300) for _ in procs))
    for p in procs:
        p.join(timeout=60)
    # one GPU, whole batch
    torch.cuda.set_device(0)
    one = mm.Trainer(cfg, mm.hyper_array(), seed=0, batch=2 * B, seq=T, precision=1)
    one.load_params(params)
    loss1 = one.loss_and_grads(inputs, targets)
    g1 = one.grads()
    rec1, _ = one.step(inputs, targets)
    p1 = one.params()
    one.close()
    for rank in (0, 1):
        loss, grads, status, rec, after = out[rank]
        assert status == 0
        assert abs(loss - loss1) <= 1e-6 * abs(loss1)
        assert np.linalg.norm(grads - g1) / np.linalg.norm(g1) <= 1e-5
        assert abs(rec[1] - rec1[1]) <= 1e-5 * rec1[1]  # global gradient norm
        assert np.max(np.abs(after - p1)) <= 1e-6
    assert np.array_equal(out[0][3], out[1][3])  # ranks agree exactly: step record
    assert np.array_equal(out[0][4], out[1][4])  # and updated parameters
