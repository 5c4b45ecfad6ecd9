"""Failure paths and the kernel-level gradient exchange (mm_gpu_comm_*, mm_gpu_allreduce_bucket,
mm_gpu_wait_selftest).

No test here faults or hangs a GPU. A bounded device wait is made to run out by a
barrier that nothing completes (the kernel then records its code and returns); a
stalled exchange is a stream that does not finish before the caller's deadline, after
which the communicator is aborted; a rank leaves a two-rank group only between
steps, with none of its work in flight, and NVLink SHARP (NVLS) is off in the
child processes.
"""
import os
import time

import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu


def test_a_bounded_wait_runs_out_and_is_reported(mm):
    mm.device_status()  # clear anything earlier
    mm.wait_selftest(200_000)  # 0.2 s
    with pytest.raises(mm.MidmanGpuError, match="bounded wait ran out") as e:
        mm.device_status()
    assert e.value.status == -6
    # the context is still usable: a product runs and the flag is clear again
    a = torch.randn(256, 128, device="cuda")
    b = torch.randn(256, 128, device="cuda")
    c = torch.empty(256, 256, device="cuda")
    mm.gemm(a, b, c, m=256, n=256, k=128, lda=128, ldb=128, ldc=256, a_mn_major=False, b_mn_major=False)
    mm.device_status()
    assert torch.allclose(c, a @ b.t(), rtol=1e-2, atol=1e-1)


def test_comm_wait_aborts_the_communicator_after_its_deadline(mm):
    comm = mm.Comm(mm.nccl_unique_id(), 1, 0)
    s = torch.cuda.Stream()
    x = torch.ones(1024, device="cuda")
    comm.allreduce(x, stream=s.cuda_stream)
    comm.wait(stream=s.cuda_stream, timeout_ms=10_000)  # finishes well inside its deadline
    assert torch.equal(x, torch.ones_like(x))
    mm.device_status()
    mm.wait_selftest(1_500_000, stream=s.cuda_stream)  # holds the stream for 1.5 s
    with pytest.raises(mm.MidmanGpuError, match="did not finish within 100 ms"):
        comm.wait(stream=s.cuda_stream, timeout_ms=100)
    with pytest.raises(mm.MidmanGpuError, match="aborted"):
        comm.allreduce(x, stream=s.cuda_stream)
    comm.close()
    s.synchronize()
    with pytest.raises(mm.MidmanGpuError, match="bounded wait ran out"):
        mm.device_status(stream=s.cuda_stream)


def _send_and_exit(q, item):
    q.put(item)
    q.close()
    q.join_thread()  # the item has left this process before it ends
    os._exit(0)


def _rank(rank, world, port, mode, q):
    import sys
    from pathlib import Path
    root = Path(__file__).resolve().parent.parent
    sys.path.insert(0, str(root / "midman-ai_b200"))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import torch
    import torch.distributed as dist
    import midman_b200 as mm
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    obj = [mm.nccl_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(obj, src=0)
    comm = mm.Comm(obj[0], world, rank)
    out = {}
    n = 1 << 20
    # step 1 on every rank: sum and mean of rank-dependent buckets
    x = torch.arange(n, device="cuda", dtype=torch.float32) * (rank + 1)
    y = torch.full((n,), float(rank + 1), device="cuda")
    comm.allreduce(x, average=False)
    comm.allreduce(y, average=True)
    comm.wait(timeout_ms=60_000)
    out["sum_ok"] = bool(torch.equal(x, torch.arange(n, device="cuda", dtype=torch.float32) * 3))
    out["mean_ok"] = bool(torch.equal(y, torch.full((n,), 1.5, device="cuda")))
    if mode == "leave":
        dist.barrier()  # both ranks finished step 1; nothing of rank 1's is in flight
        if rank == 1:
            _send_and_exit(q, (rank, out))  # leaves between steps, without a word to the others
        # step 2: the peer is gone, so the bucket's exchange cannot finish
        time.sleep(1.0)
        comm.allreduce(y, average=True)
        try:
            comm.wait(timeout_ms=5_000)
            out["error"] = None
        except mm.MidmanGpuError as e:
            out["error"] = str(e)
        comm.close()
        _send_and_exit(q, (rank, out))
    comm.close()
    dist.barrier()
    dist.destroy_process_group()
    q.put((rank, out))


def _spawn(mode):
    import multiprocessing as mp
    import socket
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    procs = [ctx.Process(target=_rank, args=(r, 2, port, mode, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=240) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    return results


def test_allreduce_bucket_on_two_ranks(mm):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    res = _spawn("ok")
    assert all(r["sum_ok"] and r["mean_ok"] for r in res.values()), res


def test_a_rank_that_leaves_ends_the_others_exchange_with_an_error(mm):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    res = _spawn("leave")
    assert res[1]["sum_ok"] and res[0]["sum_ok"]
    err = res[0]["error"]
    assert err is not None and ("did not finish" in err or "asynchronous error" in err), err

