"""Token feed (midman_batcher_*, crates/midman-data/src/batch.rs) on the CPU: bit-exact with the
oracle's restatement across epochs, and the data-parallel split of a global batch across ranks
(rank r trains rows [r*B, (r+1)*B)) checked with two gloo processes.
"""
import os

import numpy as np
import pytest

import oracle as orc


def test_batcher_matches_the_oracle_bit_for_bit(mm):
    toks = orc.Rng(3)
    tokens = np.array([toks.below(500) for _ in range(4001)], np.uint32)
    ours = mm.Batcher(tokens, vocab=500, seq=16, batch=7, seed=99)
    ref = orc.Batcher(tokens, 16, 7, 99)
    assert len(ref) == 250
    for _ in range(3 * (250 // 7) + 5):  # crosses epoch boundaries
        i, t, e, x = ours.next()
        ri, rt, re, rx = ref.next()
        assert np.array_equal(i, ri) and np.array_equal(t, rt) and (e, x) == (re, rx)
    ours.close()


def test_synthetic_shard_is_rng_below(mm):
    b = mm.Batcher(vocab=1000, seq=4, batch=1, seed=0, synthetic_tokens=41, token_seed=5)
    r = orc.Rng(5)
    want = [r.below(1000) for _ in range(41)]
    seen = {}
    for _ in range(10):
        i, t, _, _ = b.next()
        seen[tuple(i)] = t
    windows = {tuple(want[4 * k:4 * k + 4]) for k in range(10)}
    assert set(seen) == windows
    b.close()


def test_bad_batcher_arguments(mm):
    with pytest.raises(mm.MidmanError) as e:
        mm.Batcher(np.arange(10, dtype=np.uint32), vocab=5, seq=4, batch=1)
    assert e.value.status == -4
    with pytest.raises(mm.MidmanError) as e:
        mm.Batcher(np.arange(10, dtype=np.uint32), vocab=50, seq=4, batch=5)
    assert e.value.status == -1 and "fewer than one batch" in e.value.message


def _rank(rank, world, port, q):
    import sys
    from pathlib import Path
    root = Path(__file__).resolve().parent.parent
    sys.path.insert(0, str(root / "midman-ai_b200"))
    import torch
    import torch.distributed as dist
    import midman_b200 as mm
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    B, T = 3, 8
    b = mm.Batcher(vocab=777, seq=T, batch=B * world, seed=0, synthetic_tokens=2000, token_seed=0)
    ok = True
    for _ in range(4):
        i, t, _, _ = b.next()
        mine = torch.from_numpy(i[rank * B * T:(rank + 1) * B * T].copy())
        parts = [torch.zeros_like(mine) for _ in range(world)]
        dist.all_gather(parts, mine)
        ok &= bool(torch.equal(torch.cat(parts), torch.from_numpy(i)))
    dist.destroy_process_group()
    q.put((rank, ok))


def test_data_parallel_shards_partition_the_global_batch():
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
    results = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert results == {0: True, 1: True}
