"""Training-step throughput of the MidMan decoder on B200: tokens/s (fwd + bwd + AdamW).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config large|mid|tiny|smoke|linear|attention]
                    [--precision tf32|3xtf32] [--impl ours|reference]

One process per GPU (torchrun for N > 1); each rank trains its own B x T shard of
a global batch drawn by the reference's Batcher from a synthetic shard of
uniform token ids (seed 0), with weights from the reference's seeded init.
Gradients are averaged across ranks with NCCL inside the library (weak scaling:
the per-GPU batch is fixed). Rank 0 prints one JSON line.

`value` times K steps on a batch already in HBM (midman_train_step_staged),
with CUDA events on the library's stream, max over ranks. `e2e` times K steps
of midman_train_run, the library's training loop over the batcher: taking each
global batch on the host, the host-to-device copy of this rank's ids and the
read-back of its loss and gradient norm are inside the timed region (the host
prepares batch s+1 while the GPU runs step s). `--impl reference` times the CPU restatement of the reference's
f32 path (oracle/) on a bounded sample of the same workload on all host cores.
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
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "midman-ai_b200"))

# (preset/config tuple, batch per GPU, seq)
CONFIGS = {
    # large preset, 1,009,338,368 params, 4 x 2048 per GPU
    "large": ((32000, 2048, 20, 16, 8, 5632, 2048), 4, 2048),
    # mid-size decoder (Hkv assumed 16 = MHA), 8 x 1024 per GPU
    "mid": ((32768, 1024, 16, 16, 16, 2816, 1024), 8, 1024),
    # tiny preset, 8 x 256
    "tiny": ((4096, 128, 4, 4, 4, 344, 256), 8, 256),
    "smoke": ((256, 64, 2, 4, 4, 176, 128), 4, 128),
}


def flops_per_token(cfg, seq):
    """Algorithmic training FLOPs per token: 6 x (matmul params incl. the head) + causal attention
    (QK^T and PV forward, twice that backward: 3 x 2 x 2 x T/2 x d per layer)."""
    v, d, l, h, kv_h, ff, _ = cfg
    hd = d // h
    kv = kv_h * hd
    matmul = l * (2 * d * d + 2 * d * kv + 3 * d * ff) + d * v
    attn = l * 3 * 2 * 2 * seq / 2 * d
    return 6 * matmul + attn


def sample_clocks(stop: threading.Event, out: list, gpu_index: int):
    q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    try:
        p = subprocess.Popen(["nvidia-smi", f"--query-gpu={q}", "--format=csv,noheader,nounits", "-lms", "200",
                              "-i", str(gpu_index)], stdout=subprocess.PIPE, text=True)
    except FileNotFoundError:
        return
    try:
        while not stop.is_set():
            line = p.stdout.readline()
            if not line:
                break
            out.append([x.strip() for x in line.split(",")])
    finally:
        p.terminate()
        try:
            p.wait(timeout=5)
        except subprocess.TimeoutExpired:
            p.kill()


def summarize_clocks(rows):
    if not rows:
        return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unavailable"]}
    sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
    mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
    names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
    reasons = set()
    for r in rows:
        for i, n in enumerate(names):
            if len(r) > 5 + i and r[5 + i].lower().startswith("active"):
                reasons.add(n)
    return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
            "reasons": sorted(reasons), "samples": len(rows)}


def tf32_peak_tflops(torch):
    """cuBLAS TF32 GEMM throughput (8192^3, best of 5), the denominator for TF32 kernels."""
    n = 8192
    a = torch.randn(n, n, device="cuda")
    b = torch.randn(n, n, device="cuda")
    old = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = True
    try:
        for _ in range(3):
            torch.matmul(a, b)
        best = 0.0
        for _ in range(5):
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            torch.matmul(a, b)
            e.record()
            e.synchronize()
            best = max(best, 2 * n ** 3 / (s.elapsed_time(e) * 1e-3) / 1e12)
    finally:
        torch.backends.cuda.matmul.allow_tf32 = old
    del a, b
    torch.cuda.empty_cache()
    return best


def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    return json.loads(p.read_text()) if p.exists() else {}


def cpu_baseline(cfg, seq_full, steps=1, warmup=0, threads=None):
    """The oracle (CPU restatement of the reference f32 step) on a bounded sample of the workload: full
    steps (forward, backward, clip, AdamW) of the same model on 1 x S tokens, S = min(64, seq) for models
    above 100M parameters, else min(256, seq). Returns the median tokens/s over `steps` steps."""
    sys.path.insert(0, str(ROOT / "oracle"))
    import oracle as orc
    threads = threads or os.cpu_count() or 1
    orc.set_threads(threads)
    c = orc.config_array(*cfg)
    big = orc.param_breakdown(c)["total"] > 100_000_000
    sample_seq = min(64 if big else 256, seq_full)
    rng = orc.Rng(0)
    model = orc.Model(c, rng=rng)
    ids = np.array([rng.below(cfg[0]) for _ in range(sample_seq + 1)], np.int32)
    opt = orc.AdamW(model, 0.9, 0.95, 1e-8, 0.1)
    times = []
    for k in range(warmup + steps):
        t0 = time.perf_counter()
        orc.train_update(model, opt, ids[:-1], ids[1:], 1, sample_seq, 1.0, 3e-4)
        if k >= warmup:
            times.append(time.perf_counter() - t0)
    dt = statistics.median(times)
    return {"value": sample_seq / dt, "unit": "tokens/s", "cores": threads, "kind": "port",
            "sample": f"{len(times)} full step(s) (fwd+bwd+clip+AdamW) of the same model on 1 x {sample_seq} "
                      f"tokens, median {dt:.2f} s on {threads} threads; the C++ restatement of the reference CPU "
                      f"path (oracle/), not the Rust binary (no cargo on this image); shorter sequences than the "
                      f"workload's {seq_full} make the CPU's attention share smaller, so this favours the CPU"}


LINEAR_SHAPES = [(512, 512), (512, 1408), (1024, 4096), (2048, 5632)]  # configs[1]: (K, N), M = 4096 tokens


def run_kernels(args):
    """configs[1] (isolated Linear fwd+bwd: Y = XW, dX = dY W^T, dW = X^T dY, M = 4096) or configs[2] (causal
    attention B8 H16 hd64 T1024 fwd+bwd) through the kernel-level C ABI, timed with CUDA events."""
    import torch
    import midman_b200 as mm
    mm.load()
    torch.cuda.set_device(0)
    precision = 0 if args.precision == "tf32" else 1
    g = torch.Generator(device="cuda").manual_seed(0)
    results = []
    if args.config == "linear":
        M = 4096
        for K, N in LINEAR_SHAPES:
            x = torch.randn(M, K, device="cuda", generator=g)
            w = torch.randn(K, N, device="cuda", generator=g)
            dy = torch.randn(M, N, device="cuda", generator=g)
            y, dx, dw = torch.empty(M, N, device="cuda"), torch.empty(M, K, device="cuda"), torch.empty(K, N,
                                                                                                        device="cuda")

            def fwd(x=x, w=w, y=y, K=K, N=N):  # Y = X W (bind this shape's tensors)
                mm.gemm(x, w, y, m=M, n=N, k=K, lda=K, ldb=N, ldc=N, a_mn_major=False, b_mn_major=True,
                        precision=precision)

            def bwd_x(dy=dy, w=w, dx=dx, K=K, N=N):  # dX = dY W^T
                mm.gemm(dy, w, dx, m=M, n=K, k=N, lda=N, ldb=N, ldc=K, a_mn_major=False, b_mn_major=False,
                        precision=precision)

            def bwd_w(x=x, dy=dy, dw=dw, K=K, N=N):  # dW = X^T dY
                mm.gemm(x, dy, dw, m=K, n=N, k=M, lda=K, ldb=N, ldc=N, a_mn_major=True, b_mn_major=True,
                        precision=precision)

            def step(parts=(fwd, bwd_x, bwd_w)):
                for p in parts:
                    p()
            flops = 3 * 2 * M * K * N
            results.append(({"K": K, "N": N, "M": M}, flops, step,
                            {"Y=XW": (fwd, flops / 3), "dX=dYW^T": (bwd_x, flops / 3),
                             "dW=X^TdY": (bwd_w, flops / 3)}))
    else:
        # configs[2] (B8 H16 hd64 T1024), or with attention-large the attention of configs[4]'s layers
        B, H, Hkv, hd, T = (8, 16, 16, 64, 1024) if args.config == "attention" else (4, 16, 8, 128, 2048)
        q = torch.randn(B, T, H, hd, device="cuda", generator=g)
        k = torch.randn(B, T, Hkv, hd, device="cuda", generator=g)
        v = torch.randn(B, T, Hkv, hd, device="cuda", generator=g)
        do = torch.randn(B, T, H, hd, device="cuda", generator=g)
        o, lse = torch.empty_like(q), torch.empty(B, H, T, device="cuda")
        dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
        kw = dict(batch=B, seq=T, n_heads=H, n_kv_heads=Hkv, head_dim=hd, ldq=H * hd, ldk=Hkv * hd,
                  precision=precision)

        def fwd():
            mm.attention_forward(q, k, v, o, lse, **kw)

        def bwd():
            mm.attention_backward(q, k, v, o, lse, do, dq, dk, dv, **kw)

        def step():
            fwd()
            bwd()
        flops = 6 * 2 * B * H * (T * T // 2) * hd  # six causal T x T x hd products, no recompute
        results.append(({"B": B, "H": H, "Hkv": Hkv, "hd": hd, "T": T}, flops, step,
                        {"forward": (fwd, flops / 3), "backward": (bwd, flops * 2 / 3)}))
    tf32 = tf32_peak_tflops(torch)
    def timed(fn):
        for _ in range(max(3, args.warmup)):
            fn()
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(args.steps):
            fn()
        e.record()
        e.synchronize()
        mm.device_status()
        return s.elapsed_time(e) / args.steps

    out = []
    for shape, flops, step, parts in results:
        ms = timed(step)
        row = {**shape, "ms": ms, "tflops": flops / (ms * 1e-3) / 1e12, "frac_of_cublas_tf32": flops / (ms * 1e-3)
               / 1e12 / tf32}
        if parts:  # TFLOP/s of each part alone
            row["parts"] = {name: round(f / (timed(fn) * 1e-3) / 1e12, 1) for name, (fn, f) in parts.items()}
        out.append(row)
    line = {"metric": "fwd+bwd TFLOP/s" if args.config == "linear" else "attention fwd+bwd TFLOP/s",
            "value": statistics.mean(r["tflops"] for r in out), "unit": "TFLOP/s", "n_gpus": 1, "steps": args.steps,
            "warmup": args.warmup, "higher_is_better": True, "dtype": args.precision, "data": "synthetic N(0,1)",
            "config": {"workload": args.config, "shapes": out}, "tf32_peak_cublas": tf32}
    print(json.dumps(line), flush=True)
    return 0


GEMM_TRAFFIC_BYTES = 547e6  # see the roofline entry below


def gemm_shapes(prof, steps, top=10):
    """The slowest GEMM shapes of the profiled steps: [shape "MxNxK AB", launches/step, ms/step, TFLOP/s]."""
    rows = sorted(prof.items(), key=lambda kv: -kv[1]["ms"])[:top]
    return [[k, v["launches"] // steps, round(v["ms"] / steps, 3), round(v["flops"] / (v["ms"] * 1e-3) / 1e12, 1)]
            for k, v in rows if v["ms"] > 0]


def workload_config(args, cfg, B, T, world):
    """The `config` of both arms' JSON lines (the reference arm times the same workload)."""
    optimizer = args.optimizer if args.optimizer != "auto" else ("sharded" if world > 1 else "replicated")
    return {"workload": args.config, "preset": list(cfg), "batch_per_gpu": B, "global_batch": B * world,
            "seq_len": T, "parallelism": f"dp{world}", "optimizer": optimizer,
            "l2": "no flush: the step's working set (weights, moments, activations) is far above the 126 MB L2"}


def run_reference(args, cfg, B, T, world, rank):
    if rank != 0:
        return 0
    cb = cpu_baseline(cfg, T, steps=max(1, min(args.steps, 3)), warmup=min(args.warmup, 1))
    value = cb["value"]
    line = {"impl": "reference", "metric": "train tokens/s (fwd+bwd+AdamW)", "value": value, "unit": "tokens/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": workload_config(args, cfg, B, T, world),
            "cpu_baseline": cb,
            "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=8)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--config", default="large", choices=sorted(CONFIGS) + ["linear", "attention", "attention-large"])
    ap.add_argument("--precision", default="tf32", choices=["tf32", "3xtf32"])
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--optimizer", default="auto", choices=["auto", "replicated", "sharded"],
                    help="sharded: ZeRO-1, each rank keeps and updates 1/N of the AdamW state; auto: sharded "
                         "for N > 1 (measured 2-3%% faster at N = 2 and 8)")
    args = ap.parse_args()

    if args.config in ("linear", "attention", "attention-large"):
        return run_kernels(args) if args.impl == "ours" else 0
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    cfg, B, T = CONFIGS[args.config]
    if args.impl == "reference":
        return run_reference(args, cfg, B, T, world, rank)

    # NCCL's version banner (printed at NCCL_DEBUG=VERSION) would land on stdout beside the JSON line
    if os.environ.get("NCCL_DEBUG", "").upper() in ("", "VERSION"):
        os.environ["NCCL_DEBUG"] = "WARN"
    import torch
    import midman_b200 as mm
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=torch.device("cuda", local))
    mm.load()

    # global batch from one Batcher over a synthetic shard; rank r takes rows [rB, (r+1)B)
    steps_needed = args.warmup + 2 * args.steps + 1
    n_tokens = (steps_needed * B * world + 1) * T + 1
    batcher = mm.Batcher(vocab=cfg[0], seq=T, batch=B * world, seed=0, synthetic_tokens=n_tokens, token_seed=0)
    batches = []
    for _ in range(steps_needed):
        i, t, _, _ = batcher.next()
        batches.append((i[rank * B * T:(rank + 1) * B * T].copy(), t[rank * B * T:(rank + 1) * B * T].copy()))

    nccl_id = None
    if world > 1:
        obj = [mm.nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        nccl_id = obj[0]
    precision = 0 if args.precision == "tf32" else 1
    hyper = mm.hyper_array(max_lr=3e-4, min_lr=3e-4, warmup=0, total=10**9, weight_decay=0.1, clip_norm=1.0,
                           beta1=0.9, beta2=0.95)
    trainer = mm.Trainer(mm.config_array(*cfg), hyper, seed=0, batch=B, seq=T, precision=precision, world=world,
                         rank=rank, nccl_id=nccl_id)
    if args.optimizer == "auto":
        args.optimizer = "sharded" if world > 1 else "replicated"
    if args.optimizer == "sharded":
        trainer.shard_optimizer(True)
    stream = torch.cuda.ExternalStream(trainer.stream())

    def barrier():
        torch.cuda.synchronize()
        if dist:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(x):
        if not dist:
            return x
        t = torch.tensor([x], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # ---- value: staged batch (ids in HBM), device time of K steps
    trainer.stage(*batches[0])
    for _ in range(args.warmup):
        trainer.step_staged(1)
    launches0 = trainer.describe()["kernel_launches"]
    barrier()
    clock_rows, stop = [], threading.Event()
    sampler = threading.Thread(target=sample_clocks, args=(stop, clock_rows, local), daemon=True)
    sampler.start()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    rec, status = trainer.step_staged(args.steps)
    end.record(stream)
    end.synchronize()
    barrier()
    ms = max_over_ranks(start.elapsed_time(end))
    gpu_launches = trainer.describe()["kernel_launches"] - launches0

    # ---- kernel breakdown: the same K steps again with every GEMM and attention
    # launch bracketed by CUDA events on the library's stream
    trainer.profile(True)
    p_start, p_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    p_start.record(stream)
    trainer.step_staged(args.steps)
    p_end.record(stream)
    p_end.synchronize()
    prof_ms = p_start.elapsed_time(p_end)
    desc = trainer.describe()
    trainer.profile(False)

    # ---- e2e: the training loop of the public API (midman_train_run) over the
    # batcher: per step the host takes the global batch, checks it and builds the
    # embedding index in pinned memory, copies this rank's ids to the device and
    # reads back loss and gradient norm, all inside the timed region
    batcher.seek(0, 1 + args.warmup)
    barrier()
    t0 = time.perf_counter()
    e_start, e_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e_start.record(stream)
    e_rec, e_status, _ = trainer.run(batcher, args.steps)
    e_end.record(stream)
    e_end.synchronize()
    barrier()
    assert e_status == 0 and len(e_rec) == args.steps
    e2e_ms = max_over_ranks(max(e_start.elapsed_time(e_end), (time.perf_counter() - t0) * 1e3))
    stop.set()
    sampler.join(timeout=10)

    tokens = B * T * world * args.steps
    value = tokens / (ms * 1e-3)
    e2e = tokens / (e2e_ms * 1e-3)
    fpt = flops_per_token(cfg, T)

    line = None
    if rank == 0:
        prof = desc.get("profile", {})
        gk = "gemm_tf32" if precision == 0 else "gemm_3xtf32"
        g = prof.get(gk, {"ms": 0.0, "flops": 0.0, "launches": 0})
        tf32 = tf32_peak_tflops(torch)
        peaks = measured_peaks()
        achieved = g["flops"] / (g["ms"] * 1e-3) / 1e12 if g["ms"] else None
        kernel_share = {k: round(v["ms"] / prof_ms, 4) for k, v in prof.items()} if prof_ms else {}
        line = {
            "metric": "train tokens/s (fwd+bwd+AdamW)", "value": value, "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "tf32" if precision == 0 else "3xtf32",
            "data": "synthetic uniform token ids (Rng(0).below(vocab)), seeded init",
            "config": workload_config(args, cfg, B, T, world),
            "loss_first_last": [float(rec[0, 0]), float(rec[-1, 0])],
            "roofline": {"bound": "tensor", "kernel": gk, "achieved": achieved, "peak": tf32, "unit": "TFLOP/s",
                         "frac": (achieved / tf32) if achieved else None,
                         "peak_source": "cuBLAS TF32 GEMM 8192^3 measured in this run (MEASURED_PEAKS.json has "
                                        f"bf16 only: {peaks.get('bf16_tflops')} TF/s burst)",
                         # DRAM read+write bytes per GEMM launch, averaged over one step's 423 GEMM launches
                         # of this command under ncu (one-pass launch list; measured, not computed here)
                         "traffic": GEMM_TRAFFIC_BYTES if args.config == "large" and precision == 0 else None,
                         "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum, large preset step, "
                                           "mean over the step's GEMM launches",
                         "kernel_launches": g["launches"],
                         "step_tflops": fpt * B * T * args.steps / (ms * 1e-3) / 1e12 / world,
                         "step_frac": fpt * B * T * args.steps / (ms * 1e-3) / 1e12 / world / tf32,
                         "time_share": kernel_share,
                         "gemm_shapes": gemm_shapes(desc.get("profile_gemm", {}), args.steps),
                         "measured": f"CUDA events around each launch in a second run of the same {args.steps} "
                                     f"steps ({prof_ms / args.steps:.2f} ms/step with the events)"},
            "e2e": {"value": e2e, "unit": "tokens/s", "h2d_bytes_per_step": int((5 * B * T + 1) * 4),
                    "d2h_bytes_per_step": 20},
            "gpu_launches": gpu_launches,
            "clocks": summarize_clocks(clock_rows),
        }
    trainer.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline(cfg, T, steps=1, warmup=0)
        print(json.dumps(line), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
