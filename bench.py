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
f32 path (oracle/) on one host thread, as the reference runs (its step time at the workload's size extrapolated
in FLOPs from a bounded sample, and labelled so). A one-GPU run of the default workload also measures
BASELINE.json's other configs (tiny, mid, Linear, attention block) under the `configs` key.
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


def executed_flops_per_token(cfg, seq):
    """FLOPs per token the reference's CPU path executes: 6 x (matmul params incl. the head) plus the
    full T x T score and value products (the reference computes the masked half too,
    attention.rs:79-85), forward and backward."""
    v, d, l, h, kv_h, ff, _ = cfg
    kv = kv_h * (d // h)
    matmul = l * (2 * d * d + 2 * d * kv + 3 * d * ff) + d * v
    return 6 * matmul + l * 3 * 2 * 2 * seq * d


def cpu_baseline(cfg, batch, seq, steps=1, threads=1):
    """The oracle (C++ restatement of the reference's f32 training step, AVX register-tile products with
    separate multiply and add like the reference's `--features avx` kernels) on `threads` host threads
    (1 = the reference, which is single-threaded).

    Models up to 10M parameters: full steps (forward, loss, backward, clip, AdamW) of the workload itself.
    Larger models: forward + backward of a sample of 1 x 64 tokens, and clip + AdamW over every parameter,
    timed apart; the step time at the workload's batch x seq is extrapolated linearly in the executed FLOPs
    of forward + backward, plus the measured optimizer time."""
    sys.path.insert(0, str(ROOT / "oracle"))
    import oracle as orc
    nproc = os.cpu_count() or 1
    orc.set_threads(nproc)  # the seeded init may use every core; it is not timed
    c = orc.config_array(*cfg)
    n_params = orc.param_breakdown(c)["total"]
    rng = orc.Rng(0)
    model = orc.Model(c, rng=rng)
    opt = orc.AdamW(model, 0.9, 0.95, 1e-8, 0.1)
    orc.set_threads(threads)
    out = {"unit": "tokens/s", "cores": threads, "nproc": nproc, "kind": "port", "params": n_params}
    if n_params <= 10_000_000:
        n = batch * seq
        ids = np.array([rng.below(cfg[0]) for _ in range(n + 1)], np.int32)
        times = []
        for _ in range(steps + 1):  # the first step warms the caches and the allocator
            t0 = time.perf_counter()
            orc.train_update(model, opt, ids[:-1], ids[1:], batch, seq, 1.0, 3e-4)
            times.append(time.perf_counter() - t0)
        dt = statistics.median(times[1:])
        out.update(value=n / dt, extrapolated=False,
                   sample=f"{steps} full step(s) (fwd+bwd+clip+AdamW) of the workload ({batch} x {seq} tokens) after "
                          f"one warm-up step, median {dt:.3f} s on {threads} of {nproc} host threads; the C++ "
                          f"restatement of the reference CPU path (oracle/), not the Rust binary (no cargo here)")
        return out
    s_tok = min(64, seq)
    ids = np.array([rng.below(cfg[0]) for _ in range(s_tok + 1)], np.int32)
    g = np.zeros(n_params, np.float32)
    fb = []
    for k in range(steps + 1):  # the first pass warms the caches and maps the buffers
        t0 = time.perf_counter()
        model.loss(ids[:-1], ids[1:], 1, s_tok, grads=True, out=g)
        if k:
            fb.append(time.perf_counter() - t0)
    t0 = time.perf_counter()
    orc.clip_global_norm(g, 1.0)
    opt.step(g, 3e-4)
    t_opt = time.perf_counter() - t0
    t_fb = statistics.median(fb)
    scale = batch * seq * executed_flops_per_token(cfg, seq) / (s_tok * executed_flops_per_token(cfg, s_tok))
    step = t_fb * scale + t_opt
    out.update(value=batch * seq / step, extrapolated=True, step_s=step, sample_fwd_bwd_s=t_fb, optimizer_s=t_opt,
               sample=f"EXTRAPOLATED: forward+backward of 1 x {s_tok} tokens of the same model ({n_params:,} "
                      f"parameters) took {t_fb:.2f} s (median of {steps} after one warm-up pass) and clip+AdamW "
                      f"over all parameters {t_opt:.2f} s, on {threads} of {nproc} host threads; the "
                      f"forward+backward time is scaled by executed FLOPs ({scale:.0f}x, full T x T attention as "
                      f"the reference computes it) to {batch} x {seq} tokens and the optimizer time added: "
                      f"{step:.0f} s per step. The C++ restatement of the reference CPU path (oracle/), not the "
                      f"Rust binary (no cargo here)")
    return out


LINEAR_SHAPES = [(512, 512), (512, 1408), (1024, 4096), (2048, 5632)]  # configs[1]: (K, N), M = 4096 tokens


def _timed(torch, mm, fn, steps, warmup):
    """Mean ms of fn() over `steps` calls after `warmup` (>= 3) untimed ones: CUDA events on the current stream,
    on which every launch of fn is queued."""
    for _ in range(max(3, warmup)):
        fn()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(steps):
        fn()
    e.record()
    e.synchronize()
    mm.device_status()
    return s.elapsed_time(e) / steps


def linear_config(torch, mm, precision, steps, warmup, tf32):
    """the isolated Linear op fwd+bwd (Y = XW, dX = dY W^T, dW = X^T dY, M = 4096 tokens) per
    (K, N), through the kernel-level C ABI (mm_gpu_gemm)."""
    g = torch.Generator(device="cuda").manual_seed(0)
    M = 4096
    out = []
    for K, N in LINEAR_SHAPES:
        x = torch.randn(M, K, device="cuda", generator=g)
        w = torch.randn(K, N, device="cuda", generator=g)
        dy = torch.randn(M, N, device="cuda", generator=g)
        y, dx, dw = (torch.empty(M, N, device="cuda"), torch.empty(M, K, device="cuda"),
                     torch.empty(K, N, device="cuda"))

        def fwd():  # Y = X W
            mm.gemm(x, w, y, m=M, n=N, k=K, lda=K, ldb=N, ldc=N, a_mn_major=False, b_mn_major=True,
                    precision=precision)

        def bwd_x():  # dX = dY W^T
            mm.gemm(dy, w, dx, m=M, n=K, k=N, lda=N, ldb=N, ldc=K, a_mn_major=False, b_mn_major=False,
                    precision=precision)

        def bwd_w():  # dW = X^T dY
            mm.gemm(x, dy, dw, m=K, n=N, k=M, lda=K, ldb=N, ldc=N, a_mn_major=True, b_mn_major=True,
                    precision=precision)

        def step():
            fwd()
            bwd_x()
            bwd_w()
        flops = 3 * 2 * M * K * N
        ms = _timed(torch, mm, step, steps, warmup)
        parts = {name: round(flops / 3 / (_timed(torch, mm, fn, steps, warmup) * 1e-3) / 1e12, 1)
                 for name, fn in (("Y=XW", fwd), ("dX=dYW^T", bwd_x), ("dW=X^TdY", bwd_w))}
        tfl = flops / (ms * 1e-3) / 1e12
        out.append({"M": M, "K": K, "N": N, "ms": round(ms, 4), "tflops": round(tfl, 1),
                    "frac_of_cublas_tf32": round(tfl / tf32, 3), "parts": parts})
        del x, w, dy, y, dx, dw
    return {"metric": "Linear fwd+bwd TFLOP/s", "value": statistics.mean(r["tflops"] for r in out),
            "unit": "TFLOP/s", "shapes": out}


def attention_block_config(torch, mm, precision, steps, warmup, tf32, large=False):
    """causal attention B 8, H 16, hd 64, T 1024 (RoPE theta 10000 on Q and K, scale 1/8) forward
    and backward, with the RMSNorm (eps 1e-5) and the SwiGLU MLP (d_model 1024, hidden 2816) forward and
    backward on the same 8,192 tokens, each part through the kernel-level C ABI. With large=True the
    attention alone at configs[4]'s layer shape (B 4, H 16 / 8 key-value heads, hd 128, T 2048)."""
    import oracle as orc
    B, H, Hkv, hd, T = (4, 16, 8, 128, 2048) if large else (8, 16, 16, 64, 1024)
    D, KV, F, N = H * hd, Hkv * hd, 2816, B * T
    g = torch.Generator(device="cuda").manual_seed(0)
    q = torch.randn(N, D, device="cuda", generator=g)
    k = torch.randn(N, KV, device="cuda", generator=g)
    v = torch.randn(N, KV, device="cuda", generator=g)
    do = torch.randn(N, D, device="cuda", generator=g)
    o, lse = torch.empty_like(q), torch.empty(B, H, T, device="cuda")
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    cos_np, sin_np = orc.rope_table(hd, T, 10000.0)
    cos_t, sin_t = torch.from_numpy(cos_np).cuda(), torch.from_numpy(sin_np).cuda()
    kw = dict(batch=B, seq=T, n_heads=H, n_kv_heads=Hkv, head_dim=hd, ldq=D, ldk=KV, precision=precision)

    def attention():
        mm.rope(q, cos_t, sin_t, rows=N, seq=T, heads=H, head_dim=hd, ld=D)
        mm.rope(k, cos_t, sin_t, rows=N, seq=T, heads=Hkv, head_dim=hd, ld=KV)
        mm.attention_forward(q, k, v, o, lse, **kw)
        mm.attention_backward(q, k, v, o, lse, do, dq, dk, dv, **kw)
        mm.rope(dq, cos_t, sin_t, rows=N, seq=T, heads=H, head_dim=hd, ld=D, backward=True)
        mm.rope(dk, cos_t, sin_t, rows=N, seq=T, heads=Hkv, head_dim=hd, ld=KV, backward=True)
        # q and k rotate back so that every timed pass sees the same inputs
        mm.rope(q, cos_t, sin_t, rows=N, seq=T, heads=H, head_dim=hd, ld=D, backward=True)
        mm.rope(k, cos_t, sin_t, rows=N, seq=T, heads=Hkv, head_dim=hd, ld=KV, backward=True)

    attn_flops = 6 * 2 * B * H * (T * T // 2) * hd  # six causal T x T x hd products, no recompute
    res = {"shape": {"B": B, "H": H, "Hkv": Hkv, "hd": hd, "T": T}}
    ms_attn = _timed(torch, mm, attention, steps, warmup)
    res["attention"] = {"ms": round(ms_attn, 4), "tflops": round(attn_flops / (ms_attn * 1e-3) / 1e12, 1),
                        "frac_of_cublas_tf32": round(attn_flops / (ms_attn * 1e-3) / 1e12 / tf32, 3),
                        "includes": "RoPE of q and k forward, backward and undo (6 HBM passes)"}
    if large:
        return res
    x = torch.randn(N, D, device="cuda", generator=g)
    wn = 1 + 0.1 * torch.randn(D, device="cuda", generator=g)
    wg = 0.03 * torch.randn(D, F, device="cuda", generator=g)
    wu = 0.03 * torch.randn(D, F, device="cuda", generator=g)
    wd = 0.02 * torch.randn(F, D, device="cuda", generator=g)
    dout = torch.randn(N, D, device="cuda", generator=g)
    y, rstd = torch.empty(N, D, device="cuda"), torch.empty(N, device="cuda")
    gate, up, act = (torch.empty(N, F, device="cuda") for _ in range(3))
    out, dact, dy, dx = (torch.empty(N, D, device="cuda"), torch.empty(N, F, device="cuda"),
                         torch.empty(N, D, device="cuda"), torch.empty(N, D, device="cuda"))
    dwn, dwg, dwu, dwd = (torch.empty(D, device="cuda"), torch.empty(D, F, device="cuda"),
                          torch.empty(D, F, device="cuda"), torch.empty(F, D, device="cuda"))

    def norm_fwd():
        mm.rmsnorm_forward(x, wn, y, rstd, rows=N, dim=D, eps=1e-5)

    def mlp():
        mm.gemm(y, wg, gate, m=N, n=F, k=D, lda=D, ldb=F, ldc=F, a_mn_major=False, b_mn_major=True,
                precision=precision)
        mm.gemm(y, wu, up, m=N, n=F, k=D, lda=D, ldb=F, ldc=F, a_mn_major=False, b_mn_major=True,
                precision=precision)
        mm.swiglu_forward(gate, up, act, n=N * F)
        mm.gemm(act, wd, out, m=N, n=D, k=F, lda=F, ldb=D, ldc=D, a_mn_major=False, b_mn_major=True,
                precision=precision)
        # backward: dact = dout Wd^T, dWd = act^T dout, SwiGLU in place, dy = dG Wg^T + dU Wu^T, dW = y^T dG|dU
        mm.gemm(dout, wd, dact, m=N, n=F, k=D, lda=D, ldb=D, ldc=F, a_mn_major=False, b_mn_major=False,
                precision=precision)
        mm.gemm(act, dout, dwd, m=F, n=D, k=N, lda=F, ldb=D, ldc=D, a_mn_major=True, b_mn_major=True,
                precision=precision)
        mm.swiglu_backward(gate, up, dact, n=N * F)
        if precision == 0:
            mm.gemm_sum([(gate, F, wg, F, F), (up, F, wu, F, F)], dy, m=N, n=D, ldc=D, a_mn_major=False,
                        b_mn_major=False)
        else:
            mm.gemm(gate, wg, dy, m=N, n=D, k=F, lda=F, ldb=F, ldc=D, a_mn_major=False, b_mn_major=False,
                    precision=precision)
            mm.gemm(up, wu, dy, m=N, n=D, k=F, lda=F, ldb=F, ldc=D, a_mn_major=False, b_mn_major=False,
                    r=dy, ldr=D, precision=precision)
        mm.gemm(y, gate, dwg, m=D, n=F, k=N, lda=D, ldb=F, ldc=F, a_mn_major=True, b_mn_major=True,
                precision=precision)
        mm.gemm(y, up, dwu, m=D, n=F, k=N, lda=D, ldb=F, ldc=F, a_mn_major=True, b_mn_major=True,
                precision=precision)

    def norm_bwd():
        mm.rmsnorm_backward(x, wn, rstd, dy, dx, dwn, rows=N, dim=D)

    norm_fwd()
    ms_nf = _timed(torch, mm, norm_fwd, steps, warmup)
    ms_mlp = _timed(torch, mm, mlp, steps, warmup)
    ms_nb = _timed(torch, mm, norm_bwd, steps, warmup)
    mlp_flops = 9 * 2 * N * D * F  # three products forward, six backward
    res["swiglu_mlp"] = {"ms": round(ms_mlp, 4), "tflops": round(mlp_flops / (ms_mlp * 1e-3) / 1e12, 1),
                         "frac_of_cublas_tf32": round(mlp_flops / (ms_mlp * 1e-3) / 1e12 / tf32, 3),
                         "includes": "SwiGLU forward and backward (HBM) between the nine products"}
    res["rmsnorm"] = {"forward_ms": round(ms_nf, 4), "backward_ms": round(ms_nb, 4),
                      "forward_gbs": round(2 * N * D * 4 / (ms_nf * 1e-3) / 1e9, 1),
                      "backward_gbs": round(3 * N * D * 4 / (ms_nb * 1e-3) / 1e9, 1),
                      "bytes": "forward reads x, writes y (8 B/element); backward reads x and dy, writes dx "
                               "(12 B/element)"}
    res["block_ms"] = round(ms_attn + ms_nf + ms_mlp + ms_nb, 4)
    return res


def run_kernels(args):
    """`--config linear|attention|attention-large`: one JSON line for configs[1] or configs[2] alone."""
    import torch
    import midman_b200 as mm
    mm.load()
    torch.cuda.set_device(0)
    sys.path.insert(0, str(ROOT / "oracle"))
    precision = 0 if args.precision == "tf32" else 1
    tf32 = tf32_peak_tflops(torch)
    if args.config == "linear":
        res = linear_config(torch, mm, precision, args.steps, args.warmup, tf32)
        line = {"metric": res["metric"], "value": res["value"], "unit": "TFLOP/s",
                "config": {"workload": "linear", "shapes": res["shapes"]}}
    elif args.config == "gemm-step":
        res = gemm_step_config(torch, mm, args.steps, args.warmup, tf32, precision)
        line = {"metric": res["metric"], "value": res["value"], "unit": "TFLOP/s",
                "config": {"workload": "gemm-step", **{k: v for k, v in res.items() if k not in ("metric", "value")}}}
    else:
        res = attention_block_config(torch, mm, precision, args.steps, args.warmup, tf32,
                                     large=args.config == "attention-large")
        line = {"metric": "attention fwd+bwd TFLOP/s", "value": res["attention"]["tflops"], "unit": "TFLOP/s",
                "config": {"workload": args.config, **res}}
    line.update({"n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
                 "dtype": args.precision, "data": "synthetic N(0,1)", "tf32_peak_cublas": tf32})
    print(json.dumps(line), flush=True)
    return 0


# The TF32 products of one large-preset step (configs[4], 4 x 2048 tokens): (M, N, K-list, A MN-major,
# B MN-major, launches per step). Summed K lists are one launch (dX of the projections that share an input).
LARGE_STEP_GEMMS = [
    (8192, 2048, [2048], False, True, 40),         # q, o projections
    (8192, 1024, [2048], False, True, 40),         # k, v projections
    (8192, 5632, [2048], False, True, 40),         # gate, up
    (8192, 2048, [5632], False, True, 20),         # down
    (8192, 32000, [2048], False, False, 1),        # logits = x E^T
    (8192, 2048, [32000], False, True, 1),         # dX of the head
    (32000, 2048, [8192], True, True, 1),          # dE of the head
    (5632, 2048, [8192], True, True, 20),          # dW down
    (8192, 5632, [2048], False, False, 20),        # d act = dx Wd^T
    (2048, 5632, [8192], True, True, 40),          # dW gate, up
    (8192, 2048, [5632, 5632], False, False, 20),  # dX = dG Wg^T + dU Wu^T
    (2048, 2048, [8192], True, True, 40),          # dW o, q
    (8192, 2048, [2048], False, False, 20),        # d o = dh Wo^T
    (2048, 1024, [8192], True, True, 40),          # dW k, v
    (8192, 2048, [2048, 1024, 1024], False, False, 20),  # dX = dQ Wq^T + dK Wk^T + dV Wv^T
]


def gemm_step_config(torch, mm, steps, warmup, tf32, precision=0):
    """Each distinct product of the large step once, standalone (operands < 2 GB on the device): TFLOP/s per
    shape and the step's mix. Small enough for an ncu capture of the products' DRAM traffic. In 3xTF32
    (precision 1) a summed product runs as one launch per term, each after the first adding into C (the
    kernel-level ABI's sum is TF32 only; the trainer sums the terms in one launch)."""
    g = torch.Generator(device="cuda").manual_seed(0)
    out, total_ms, total_flops = [], 0.0, 0.0
    for M, N, ks, a_mn, b_mn, per_step in LARGE_STEP_GEMMS:
        terms = []
        for K in ks:
            a = torch.randn(*((K, M) if a_mn else (M, K)), device="cuda", generator=g)
            b = torch.randn(*((K, N) if b_mn else (N, K)), device="cuda", generator=g)
            terms.append((a, a.shape[1], b, b.shape[1], K))
        c = torch.empty(M, N, device="cuda")
        if len(terms) == 1 or precision:
            def fn():
                for g, (a, lda, b, ldb, K) in enumerate(terms):
                    mm.gemm(a, b, c, m=M, n=N, k=K, lda=lda, ldb=ldb, ldc=N, a_mn_major=a_mn, b_mn_major=b_mn,
                            r=c if g else None, ldr=N if g else 0, precision=precision)
        else:
            def fn():
                mm.gemm_sum(terms, c, m=M, n=N, ldc=N, a_mn_major=a_mn, b_mn_major=b_mn)
        ms = _timed(torch, mm, fn, steps, warmup)
        flops = 2.0 * M * N * sum(ks)
        out.append({"shape": f"{M}x{N}x{'+'.join(map(str, ks))} {'M' if a_mn else 'K'}{'M' if b_mn else 'K'}",
                    "per_step": per_step, "ms": round(ms, 4), "tflops": round(flops / (ms * 1e-3) / 1e12, 1),
                    "algorithmic_bytes": int(4 * (M * sum(ks) + N * sum(ks) + M * N))})
        total_ms += per_step * ms
        total_flops += per_step * flops
        del terms, c
    return {"metric": f"{'3xTF32' if precision else 'TF32'} GEMM TFLOP/s over the large step's products",
            "value": total_flops / (total_ms * 1e-3) / 1e12,
            "unit": "TFLOP/s", "frac_of_cublas_tf32": total_flops / (total_ms * 1e-3) / 1e12 / tf32, "shapes": out,
            "step_gemm_ms_serialized": total_ms}


def trainer_tokens_per_s(torch, mm, cfg, B, T, precision, steps, warmup):
    """tokens/s of K staged training steps of a config on one GPU (CUDA events on the library's stream)."""
    batcher = mm.Batcher(vocab=cfg[0], seq=T, batch=B, seed=0, synthetic_tokens=(B + 1) * T * 2 + 1, token_seed=0)
    i, t, _, _ = batcher.next()
    batcher.close()
    hyper = mm.hyper_array(max_lr=3e-4, min_lr=3e-4, warmup=0, total=10**9, weight_decay=0.1, clip_norm=1.0,
                           beta1=0.9, beta2=0.95)
    tr = mm.Trainer(mm.config_array(*cfg), hyper, seed=0, batch=B, seq=T, precision=precision)
    try:
        stream = torch.cuda.ExternalStream(tr.stream())
        tr.stage(i, t)
        tr.step_staged(max(3, warmup))
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record(stream)
        rec, status = tr.step_staged(steps)
        e.record(stream)
        e.synchronize()
        ms = s.elapsed_time(e) / steps
    finally:
        tr.close()
    return {"value": B * T / (ms * 1e-3), "unit": "tokens/s", "ms_per_step": ms, "steps": steps,
            "batch": B, "seq_len": T, "loss_first_last": [float(rec[0, 0]), float(rec[-1, 0])]}


# DRAM read + write bytes per TF32 GEMM launch of the large step, the step's mix of products (weights: launches
# per step): measured by ncu (dram__bytes_read.sum + dram__bytes_write.sum) on each product of LARGE_STEP_GEMMS
# run alone (`--config gemm-step`), summarized in profiles/gemm_tf32_large_step_shapes.md. Algorithmic (each
# operand read once, C written once): 233.9e6 bytes per launch.
GEMM_TRAFFIC_BYTES = 334.4e6
GEMM_ALGORITHMIC_BYTES = 233.9e6


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
    cb = cpu_baseline(cfg, B, T, steps=max(1, min(args.steps, 2)))
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
    ap.add_argument("--config", default="large",
                    choices=sorted(CONFIGS) + ["linear", "attention", "attention-large", "gemm-step"])
    ap.add_argument("--precision", default="tf32", choices=["tf32", "3xtf32"])
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-configs", action="store_true",
                    help="skip the other BASELINE configs (tiny, mid, Linear, attention block) that a one-GPU run "
                         "of the default workload adds under the `configs` key")
    ap.add_argument("--optimizer", default="auto", choices=["auto", "replicated", "sharded"],
                    help="sharded: ZeRO-1, each rank keeps and updates 1/N of the AdamW state; auto: sharded "
                         "for N > 1 (measured 2-3%% faster at N = 2 and 8)")
    args = ap.parse_args()

    if args.config in ("linear", "attention", "attention-large", "gemm-step"):
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
                         "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum of each product of the "
                                           "large step run alone (--config gemm-step), weighted by launches per "
                                           "step (profiles/gemm_tf32_large_step_shapes.md)",
                         "algorithmic_bytes": GEMM_ALGORITHMIC_BYTES if args.config == "large" and precision == 0
                         else None,
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
        if world == 1 and not args.no_configs and args.config == "large":
            line["configs"] = other_configs(args, torch, mm, precision, with_cpu=not args.no_cpu_baseline)
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline(cfg, B, T, steps=1)
        print(json.dumps(line), flush=True)
    return 0


PUBLISHED_TINY = ("reference tiny preset, batch 8 x seq 256, --features avx, one CPU thread: ~2,000-2,300 tokens/s "
                  "(README.md:109), 1,282 tokens/s on a 2.1 GHz Xeon (docs/midman-training.md:100)")


def other_configs(args, torch, mm, precision, with_cpu=True):
    """BASELINE.json's other configs on this GPU: configs[0] tiny and configs[3] mid (training steps,
    tokens/s, with the CPU baseline of the same workload), configs[1] (Linear fwd+bwd) and configs[2]
    (attention block fwd+bwd) through the kernel-level C ABI."""
    sys.path.insert(0, str(ROOT / "oracle"))
    tf32 = tf32_peak_tflops(torch)
    out = {}
    for name, idx, steps in (("tiny", 0, 20), ("mid", 3, 10)):
        cfg, B, T = CONFIGS[name]
        r = trainer_tokens_per_s(torch, mm, cfg, B, T, precision, steps, max(3, args.warmup))
        fpt = flops_per_token(cfg, T)
        r.update(config=f"configs[{idx}]", preset=list(cfg), step_tflops=r["value"] * fpt / 1e12,
                 step_frac_of_cublas_tf32=r["value"] * fpt / 1e12 / tf32)
        if with_cpu:
            r["cpu_baseline"] = cpu_baseline(cfg, B, T, steps=2 if name == "tiny" else 1)
        if name == "tiny":
            r["published_reference"] = PUBLISHED_TINY
        out[name] = r
    if precision == 0:
        # the same large-preset step in the exact mode (3xTF32 products, FP32 attention), a few steps
        cfg, B, T = CONFIGS["large"]
        r = trainer_tokens_per_s(torch, mm, cfg, B, T, 1, 4, 3)
        fpt = flops_per_token(cfg, T)
        r.update(config="configs[4] in 3xTF32", step_tflops=r["value"] * fpt / 1e12,
                 step_frac_of_cublas_tf32=r["value"] * fpt / 1e12 / tf32)
        out["large_3xtf32"] = r
    out["linear"] = {"config": "configs[1]", **linear_config(torch, mm, precision, 10, 3, tf32)}
    out["attention_block"] = {"config": "configs[2]", **attention_block_config(torch, mm, precision, 10, 3, tf32)}
    out["tf32_peak_cublas"] = tf32
    torch.cuda.empty_cache()
    return out


if __name__ == "__main__":
    sys.exit(main())
