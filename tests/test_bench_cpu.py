"""bench.py's bookkeeping on the CPU: the FLOP counts it reports against, the list of the large step's
products that `--config gemm-step` (and its ncu traffic figure) stands for, and the CPU baseline's fields."""
import importlib.util
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent


@pytest.fixture(scope="module")
def bench():
    spec = importlib.util.spec_from_file_location("bench_mod", ROOT / "bench.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_flops_per_token_match_the_published_plan(bench):
    # algorithmic training FLOPs per token: 6 x matmul parameters (incl. the tied head) + causal attention
    assert bench.flops_per_token(bench.CONFIGS["large"][0], 2048) == 6_558_842_880
    assert bench.flops_per_token(bench.CONFIGS["mid"][0], 1024) == 1_535_115_264
    assert bench.flops_per_token(bench.CONFIGS["tiny"][0], 256) == 8_675_328
    # the reference computes the masked half of T x T too
    for name, (cfg, _b, t) in bench.CONFIGS.items():
        assert bench.executed_flops_per_token(cfg, t) > bench.flops_per_token(cfg, t)


def test_the_gemm_step_list_is_the_large_steps_products(bench):
    v, d, l, h, kv_h, ff, _ = bench.CONFIGS["large"][0]
    kv = kv_h * (d // h)
    matmul_params = l * (2 * d * d + 2 * d * kv + 3 * d * ff) + d * v
    tokens = 4 * 2048
    listed = sum(2 * m * n * sum(ks) * per for m, n, ks, _a, _b, per in bench.LARGE_STEP_GEMMS)
    assert listed == 6 * matmul_params * tokens  # forward 2, backward 4 FLOP per parameter and token
    # 18 products per layer (7 forward, 11 backward with the summed dX of q/k/v and of gate/up), plus the head's 3
    assert sum(per for *_x, per in bench.LARGE_STEP_GEMMS) == 18 * l + 3
    assert bench.GEMM_TRAFFIC_BYTES > bench.GEMM_ALGORITHMIC_BYTES


def test_cpu_baseline_of_the_tiny_preset(bench):
    cb = bench.cpu_baseline(bench.CONFIGS["tiny"][0], 2, 64, steps=1)
    assert cb["cores"] == 1 and cb["kind"] == "port" and not cb["extrapolated"]
    assert cb["params"] == 1_315_968 and cb["value"] > 0 and cb["nproc"] >= 1
