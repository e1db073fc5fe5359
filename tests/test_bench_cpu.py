"""The measurement contract of bench.py, checked on CPU: the algorithmic byte
counts behind every roofline figure, the traffic figure read from the
committed ncu summary, and the CPU baselines' record format."""
import importlib.util
import os

import pytest
import torch

from conftest import ROOT


@pytest.fixture(scope="module")
def bench():
    spec = importlib.util.spec_from_file_location("bench_under_test", os.path.join(ROOT, "bench.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_weight_and_kv_bytes(bench):
    # Every fp16 weight once per token (layers + the tied lm_head / embedding):
    # 440,466,432 layer parameters + 1,024 final-norm weights + 155,582,464
    # embedding parameters; K+V of one cached position over 28 layers x 8 heads.
    assert bench.W_BYTES == 1_192_099_840
    assert bench.KV_BYTES_PER_POS == 28 * 8 * 128 * 2 * 2 == 114_688


def test_config2_launch_bytes(bench):
    # One 128-token launch at positions 1920..2047 attends 1921..2048 positions.
    expect = 128 * 1_192_099_840 + 114_688 * sum(range(1921, 2049))
    assert bench.algorithmic_bytes(1920, 128) == expect == 181_721_366_528


def test_profile_traffic_is_per_launch(bench):
    traffic = bench.profile_traffic()
    assert traffic is not None, "profiles/decode_kernel_longctx.txt lacks traffic_bytes_per_token"
    alg = bench.algorithmic_bytes(1920, 128)
    # DRAM traffic of the kernel within a few percent of the bytes it must read.
    assert 0.9 < traffic / alg < 1.05


def test_torch_ops_baseline_record(bench):
    g = torch.Generator().manual_seed(3)
    x = torch.randn(4, 1024, generator=g).half()
    w = torch.ones(1024).half()
    wg = (torch.randn(1024, 3072, generator=g) * 0.02).half()
    wu = (torch.randn(1024, 3072, generator=g) * 0.02).half()
    wd = (torch.randn(3072, 1024, generator=g) * 0.02).half()
    rec = bench.torch_ops_cpu_baseline(x, w, wg, wu, wd, 1e-6, seconds=0.05)
    assert rec["unit"] == "rows/s" and rec["kind"] == "torch-fp32"
    assert rec["value"] > 0 and rec["cores"] >= 1 and rec["torch_threads"] >= 1
    assert "4 rows" in rec["sample"]
