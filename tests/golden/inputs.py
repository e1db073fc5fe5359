"""Seeded inputs of the golden fixtures (shared by make_golden.py and tests).

Only seeds and shapes live here; tensors are regenerated on demand, so the
committed fixtures hold outputs only.
"""
from __future__ import annotations

import torch

VOCAB = 151936


def _tokens(seed: int, n: int) -> list[int]:
    g = torch.Generator().manual_seed(seed)
    return torch.randint(0, VOCAB, (n,), generator=g).tolist()


# Greedy decode: prompt tokens stepped one by one from position 0 through the
# upstream decode op, then generate_nosync(prompt[-1], gen_steps) at
# position len(prompt)-1 (what upstream Decoder.generate does).
DECODE_CASES = [
    dict(name="s1234_l28", seed=1234, num_layers=28, prompt=_tokens(99, 16), gen_steps=8),
    dict(name="s7_l2", seed=7, num_layers=2, prompt=_tokens(5, 8), gen_steps=0),
]

# Long context: a seeded random KV cache holds positions [0, start); the
# tokens are decoded at positions start, start+1, ...
LONGCTX_CASES = [
    dict(name="s7_l2_p1920", seed=7, num_layers=2, start=1920, tokens=_tokens(11, 4), kv_seed=2024),
    # The benchmarked long-context shape at full depth: the first positions of
    # the timed range and its last positions (up to max_seq - 1 = 2047).
    dict(name="s1234_l28_p1920", seed=1234, num_layers=28, start=1920, tokens=_tokens(12, 6),
         kv_seed=2025),
    dict(name="s1234_l28_p2042", seed=1234, num_layers=28, start=2042, tokens=_tokens(13, 6),
         kv_seed=2026),
]

OPS_CASE = dict(eps=1e-6, batches=[1, 8, 64, 256], swiglu_batches=[1, 8], seed=31337)


def longctx_cache(case: dict) -> tuple[torch.Tensor, torch.Tensor]:
    """fp16 [L, 8, 2048, 128] K/V caches: K ~ N(0,1), V ~ N(0,0.5) on
    positions [0, start), zeros elsewhere."""
    g = torch.Generator().manual_seed(case["kv_seed"])
    L, start = case["num_layers"], case["start"]
    kc = torch.zeros(L, 8, 2048, 128, dtype=torch.float16)
    vc = torch.zeros_like(kc)
    kc[:, :, :start] = torch.randn(L, 8, start, 128, generator=g).half()
    vc[:, :, :start] = (0.5 * torch.randn(L, 8, start, 128, generator=g)).half()
    return kc, vc


def ops_inputs(batch: int):
    """x [B,1024] ~ N(0,1); RMSNorm weight ~ N(1,0.1); residual [B,1024] ~ N(0,1);
    Wg, Wu [1024,3072] and Wd [3072,1024] ~ N(0,0.02) in the upstream Tools/swiglu
    layout (transposed vs HF).  All fp16; the weights do not depend on B."""
    g = torch.Generator().manual_seed(OPS_CASE["seed"])
    w = (1.0 + 0.1 * torch.randn(1024, generator=g)).half()
    wg = (0.02 * torch.randn(1024, 3072, generator=g)).half()
    wu = (0.02 * torch.randn(1024, 3072, generator=g)).half()
    wd = (0.02 * torch.randn(3072, 1024, generator=g)).half()
    gb = torch.Generator().manual_seed(OPS_CASE["seed"] + batch)
    x = torch.randn(batch, 1024, generator=gb).half()
    resid = torch.randn(batch, 1024, generator=gb).half()
    return x, w, resid, wg, wu, wd
