"""Parity of the B200 decode kernel with the CPU oracle, through the C ABI.

The oracle (oracle/oracle.c) restates the upstream megakernel step by step
with its fp16 rounding points; tokens and logits are compared under teacher
forcing (both sides are fed the oracle's greedy token) with the rules of
decode_helpers (token bit-exact where the margin > 1e-2, logits within 3e-2).
"""
import os
import sys

import pytest
import torch

from conftest import GOLDEN
from decode_helpers import CAbiDecoder, check_step, last_error, lib, logits_from_norm

sys.path.insert(0, GOLDEN)
from inputs import DECODE_CASES, LONGCTX_CASES, longctx_cache  # noqa: E402
from oracle.oracle import OracleModel  # noqa: E402

pytestmark = pytest.mark.gpu


def _teacher_forced(weights, num_layers, tokens, start=0, kv=None, extra_steps=0):
    """Runs oracle and GPU side by side; returns per-step stats."""
    orc = OracleModel(weights, num_layers=num_layers)
    gpu = CAbiDecoder(weights, num_layers)
    if kv is not None:
        orc.k_cache.copy_(kv[0])
        orc.v_cache.copy_(kv[1])
        gpu.kc.copy_(kv[0].cuda())
        gpu.vc.copy_(kv[1].cuda())
    orc.position = start
    embed_gpu = gpu.w["embed_weight"]
    seq = list(tokens)
    stats = []
    i = 0
    while i < len(seq):
        pos = start + i
        r = orc.step(seq[i], want_logits=True)
        g_tok = gpu.step(seq[i], pos)
        g_logits = logits_from_norm(gpu.norm, embed_gpu)
        r_logits = logits_from_norm(r["norm_out"], embed_gpu)
        diff, margin = check_step(r_logits, g_logits, g_tok, f"step {i} pos {pos}")
        # GPU norm_out vs oracle norm_out, and the fp16 hidden.
        nd = float((gpu.norm.cpu() - r["norm_out"]).abs().max())
        hd = float((gpu.hidden.float().cpu() - r["hidden"].float()).abs().max())
        # K/V written at this position, first and last layer.
        for li in (0, num_layers - 1):
            kd = float((gpu.kc[li, :, pos].float().cpu() - orc.k_cache[li, :, pos].float()).abs().max())
            vd = float((gpu.vc[li, :, pos].float().cpu() - orc.v_cache[li, :, pos].float()).abs().max())
            assert kd <= 5e-2 and vd <= 5e-2, f"step {i} layer {li}: KV diff k={kd} v={vd}"
        stats.append(dict(diff=diff, margin=margin, norm=nd, hidden=hd, tok=g_tok, ref=r["token"]))
        if i == len(seq) - 1 and extra_steps > 0:
            seq.append(r["token"])
            extra_steps -= 1
        i += 1
    return stats, gpu, orc


def test_decode_parity_2_layers(weights_2l):
    toks = DECODE_CASES[1]["prompt"]
    stats, _, _ = _teacher_forced(weights_2l, 2, toks, extra_steps=8)
    assert max(s["norm"] for s in stats) < 5e-2


def test_decode_parity_28_layers(weights_28l):
    toks = DECODE_CASES[0]["prompt"]
    stats, _, _ = _teacher_forced(weights_28l, 28, toks, extra_steps=8)
    assert len(stats) == len(toks) + 8


def test_long_context_parity(weights_2l):
    case = LONGCTX_CASES[0]
    kv = longctx_cache(case)
    _teacher_forced(weights_2l, case["num_layers"], case["tokens"], start=case["start"], kv=kv)


@pytest.mark.parametrize("start", [0, 40, 63, 64, 65, 200, 1100, 2040])
def test_split_boundaries(weights_2l, start):
    """Positions around the split-count thresholds of the split-KV attention."""
    g = torch.Generator().manual_seed(start)
    kc = torch.zeros(2, 8, 2048, 128, dtype=torch.float16)
    vc = torch.zeros_like(kc)
    if start:
        kc[:, :, :start] = torch.randn(2, 8, start, 128, generator=g).half()
        vc[:, :, :start] = torch.randn(2, 8, start, 128, generator=g).half()
    toks = torch.randint(0, 151936, (min(3, 2048 - start),), generator=g).tolist()
    _teacher_forced(weights_2l, 2, toks, start=start, kv=(kc, vc))


def test_generate_equals_steps(weights_2l):
    """One multi-step launch == the same steps launched one at a time."""
    a = CAbiDecoder(weights_2l, 2)
    b = CAbiDecoder(weights_2l, 2)
    prompt = DECODE_CASES[1]["prompt"]
    for i, t in enumerate(prompt[:-1]):
        a.step(t, i)
        b.step(t, i)
    pos = len(prompt) - 1
    gen = a.generate(prompt[-1], pos, 70)  # crosses the 64-token split threshold
    ref, t = [], prompt[-1]
    for s in range(70):
        t = b.step(t, pos + s)
        ref.append(t)
    assert gen == ref
    assert torch.equal(a.kc, b.kc) and torch.equal(a.vc, b.vc)
    assert torch.equal(a.norm, b.norm)


def test_generate_vs_oracle_28_layers(weights_28l):
    case = DECODE_CASES[0]
    orc = OracleModel(weights_28l)
    gpu = CAbiDecoder(weights_28l, 28)
    prompt = case["prompt"]
    for i, t in enumerate(prompt[:-1]):
        orc.step(t)
        gpu.step(t, i)
    gen = gpu.generate(prompt[-1], len(prompt) - 1, 16)
    # Free-running comparison up to the first low-margin step.
    t = prompt[-1]
    for s, g_tok in enumerate(gen):
        r = orc.step(t, want_logits=True)
        top2 = torch.topk(r["logits"], 2)
        if float(top2.values[0] - top2.values[1]) <= 1e-2:
            break
        assert g_tok == r["token"], f"generate step {s}: {g_tok} != {r['token']}"
        t = r["token"]


def test_position_out_of_range_is_rejected(weights_2l):
    d = CAbiDecoder(weights_2l, 2)
    with pytest.raises(RuntimeError, match="max_seq_len"):
        d.step(1, 2048)
    with pytest.raises(RuntimeError, match="max_seq_len"):
        d.generate(1, 2040, 9)
    rc, _ = last_error()
    assert rc != 0
    assert d.step(1, 0) >= 0  # library still usable


def test_bad_token_is_rejected(weights_2l):
    d = CAbiDecoder(weights_2l, 2)
    with pytest.raises(RuntimeError, match="token id"):
        d.step(151936, 0)


def test_bounded_wait_times_out_and_context_survives(weights_2l):
    """A device wait on a word nothing writes gives up after its bound and
    reports the timeout code; the context stays usable."""
    stream = torch.cuda.current_stream().cuda_stream
    code = lib().qwen_b200_selftest_wait_timeout(50_000_000, stream)
    assert code == 1  # timeout of a handoff-word wait
    d = CAbiDecoder(weights_2l, 2)
    assert d.step(5, 0) >= 0
    assert lib().qwen_b200_device_status(torch.cuda.current_device(), None) == 0
