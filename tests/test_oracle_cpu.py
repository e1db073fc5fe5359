"""The CPU oracle against independent implementations (CPU only).

* HF transformers Qwen3ForCausalLM in fp32 (the comparator the upstream project
  uses, Model/benchmark.py:128-246) on the same seeded weights: logits within
  3e-2 max-abs, argmax equal wherever the margin > 1e-2.
* Golden fixtures recorded from the upstream CUDA implementation itself
  (tests/golden/make_golden.py): same rules for decode; the Tools operators
  (fp16 RMSNorm, fp16-accumulating SwiGLU) nearly bit for bit.
"""
import os
import sys

import numpy as np
import pytest
import torch

from conftest import GOLDEN

sys.path.insert(0, GOLDEN)
from inputs import DECODE_CASES, LONGCTX_CASES, OPS_CASE, longctx_cache, ops_inputs  # noqa: E402
from oracle import oracle as O  # noqa: E402

MARGIN, LOGIT_ATOL = 1e-2, 3e-2


def _hf_logits(weights, num_layers, tokens):
    from transformers import Qwen3Config, Qwen3ForCausalLM
    from qwen_weights import hf_state_dict

    cfg = Qwen3Config(vocab_size=151936, hidden_size=1024, intermediate_size=3072,
                      num_hidden_layers=num_layers, num_attention_heads=16, num_key_value_heads=8,
                      head_dim=128, rope_theta=1e6, rms_norm_eps=1e-6, tie_word_embeddings=True,
                      max_position_embeddings=2048, attention_bias=False)
    m = Qwen3ForCausalLM(cfg).float().eval()
    m.load_state_dict(hf_state_dict(weights), strict=False)
    with torch.no_grad():
        return m(torch.tensor([tokens])).logits[0]


def _check(ref_logits, got_logits, got_tok, where):
    top2 = torch.topk(ref_logits, 2)
    diff = float((ref_logits - got_logits).abs().max())
    assert diff <= LOGIT_ATOL, f"{where}: logits diff {diff}"
    if float(top2.values[0] - top2.values[1]) > MARGIN:
        assert got_tok == int(top2.indices[0]), where


@pytest.mark.parametrize("layers", [2, 28])
def test_oracle_matches_hf_fp32(layers, weights_2l, weights_28l):
    w = weights_2l if layers == 2 else weights_28l
    toks = DECODE_CASES[0]["prompt"][:6]
    hf = _hf_logits(w, layers, toks)
    orc = O.OracleModel(w, num_layers=layers)
    for i, t in enumerate(toks):
        r = orc.step(t, want_logits=True)
        _check(hf[i], r["logits"], r["token"], f"L={layers} step {i}")


def test_silu_half_matches_fp16_arithmetic():
    xs = np.linspace(-12, 12, 4001, dtype=np.float32)
    L2E = np.float16(1.44269504088896340736)
    for x in xs[::7]:
        xh = np.float16(x)
        t = np.float16(-xh * L2E)
        e = np.float16(np.exp2(np.float32(t)))
        d = np.float16(np.float16(1.0) + e)
        r = np.float16(np.float32(1.0) / np.float32(d))
        want = np.float16(xh * r)
        got = O.lib().oracle_silu_half(float(x))
        assert np.float16(got) == want, x


def _golden(name):
    path = os.path.join(GOLDEN, name)
    if not os.path.exists(path):
        pytest.skip(f"fixture {name} not generated yet (tests/golden/make_golden.py on a GPU)")
    return np.load(path)


def _logits(norm, embed):
    return embed.float() @ torch.as_tensor(norm, dtype=torch.float32)


@pytest.mark.parametrize("case", DECODE_CASES, ids=[c["name"] for c in DECODE_CASES])
def test_oracle_matches_upstream_decode(case, weights_2l, weights_28l):
    g = _golden(f"ref_decode_{case['name']}.npz")
    w = weights_28l if case["num_layers"] == 28 else weights_2l
    assert case["seed"] == (1234 if case["num_layers"] == 28 else 7)
    orc = O.OracleModel(w, num_layers=case["num_layers"])
    emb = w["embed_weight"]
    for i, (t, pos) in enumerate(zip(g["inp"], g["pos"])):
        assert orc.position == pos
        r = orc.step(int(t))
        ref_l = _logits(g["norm"][i], emb)
        got_l = _logits(r["norm_out"], emb)
        _check(ref_l, got_l, r["token"], f"{case['name']} step {i}")
        top2 = torch.topk(ref_l, 2).values
        if float(top2[0] - top2[1]) > MARGIN:
            assert r["token"] == int(g["out"][i])
        ref_h = torch.from_numpy(g["hidden"][i].view(np.float16).astype(np.float32))
        assert float((ref_h - r["hidden"].float()).abs().max()) < 5e-2
        for tag, li in (("first", 0), ("last", case["num_layers"] - 1)):
            for kind, cache in (("k", orc.k_cache), ("v", orc.v_cache)):
                ref_kv = torch.from_numpy(g[f"{kind}_{tag}"][i].view(np.float16).astype(np.float32))
                d = float((ref_kv - cache[li, :, pos].float()).abs().max())
                assert d < 5e-2, f"{kind} cache layer {li} step {i}: {d}"
    if case["gen_steps"]:
        # generate_nosync from the last prompt position, free-running.
        t = int(case["prompt"][-1])
        orc.position = len(case["prompt"]) - 1
        for s, ref_tok in enumerate(g["gen"]):
            r = orc.step(t, want_logits=True)
            top2 = torch.topk(r["logits"], 2).values
            if float(top2[0] - top2[1]) <= MARGIN:
                break
            assert r["token"] == int(ref_tok), f"generate step {s}"
            t = r["token"]


@pytest.mark.parametrize("case", LONGCTX_CASES, ids=[c["name"] for c in LONGCTX_CASES])
def test_oracle_matches_upstream_long_context(case, weights_2l, weights_28l):
    g = _golden(f"ref_longctx_{case['name']}.npz")
    w = weights_28l if case["num_layers"] == 28 else weights_2l
    assert case["seed"] == (1234 if case["num_layers"] == 28 else 7)
    orc = O.OracleModel(w, num_layers=case["num_layers"])
    kc, vc = longctx_cache(case)
    orc.k_cache.copy_(kc)
    orc.v_cache.copy_(vc)
    orc.position = case["start"]
    emb = w["embed_weight"]
    for i, t in enumerate(g["inp"]):
        pos = case["start"] + i
        r = orc.step(int(t))
        ref_l = _logits(g["norm"][i], emb)
        _check(ref_l, _logits(r["norm_out"], emb), r["token"], f"longctx {case['name']} step {i}")
        top2 = torch.topk(ref_l, 2).values
        if float(top2[0] - top2[1]) > MARGIN:
            assert r["token"] == int(g["out"][i]), f"longctx {case['name']} step {i}"
        for tag, li in (("first", 0), ("last", case["num_layers"] - 1)):
            for kind, cache in (("k", orc.k_cache), ("v", orc.v_cache)):
                ref_kv = torch.from_numpy(g[f"{kind}_{tag}"][i].view(np.float16).astype(np.float32))
                d = float((ref_kv - cache[li, :, pos].float()).abs().max())
                assert d < 5e-2, f"{kind} cache layer {li} step {i}: {d}"


def test_oracle_matches_upstream_ops():
    g = _golden("ref_ops.npz")
    for b in OPS_CASE["batches"]:
        x, w, resid, wg, wu, wd = ops_inputs(b)
        out, rms = O.rmsnorm_forward(x, w, OPS_CASE["eps"])
        ref = torch.from_numpy(g[f"rms_out_{b}"].view(np.float16))
        assert (out == ref).float().mean() > 0.999 and float((out.float() - ref.float()).abs().max()) < 4e-3
        assert np.allclose(rms.numpy(), g[f"rms_rms_{b}"], rtol=1e-6)
        r2 = resid.clone()
        outf, rmsf = O.rmsnorm_forward(x, w, OPS_CASE["eps"], r2)
        assert torch.equal(r2, torch.from_numpy(g[f"rmsf_res_{b}"].view(np.float16)))
        reff = torch.from_numpy(g[f"rmsf_out_{b}"].view(np.float16))
        assert (outf == reff).float().mean() > 0.999
        if b in OPS_CASE["swiglu_batches"]:
            # Same input as upstream's run: its own RMSNorm output.  The
            # sequential fp16 accumulation is restated exactly: bit-equal.
            xs = ref.view(b, 1, 1024)
            y = O.swiglu_forward_down(xs, wg, wu, wd)
            refy = torch.from_numpy(g[f"swd_out_{b}"].view(np.float16)).view_as(y)
            assert torch.equal(y, refy), "fp16-accumulation restatement drifted"
            f, _, _ = O.swiglu_forward(xs, wg, wu)
            reff = torch.from_numpy(g[f"swf_out_{b}"].view(np.float16)).view_as(f)
            assert torch.equal(f, reff)
