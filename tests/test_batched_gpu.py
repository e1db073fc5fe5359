"""Parity of the batched decode path (qwen0.6b_b200/batched.py, C ABI
include/qwen_b200_batched.h) with the batch-1 decode kernel and the CPU oracle.

Every sequence of a batched run is replayed alone through the batch-1 C ABI
(whose parity with the oracle and with the upstream megakernel's goldens is
tested elsewhere) with the same tokens (teacher forcing), and step by step:
* greedy tokens equal wherever the batch-1 logits' top-1/top-2 margin > 1e-2;
* logits (final-normed hidden @ tied lm_head^T, fp32) within 3e-2 max-abs;
* the K/V rows written at every position within 5e-2.
One sequence is also checked directly against the CPU oracle.
"""
import pytest
import torch

from decode_helpers import LOGIT_ATOL, MARGIN, CAbiDecoder, logits_from_norm
from oracle.oracle import OracleModel

pytestmark = pytest.mark.gpu


def _batched(weights, n_seqs, num_layers, max_rows=None):
    from batched import BatchedDecoder
    return BatchedDecoder(weights, num_seqs=n_seqs, max_rows=max_rows or n_seqs, num_layers=num_layers)


def _prompts(lengths, seed):
    g = torch.Generator().manual_seed(seed)
    return [torch.randint(0, 151936, (n,), generator=g).tolist() for n in lengths]


def _run_batched(bd, prompts, steps):
    """Prefill, then `steps` greedy steps; returns tokens [steps][n] and
    norm_out [steps][n, 1024] (fp32, CPU)."""
    n = len(prompts)
    dev = bd.dev
    bd.prefill(prompts)
    ids = torch.arange(n, dtype=torch.int32, device=dev)
    pos = torch.tensor([len(p) - 1 for p in prompts], dtype=torch.int32, device=dev)
    tok = torch.tensor([p[-1] for p in prompts], dtype=torch.int32, device=dev)
    start_max = max(len(p) - 1 for p in prompts)
    toks, norms = [], []
    for s in range(steps):
        norm = torch.empty(n, 1024, dtype=torch.float32, device=dev)
        out = torch.empty(n, dtype=torch.int32, device=dev)
        bd.step(ids, pos, tok, start_max + s, norm_out=norm, out=out)
        toks.append(out.cpu().tolist())
        norms.append(norm.cpu())
        tok = out
        pos = pos + 1
    assert bd.status() == 0
    return toks, norms


def _check_against_batch1(weights, num_layers, prompts, toks, norms, bd, kv_rows=True):
    for i, prompt in enumerate(prompts):
        ref = CAbiDecoder(weights, num_layers)
        emb = ref.w["embed_weight"]
        for p, t in enumerate(prompt[:-1]):
            ref.step(t, p)
        t = prompt[-1]
        for s in range(len(toks)):
            pos = len(prompt) - 1 + s
            r_tok = ref.step(t, pos)
            r_logits = logits_from_norm(ref.norm, emb)
            b_logits = logits_from_norm(norms[s][i], emb)
            diff = float((r_logits - b_logits).abs().max())
            assert diff <= LOGIT_ATOL, f"seq {i} step {s}: logits differ by {diff}"
            top2 = torch.topk(r_logits, 2).values
            if float(top2[0] - top2[1]) > MARGIN:
                assert toks[s][i] == r_tok, f"seq {i} step {s}: token {toks[s][i]} != {r_tok}"
            t = toks[s][i]  # teacher forcing on the batched trajectory
        if kv_rows:
            last = len(prompt) - 1 + len(toks)
            for l in (0, num_layers - 1):
                kd = float((bd.k_pool[i, l, :, :last].float() - ref.kc[l, :, :last].float()).abs().max())
                vd = float((bd.v_pool[i, l, :, :last].float() - ref.vc[l, :, :last].float()).abs().max())
                assert kd <= 5e-2 and vd <= 5e-2, f"seq {i} layer {l}: KV differ k={kd} v={vd}"


def test_batched_matches_batch1_two_layers(weights_2l):
    # Prompt lengths around the 128-token attention split and the 8-row norm blocks.
    prompts = _prompts([3, 17, 64, 129, 200], seed=21)
    bd = _batched(weights_2l, len(prompts), 2)
    toks, norms = _run_batched(bd, prompts, 4)
    _check_against_batch1(weights_2l, 2, prompts, toks, norms, bd)


def test_batched_matches_oracle(weights_2l):
    prompts = _prompts([140, 9], seed=5)
    bd = _batched(weights_2l, 2, 2)
    toks, norms = _run_batched(bd, prompts, 3)
    orc = OracleModel(weights_2l, num_layers=2)
    for t in prompts[0][:-1]:
        orc.step(t)
    t = prompts[0][-1]
    emb = weights_2l["embed_weight"]
    for s in range(3):
        r = orc.step(t, want_logits=True)
        b_logits = logits_from_norm(norms[s][0], emb.cuda())
        diff = float((r["logits"] - b_logits).abs().max())
        assert diff <= LOGIT_ATOL, f"step {s}: {diff}"
        top2 = torch.topk(r["logits"], 2).values
        if float(top2[0] - top2[1]) > MARGIN:
            assert toks[s][0] == r["token"]
        t = toks[s][0]


def test_batched_matches_batch1_28_layers(weights_28l):
    prompts = _prompts([5, 40, 150], seed=8)
    bd = _batched(weights_28l, len(prompts), 28)
    toks, norms = _run_batched(bd, prompts, 3)
    _check_against_batch1(weights_28l, 28, prompts, toks, norms, bd, kv_rows=False)


def test_batched_more_than_one_row_tile(weights_2l):
    """130 rows: the GEMMs' second 128-row tile and ragged norm blocks."""
    n = 130
    g = torch.Generator().manual_seed(3)
    lengths = torch.randint(2, 6, (n,), generator=g).tolist()
    prompts = _prompts(lengths, seed=4)
    bd = _batched(weights_2l, n, 2)
    toks, norms = _run_batched(bd, prompts, 2)
    pick = [0, 1, 127, 128, 129]
    sub_prompts = [prompts[i] for i in pick]
    sub_toks = [[t[i] for i in pick] for t in toks]
    sub_norms = [nm[pick] for nm in norms]

    class _View:  # KV of the picked sequences, in pick order
        k_pool = bd.k_pool[pick]
        v_pool = bd.v_pool[pick]

    _check_against_batch1(weights_2l, 2, sub_prompts, sub_toks, sub_norms, _View)


def test_batched_step_rejects_bad_arguments(weights_2l):
    bd = _batched(weights_2l, 2, 2)
    z = torch.zeros(3, dtype=torch.int32, device=bd.dev)
    with pytest.raises(RuntimeError, match="rows=3 out of range"):
        bd.step(z, z, z, 0)
    z2 = torch.zeros(2, dtype=torch.int32, device=bd.dev)
    with pytest.raises(RuntimeError, match="max_position"):
        bd.step(z2, z2, z2, 2048)
    # A sequence id outside the pool is caught on the device, reported, and
    # touches no cache memory.
    bad = torch.tensor([0, 7], dtype=torch.int32, device=bd.dev)
    bd.step(bad, z2, z2, 0)
    assert bd.status() == 3


def test_parallel_prefill_matches_sequential(weights_2l):
    """Prompt K/V written by multi-position steps (several rows of one
    sequence per step, chunked by max_rows) equals the one-position-per-step
    prefill within the KV tolerance, and the next step agrees."""
    from batched import BatchedDecoder
    prompts = _prompts([3, 100, 200], seed=12)
    seq = BatchedDecoder(weights_2l, num_seqs=3, max_rows=3, num_layers=2)
    par = BatchedDecoder(weights_2l, num_seqs=3, max_rows=64, num_layers=2)
    seq.prefill(prompts)
    par.prefill_parallel(prompts)
    for i, p in enumerate(prompts):
        n = len(p) - 1
        for pool in ("k_pool", "v_pool"):
            a, b = getattr(seq, pool)[i, :, :, :n].float(), getattr(par, pool)[i, :, :, :n].float()
            assert float((a - b).abs().max()) <= 5e-2, f"seq {i} {pool}"
    dev = seq.dev
    ids = torch.arange(3, dtype=torch.int32, device=dev)
    pos = torch.tensor([len(p) - 1 for p in prompts], dtype=torch.int32, device=dev)
    tok = torch.tensor([p[-1] for p in prompts], dtype=torch.int32, device=dev)
    emb = seq.embed
    outs, norms = [], []
    for bd in (seq, par):
        norm = torch.empty(3, 1024, dtype=torch.float32, device=dev)
        outs.append(bd.step(ids, pos, tok, int(pos.max()), norm_out=norm,
                            out=torch.empty(3, dtype=torch.int32, device=dev)).cpu().tolist())
        norms.append(norm)
    for i in range(3):
        la, lb = logits_from_norm(norms[0][i], emb), logits_from_norm(norms[1][i], emb)
        assert float((la - lb).abs().max()) <= LOGIT_ATOL
        top2 = torch.topk(la, 2).values
        if float(top2[0] - top2[1]) > MARGIN:
            assert outs[0][i] == outs[1][i]


def test_decoder_parallel_prefill(weights_2l):
    """Decoder.prefill (batched path over the Decoder's own cache) then the
    batch-1 kernel continues: same logits and tokens as step-by-step."""
    from Qwen06B_architecture import Decoder
    w = {k: ([t.cuda() for t in v] if isinstance(v, list) else v.cuda()) for k, v in weights_2l.items()}
    prompt = _prompts([150], seed=13)[0]
    a = Decoder(weights=w, verbose=False, num_layers=2)
    b = Decoder(weights=w, verbose=False, num_layers=2)
    for t in prompt[:-1]:
        a.step(t)
    b.prefill(prompt[:-1], max_rows=64)
    assert a.position == b.position == len(prompt) - 1
    n = len(prompt) - 1
    assert float((a._k_cache[:, :, :n].float() - b._k_cache[:, :, :n].float()).abs().max()) <= 5e-2
    assert float((a._v_cache[:, :, :n].float() - b._v_cache[:, :, :n].float()).abs().max()) <= 5e-2
    ta, tb = prompt[-1], prompt[-1]
    for s in range(4):
        ta_next, tb_next = a.step(ta), b.step(ta)
        la, lb = logits_from_norm(a._norm_out, w["embed_weight"]), logits_from_norm(b._norm_out, w["embed_weight"])
        assert float((la - lb).abs().max()) <= LOGIT_ATOL, f"step {s}"
        top2 = torch.topk(la, 2).values
        if float(top2[0] - top2[1]) > MARGIN:
            assert ta_next == tb_next, f"step {s}"
        ta = ta_next
