"""Paged KV pools and contexts beyond 2048 tokens in the batched path
(qwen_b200_batched_create_paged, include/qwen_b200_batched.h).

* Paged pools change only where K/V rows live: the same prompts and steps give
  bit-identical tokens and final-normed hidden states (the logits tap) as the
  contiguous pools, including after pages are released and handed to another
  sequence.
* An unmapped page is a recorded device-side error (status 3), not a read.
* max_seq 4096: a sequence past position 2048 decodes bit-identically on paged
  and contiguous pools, and matches the CPU oracle (fed the same tokens one
  position at a time, RoPE tables of 4096 rows) within the decode tolerances.
"""
import pytest
import torch

from decode_helpers import LOGIT_ATOL, MARGIN, logits_from_norm

pytestmark = pytest.mark.gpu


def _prompts(lengths, seed):
    g = torch.Generator().manual_seed(seed)
    return [torch.randint(0, 151936, (n,), generator=g).tolist() for n in lengths]


def _decode(bd, prompts, steps, seqs=None):
    """Parallel prefill, then greedy steps; returns tokens [steps][n] and
    norm_out [steps] (fp32, CPU)."""
    n = len(prompts)
    seqs = list(range(n)) if seqs is None else seqs
    bd.prefill_parallel(prompts, seqs=seqs)
    dev = bd.dev
    ids = torch.tensor(seqs, dtype=torch.int32, device=dev)
    pos = torch.tensor([len(p) - 1 for p in prompts], dtype=torch.int32, device=dev)
    tok = torch.tensor([p[-1] for p in prompts], dtype=torch.int32, device=dev)
    for i, p in zip(seqs, prompts):
        bd.reserve(i, len(p) - 1 + steps - 1)
    toks, norms = [], []
    for s in range(steps):
        norm = torch.empty(n, 1024, dtype=torch.float32, device=dev)
        out = torch.empty(n, dtype=torch.int32, device=dev)
        bd.step(ids, pos, tok, int(pos.max()), norm_out=norm, out=out)
        toks.append(out.cpu().tolist())
        norms.append(norm.cpu())
        tok, pos = out, pos + 1
    assert bd.status() == 0
    return toks, norms


def test_paged_equals_contiguous(weights_2l):
    from batched import BatchedDecoder
    prompts = _prompts([5, 130, 257, 40], seed=31)
    a = BatchedDecoder(weights_2l, num_seqs=4, max_rows=64, num_layers=2)
    b = BatchedDecoder(weights_2l, num_seqs=4, max_rows=64, num_layers=2, paged=True, num_pages=12)
    ta, na = _decode(a, prompts, 3)
    tb, nb = _decode(b, prompts, 3)
    assert ta == tb
    for x, y in zip(na, nb):
        assert torch.equal(x, y)
    assert b.pages_in_use == 1 + 2 + 3 + 1   # ceil((len + 2) / 128) per sequence


def test_pages_released_and_reused(weights_2l):
    from batched import BatchedDecoder
    p1, p2 = _prompts([200], seed=41), _prompts([150], seed=42)
    b = BatchedDecoder(weights_2l, num_seqs=2, max_rows=32, num_layers=2, paged=True, num_pages=2)
    _decode(b, p1, 2, seqs=[0])
    b.release(0)
    t_paged, n_paged = _decode(b, p2, 2, seqs=[1])          # reuses sequence 0's pages
    ref = BatchedDecoder(weights_2l, num_seqs=2, max_rows=32, num_layers=2)
    t_ref, n_ref = _decode(ref, p2, 2, seqs=[1])
    assert t_paged == t_ref
    assert all(torch.equal(x, y) for x, y in zip(n_paged, n_ref))


def test_unmapped_page_is_a_recorded_error(weights_2l):
    from batched import BatchedDecoder
    b = BatchedDecoder(weights_2l, num_seqs=2, max_rows=2, num_layers=2, paged=True, num_pages=4)
    z = torch.zeros(1, dtype=torch.int32, device=b.dev)
    b.step(z, z + 300, z + 5, 300)                           # nothing reserved for sequence 0
    assert b.status() == 3


def test_long_context_4096(weights_2l):
    from batched import BatchedDecoder
    from oracle.oracle import OracleModel
    from qwen_weights import rope_tables
    prompt = _prompts([2100], seed=51)[0]
    a = BatchedDecoder(weights_2l, num_seqs=1, max_rows=256, max_seq=4096, num_layers=2)
    b = BatchedDecoder(weights_2l, num_seqs=1, max_rows=256, max_seq=4096, num_layers=2,
                       paged=True, num_pages=20)
    ta, na = _decode(a, [prompt], 2)
    tb, nb = _decode(b, [prompt], 2)
    assert ta == tb and all(torch.equal(x, y) for x, y in zip(na, nb))
    w = dict(weights_2l)
    w["cos_table"], w["sin_table"] = rope_tables(4096)
    orc = OracleModel(w, num_layers=2, max_seq_len=4096)
    for t in prompt[:-1]:
        orc.step(t)
    t = prompt[-1]
    emb = weights_2l["embed_weight"].cuda()
    for s in range(2):
        r = orc.step(t, want_logits=True)
        diff = float((r["logits"] - logits_from_norm(na[s][0], emb)).abs().max())
        assert diff <= LOGIT_ATOL, f"step {s}: logits differ by {diff}"
        top2 = torch.topk(r["logits"], 2).values
        if float(top2[0] - top2[1]) > MARGIN:
            assert ta[s][0] == r["token"]
        t = ta[s][0]
