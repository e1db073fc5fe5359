"""Sampling (include/qwen_b200_sample.h, qwen0.6b_b200/sampling.py) against the
transformers logits warpers that upstream's benchmark runs through generate()
(TemperatureLogitsWarper, TopKLogitsWarper, TopPLogitsWarper, in that order).

* Kept sets: the sampler reports the smallest kept z per row (z = logit / T,
  correctly rounded, as torch divides on the CPU); {z >= kept_min}
  must equal the warpers' surviving set on untied logits up to the top-p
  cut's fp32 rounding (tokens whose exact mass-above is within 2e-4 of
  top_p), keep every tie of the k-th value (as TopKLogitsWarper does), and,
  for top-p on tied values, differ only inside the boundary group.
* Draws: chi-square of 40,000 draws against the warpers' filtered softmax;
  every draw inside the kept set; same (seed, offset) -> same tokens.
* temperature 0 and top_k 1 give the greedy argmax (lowest index on ties).
* The radix selection's overflow path (a boundary bin with more elements than
  fit in shared memory).
* Decoder.sample_ids(top_k=1) equals greedy generate_ids; sampled decode is
  reproducible; the batched step's sampled tokens lie in each row's kept set.
"""
import pytest
import torch

pytestmark = pytest.mark.gpu

V = 151936


def _warpers():
    lp = pytest.importorskip("transformers.generation.logits_process")
    return lp.TemperatureLogitsWarper, lp.TopKLogitsWarper, lp.TopPLogitsWarper


def hf_filtered(logits: torch.Tensor, T: float, k: int, p: float) -> torch.Tensor:
    """Warped scores (float32, CPU): -inf where a warper removed the token."""
    Temp, TopK, TopP = _warpers()
    s = logits.float().cpu().clone()
    s = Temp(T)(None, s)
    if k > 0:
        s = TopK(k)(None, s)
    if p < 1.0:
        s = TopP(p)(None, s)
    return s


def run(logits, T, k, p, seed=1, offset=0):
    from sampling import SamplingParams, sample
    rows = logits.shape[0]
    km = torch.empty(rows, dtype=torch.float32, device="cuda")
    tok = sample(logits, SamplingParams(T, k, p, seed), offset=offset, kept_min=km)
    torch.cuda.synchronize()
    return tok.cpu(), km.cpu()


CASES = [(1.0, 50, 1.0), (0.7, 0, 0.9), (1.3, 200, 0.8), (1.0, 0, 0.5), (2.0, 1000, 0.95),
         (0.5, 5000, 1.0), (1.0, 0, 0.999)]


@pytest.mark.parametrize("T,k,p", CASES)
def test_kept_set_matches_transformers(T, k, p):
    g = torch.Generator(device="cuda").manual_seed(int(T * 100) + k + int(p * 1000))
    logits = 3.0 * torch.randn(6, V, generator=g, device="cuda")
    tok, km = run(logits, T, k, p)
    ref = hf_filtered(logits, T, k, p)
    z = logits.cpu() / T   # on the CPU: torch's CUDA scalar division is not correctly rounded
    for r in range(logits.shape[0]):
        ours = z[r] >= km[r]
        theirs = torch.isfinite(ref[r])
        diff = (ours != theirs).nonzero().flatten()
        if diff.numel():
            # Only a top-p cut may differ: both sides add fp32 masses in
            # different orders (transformers: a sequential cumsum over the
            # sorted vocabulary), so tokens whose mass-above lies within fp32
            # accumulation error of top_p can fall either way.  Checked against
            # the exact (float64) mass above each differing token.
            assert p < 1.0, (r, diff[:10])
            probs = torch.softmax(hf_filtered(logits[r:r + 1], T, k, 1.0)[0].double(), 0)
            for i in diff.tolist():
                above = float(probs[z[r] > z[r, i]].sum())
                assert abs(above - p) < 2e-4, (r, i, above)
        assert bool(ours[int(tok[r])]), (r, int(tok[r]))


def test_ties_topk_kept_like_transformers_topp_as_groups():
    g = torch.Generator(device="cuda").manual_seed(5)
    logits = torch.round(2.0 * torch.randn(4, V, generator=g, device="cuda")) / 2.0  # many ties
    _, km = run(logits, 1.0, 300, 1.0)
    ref = hf_filtered(logits, 1.0, 300, 1.0)
    for r in range(4):
        assert torch.equal(logits[r].cpu() >= km[r], torch.isfinite(ref[r]))
    _, km = run(logits, 1.0, 0, 0.7)
    ref = hf_filtered(logits, 1.0, 0, 0.7)
    for r in range(4):
        ours, theirs = logits[r].cpu() >= km[r], torch.isfinite(ref[r])
        assert bool((theirs & ~ours).sum() == 0)            # every token they keep, we keep
        extra = ours & ~theirs
        if bool(extra.any()):                                 # extras: the boundary group only
            assert bool((logits[r].cpu()[extra] == km[r]).all())


def test_draws_follow_the_filtered_softmax():
    scipy_stats = pytest.importorskip("scipy.stats")
    g = torch.Generator(device="cuda").manual_seed(11)
    base = 2.0 * torch.randn(1000, generator=g, device="cuda")
    T, k, p, n = 0.8, 50, 0.9, 40000
    logits = base.repeat(n, 1).contiguous()
    tok, km = run(logits, T, k, p, seed=123)
    ref = hf_filtered(base.view(1, -1), T, k, p)[0]
    probs = torch.softmax(ref.double(), 0)
    kept = torch.isfinite(ref)
    assert bool(kept[tok.long()].all()), "a draw outside the kept set"
    counts = torch.bincount(tok.long(), minlength=1000).double()
    exp = probs * n
    sel = exp >= 5
    chi2 = float((((counts - exp) ** 2) / exp)[sel].sum())
    df = int(sel.sum()) - 1
    assert chi2 < scipy_stats.chi2.isf(1e-6, df), (chi2, df)
    tok2, _ = run(logits, T, k, p, seed=123)
    assert torch.equal(tok, tok2)                            # same stream, same draws
    tok3, _ = run(logits, T, k, p, seed=124)
    assert not torch.equal(tok, tok3)


def test_greedy_limits():
    g = torch.Generator(device="cuda").manual_seed(3)
    logits = torch.randn(5, V, generator=g, device="cuda")
    logits[2, 10] = logits[2, 77] = logits[2].max() + 1.0     # tie: lowest index wins
    want = logits.argmax(1).cpu()
    want[2] = 10
    for T, k in ((0.0, 0), (1.0, 1), (0.0, 40)):
        tok, _ = run(logits, T, k, 1.0)
        assert torch.equal(tok.long(), want.long()), (T, k)


def test_radix_overflow_path():
    # 20,000 distinct values in one level-0 bin ([1, 1.25) shares its top 11 key bits).
    g = torch.Generator(device="cuda").manual_seed(9)
    logits = torch.full((2, V), -10.0, device="cuda")
    logits[:, :20000] = 1.0 + 0.25 * torch.rand(2, 20000, generator=g, device="cuda")
    for k, p in ((5000, 1.0), (0, 0.3), (12000, 0.5)):
        tok, km = run(logits, 1.0, k, p)
        ref = hf_filtered(logits, 1.0, k, p)
        for r in range(2):
            ours, theirs = logits[r].cpu() >= km[r], torch.isfinite(ref[r])
            assert int((ours != theirs).sum()) <= 1, (k, p, int((ours != theirs).sum()))
    zeros = torch.zeros(1, V, device="cuda")                   # every value tied
    _, km = run(zeros, 1.0, 1000, 1.0)
    assert float(km[0]) == 0.0                                 # all kept, as TopKLogitsWarper keeps ties


@pytest.mark.parametrize("T,k,p", [(1.0, 50, 1.0), (0.8, 200, 0.9), (1.0, 0, 0.7), (1.3, 0, 1.0),
                                   (0.0, 0, 1.0), (1.0, 1, 1.0)])
def test_cluster_and_one_cta_paths_agree(T, k, p):
    """The cluster-per-row path (a window that contains the kept set, held in
    shared memory) and the one-CTA path give the same kept set and tokens."""
    from sampling import set_cluster_path
    g = torch.Generator(device="cuda").manual_seed(77 + k)
    logits = 3.0 * torch.randn(5, V, generator=g, device="cuda")
    try:
        set_cluster_path(True)
        t_c, km_c = run(logits, T, k, p, seed=9, offset=3)
        set_cluster_path(False)
        t_1, km_1 = run(logits, T, k, p, seed=9, offset=3)
    finally:
        set_cluster_path(True)
    if p >= 1.0 and T > 0 and k not in (0, 1):
        assert torch.equal(km_c, km_1)                         # exact thresholds
    z = logits.cpu() / T if T > 0 else logits.cpu()
    for r in range(5):
        d = int(((z[r] >= km_c[r]) != (z[r] >= km_1[r])).sum())
        assert d <= 2, (r, d)                                  # top-p: fp32 mass order only
        if d == 0:
            assert int(t_c[r]) == int(t_1[r])                  # same set, same noise, same token


def test_rejects_bad_parameters():
    from sampling import SamplingParams, sample
    x = torch.zeros(1, 10, device="cuda")
    for T, k, p in ((-1.0, 0, 1.0), (1.0, -2, 1.0), (1.0, 0, 0.0), (1.0, 0, 1.5)):
        with pytest.raises(RuntimeError, match="bad sampling parameters"):
            sample(x, SamplingParams(T, k, p))


def test_decoder_sampling(weights_2l):
    from Qwen06B_architecture import Decoder
    w = {k: ([t.cuda() for t in v] if isinstance(v, list) else v.cuda()) for k, v in weights_2l.items()}
    dec = Decoder(weights=w, verbose=False, num_layers=2)
    prompt = [5, 900, 151000, 42]
    greedy = dec.generate_ids(prompt, 6)
    assert dec.sample_ids(prompt, 6, temperature=1.0, top_k=1) == greedy
    a = dec.sample_ids(prompt, 8, temperature=1.0, top_p=0.95, seed=7)
    b = dec.sample_ids(prompt, 8, temperature=1.0, top_p=0.95, seed=7)
    assert a == b and all(0 <= t < V for t in a)


def test_batched_sampling_tokens_in_kept_set(weights_2l):
    from batched import BatchedDecoder
    from sampling import SamplingParams, sample
    bd = BatchedDecoder(weights_2l, num_seqs=3, max_rows=3, num_layers=2)
    prompts = [[1, 2, 3], [400, 5000], [7, 8, 9, 10]]
    bd.prefill(prompts)
    ids = torch.arange(3, dtype=torch.int32, device=bd.dev)
    pos = torch.tensor([len(p) - 1 for p in prompts], dtype=torch.int32, device=bd.dev)
    tok = torch.tensor([p[-1] for p in prompts], dtype=torch.int32, device=bd.dev)
    sp = SamplingParams(0.9, 20, 0.9, seed=3)
    out = bd.step(ids, pos, tok, int(pos.max()), out=torch.empty(3, dtype=torch.int32, device=bd.dev),
                  sampling=sp).cpu()
    logits = bd._logits[:3].clone()
    km = torch.empty(3, dtype=torch.float32, device=bd.dev)
    again = sample(logits, sp, row_seq=ids, row_pos=pos, kept_min=km).cpu()
    torch.cuda.synchronize()
    assert torch.equal(out, again)                             # keyed by (sequence, position)
    z = logits.cpu() / 0.9
    for r in range(3):
        assert bool(z[r, int(out[r])] >= km.cpu()[r])
    assert bd.status() == 0
