"""Parity of the B200 RMSNorm / SwiGLU operators (modules ``rmsnorm`` and
``swiglu_fused``, C ABI include/qwen_b200_ops.h) with the upstream operators'
own outputs (tests/golden/ref_ops.npz, produced by the unmodified upstream
Tools/rmsnorm and Tools/swiglu kernels on a B200) and with the CPU oracle.

Tolerances:
* SwiGLU chains (gate, up, down, fp16 accumulation in upstream's order):
  bit-exact.  The SiLU output goes through expf, which the CPU oracle takes
  from libm, so where the oracle (not upstream's golden) is the reference the
  SwiGLU output may differ by 1 fp16 ulp in rare elements, and the down chain
  is then checked bit-exactly on the GPU's own activations.
* RMSNorm: >= 99.9% of outputs bit-equal to upstream's, the rest within
  1 fp16 ulp (the fp32 sum of squares is added in a different order); rms
  within rtol 1e-6; the fused residual update bit-exact.
"""
import sys

import numpy as np
import pytest
import torch

from conftest import GOLDEN

sys.path.insert(0, GOLDEN)
from inputs import OPS_CASE, ops_inputs  # noqa: E402
from oracle import oracle as O  # noqa: E402

pytestmark = pytest.mark.gpu


def _mods():
    import rmsnorm
    import swiglu_fused
    return rmsnorm, swiglu_fused


def _golden():
    return np.load(f"{GOLDEN}/ref_ops.npz")


def _h(a) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a).view(np.float16))


def _ordered(t: torch.Tensor) -> torch.Tensor:
    i = t.contiguous().view(torch.int16).to(torch.int32)
    return torch.where(i < 0, -(i & 0x7FFF), i)


def max_ulps(a: torch.Tensor, b: torch.Tensor) -> int:
    return int((_ordered(a.cpu()) - _ordered(b.cpu())).abs().max())


def _check_rms_out(ours, ref, what):
    ours = ours.cpu()
    eq = float((ours == ref).float().mean())
    assert eq >= 0.999, f"{what}: only {eq:.5f} of outputs bit-equal"
    assert max_ulps(ours, ref) <= 1, f"{what}: {max_ulps(ours, ref)} ulps"


def down_chain(s: torch.Tensor, wd: torch.Tensor, bd: torch.Tensor | None = None) -> torch.Tensor:
    """out = bd + sum_i s[:, i] * wd[i, :] with every product and partial sum
    rounded to fp16, i ascending (swiglu.cu:288-305).  torch's CPU fp16 ops
    round each result, so the loop reproduces the chain exactly."""
    s, wd = s.cpu(), wd.cpu()
    acc = torch.zeros(s.shape[0], wd.shape[1], dtype=torch.float16)
    if bd is not None:
        acc += bd.cpu()
    for i in range(s.shape[1]):
        acc = acc + s[:, i:i + 1] * wd[i:i + 1, :]
    return acc


@pytest.mark.parametrize("b", OPS_CASE["batches"])
def test_rmsnorm_matches_upstream(b):
    rmsnorm, _ = _mods()
    g = _golden()
    x, w, resid, *_ = ops_inputs(b)
    out, rms = rmsnorm.forward(x.cuda(), w.cuda(), OPS_CASE["eps"])
    _check_rms_out(out, _h(g[f"rms_out_{b}"]), f"simple B={b}")
    assert np.allclose(rms.cpu().numpy(), g[f"rms_rms_{b}"], rtol=1e-6)
    r2 = resid.cuda()
    outf, rmsf = rmsnorm.forward(x.cuda(), w.cuda(), OPS_CASE["eps"], r2)
    assert torch.equal(r2.cpu(), _h(g[f"rmsf_res_{b}"]))
    _check_rms_out(outf, _h(g[f"rmsf_out_{b}"]), f"fused B={b}")
    assert np.allclose(rmsf.cpu().numpy(), g[f"rmsf_rms_{b}"], rtol=1e-6)


@pytest.mark.parametrize("b", OPS_CASE["swiglu_batches"])
def test_swiglu_bit_exact_with_upstream(b):
    _, sw = _mods()
    g = _golden()
    _, _, _, wg, wu, wd = ops_inputs(b)
    xs = _h(g[f"rms_out_{b}"]).view(b, 1, 1024).cuda()
    y = sw.forward_down(xs, wg.cuda(), wu.cuda(), wd.cuda())
    assert torch.equal(y.cpu(), _h(g[f"swd_out_{b}"]).view(b, 1, 1024))
    f, gc, uc = sw.forward(xs, wg.cuda(), wu.cuda())
    assert torch.equal(f.cpu(), _h(g[f"swf_out_{b}"]).view(b, 1, 3072))


@pytest.mark.parametrize("b", [64, 256])
def test_swiglu_large_batch(b):
    _, sw = _mods()
    x, _, _, wg, wu, wd = ops_inputs(b)
    xs = x.view(b, 1, 1024)
    f, gc, uc = sw.forward(xs.cuda(), wg.cuda(), wu.cuda())
    rf, rgc, ruc = O.swiglu_forward(xs, wg, wu)
    assert torch.equal(gc.cpu(), rgc) and torch.equal(uc.cpu(), ruc)
    assert max_ulps(f, rf) <= 1 and float((f.cpu() == rf).float().mean()) >= 0.999
    y = sw.forward_down(xs.cuda(), wg.cuda(), wu.cuda(), wd.cuda(), exact=True)
    assert torch.equal(y.cpu().view(b, 1024), down_chain(f.view(b, 3072), wd))


def test_swiglu_biases_and_ragged_shapes():
    """Biases, rows not a multiple of the 16-row tile, reduction lengths that
    are not a multiple of the 128-long chunk."""
    _, sw = _mods()
    gen = torch.Generator().manual_seed(99)
    rows, h, inter = 5, 40, 24
    x = torch.randn(1, rows, h, generator=gen).half()
    wg = (0.3 * torch.randn(h, inter, generator=gen)).half()
    wu = (0.3 * torch.randn(h, inter, generator=gen)).half()
    wd = (0.3 * torch.randn(inter, h, generator=gen)).half()
    bg, bu, bd = ((0.5 * torch.randn(n, generator=gen)).half() for n in (inter, inter, h))
    f, gc, uc = sw.forward(x.cuda(), wg.cuda(), wu.cuda(), bg.cuda(), bu.cuda())
    rf, rgc, ruc = O.swiglu_forward(x, wg, wu, bg, bu)
    assert torch.equal(gc.cpu(), rgc) and torch.equal(uc.cpu(), ruc)
    assert max_ulps(f, rf) <= 1
    y = sw.forward_down(x.cuda(), wg.cuda(), wu.cuda(), wd.cuda(), bg.cuda(), bu.cuda(), bd.cuda())
    assert torch.equal(y.cpu().view(rows, h), down_chain(f.view(rows, inter), wd, bd))
    # Keyword form and None biases, as upstream's Python callers pass them.
    y0 = sw.forward_down(x.cuda(), wg.cuda(), wu.cuda(), wd.cuda(), b_gate=None, b_up=None, b_down=None)
    f0, _, _ = sw.forward(x.cuda(), wg.cuda(), wu.cuda())
    assert torch.equal(y0.cpu().view(rows, h), down_chain(f0.view(rows, inter), wd))


@pytest.mark.parametrize("cols", [1000, 36, 1030])
def test_rmsnorm_odd_widths(cols):
    """Widths that are not multiples of 8 (and of 4), where upstream's
    remainder path rounds differently."""
    rmsnorm, _ = _mods()
    gen = torch.Generator().manual_seed(cols)
    x = torch.randn(7, cols, generator=gen).half()
    w = (1.0 + 0.1 * torch.randn(cols, generator=gen)).half()
    res = torch.randn(7, cols, generator=gen).half()
    out, rms = rmsnorm.forward(x.cuda(), w.cuda(), 1e-6)
    rout, rrms = O.rmsnorm_forward(x, w, 1e-6)
    assert max_ulps(out, rout) <= 1 and np.allclose(rms.cpu().numpy(), rrms.numpy(), rtol=1e-6)
    r_gpu, r_cpu = res.cuda(), res.clone()
    out, rms = rmsnorm.forward(x.cuda(), w.cuda(), 1e-6, r_gpu)
    rout, rrms = O.rmsnorm_forward(x, w, 1e-6, r_cpu)
    assert torch.equal(r_gpu.cpu(), r_cpu)
    assert max_ulps(out, rout) <= 1 and np.allclose(rms.cpu().numpy(), rrms.numpy(), rtol=1e-6)


@pytest.mark.parametrize("b", [1, 64])
def test_rmsnorm_forward_down_equals_the_two_calls(b):
    rmsnorm, sw = _mods()
    x, w, resid, wg, wu, wd = (t.cuda() for t in ops_inputs(b))
    n, rms = rmsnorm.forward(x, w, 1e-6)
    y = sw.forward_down(n.view(b, 1, 1024), wg, wu, wd)
    y2, n2, rms2 = sw.rmsnorm_forward_down(x, w, 1e-6, wg, wu, wd)
    assert torch.equal(n2, n) and torch.equal(rms2, rms) and torch.equal(y2, y.view(b, 1024))
    r_a, r_b = resid.clone(), resid.clone()
    n, _ = rmsnorm.forward(x, w, 1e-6, r_a)
    y = sw.forward_down(n.view(b, 1, 1024), wg, wu, wd)
    y3, n3, _ = sw.rmsnorm_forward_down(x, w, 1e-6, wg, wu, wd, residual=r_b)
    assert torch.equal(r_a, r_b) and torch.equal(n3, n) and torch.equal(y3, y.view(b, 1024))


def test_operator_errors_and_empty_inputs():
    rmsnorm, sw = _mods()
    w = torch.ones(1024, dtype=torch.float16, device="cuda")
    wg = torch.zeros(1024, 3072, dtype=torch.float16, device="cuda")
    with pytest.raises(RuntimeError, match="float16"):
        rmsnorm.forward(torch.zeros(2, 1024, device="cuda"), w, 1e-6)
    with pytest.raises(RuntimeError, match="batch, seq, hidden"):
        sw.forward(torch.zeros(2, 1024, dtype=torch.float16, device="cuda"), wg, wg)
    with pytest.raises(RuntimeError, match="hidden"):
        sw.forward(torch.zeros(1, 1, 1000, dtype=torch.float16, device="cuda"), wg, wg)
    with pytest.raises(RuntimeError, match="not part of this inference build"):
        sw.backward()
    out, rms = rmsnorm.forward(torch.zeros(0, 1024, dtype=torch.float16, device="cuda"), w, 1e-6)
    assert out.shape == (0, 1024) and rms.shape == (0,)
    f, _, _ = sw.forward(torch.zeros(0, 1, 1024, dtype=torch.float16, device="cuda"), wg, wg)
    assert f.shape == (0, 1, 3072)
    import ctypes
    from decode_helpers import lib
    st = ctypes.c_uint64(0)
    lib().qwen_b200_ops_status.restype = ctypes.c_int
    assert lib().qwen_b200_ops_status(ctypes.byref(st)) == 0


# ---------------------------------------------------------------- tensor cores
# forward_down / rmsnorm_forward_down with exact=False (and by default from 64
# rows): tcgen05 GEMMs with fp32 accumulation instead of upstream's fp16
# chains.  Acceptance: every output at least as close to a float64 evaluation
# of the same operator (SwiGLU activations rounded to fp16 only where the
# operator itself stores them: not at all in the reference) as upstream's
# output, plus one fp16 ulp of the reference value.

def _ref64(x, wg, wu, wd, bg=None, bu=None, bd=None):
    x = x.double().reshape(-1, x.shape[-1])
    g = x @ wg.double()
    u = x @ wu.double()
    if bg is not None:
        g = g + bg.double()
    if bu is not None:
        u = u + bu.double()
    s = g / (1.0 + torch.exp(-g)) * u
    y = s @ wd.double()
    if bd is not None:
        y = y + bd.double()
    return y


def _ulp(ref: torch.Tensor) -> torch.Tensor:
    """fp16 ulp at |ref|: 2^(e - 11) for |ref| = m 2^e, m in [0.5, 1); 2^-24 at the bottom."""
    _, e = torch.frexp(ref.abs())
    return torch.pow(2.0, (e - 11).to(torch.float64)).clamp_min(2.0 ** -24)


def _check_closer(tc, chain, ref, what):
    tc, chain = tc.cpu().double().reshape(ref.shape), chain.cpu().double().reshape(ref.shape)
    e_tc, e_up = (tc - ref).abs(), (chain - ref).abs()
    bad = e_tc > e_up + _ulp(ref)
    assert not bool(bad.any()), (f"{what}: {int(bad.sum())} of {bad.numel()} outputs farther from the "
                                 f"float64 value than upstream's + 1 ulp; worst excess "
                                 f"{float((e_tc - e_up - _ulp(ref)).max()):.3g}")
    return float(e_tc.max()), float(e_up.max())


@pytest.mark.parametrize("b", [64, 256, 1, 8, 129])
def test_swiglu_forward_down_tensor_cores(b):
    _, sw = _mods()
    x, w, _, wg, wu, wd = ops_inputs(b)
    xg = x.cuda().view(b, 1, 1024)
    wgc, wuc, wdc = wg.cuda(), wu.cuda(), wd.cuda()
    tc = sw.forward_down(xg, wgc, wuc, wdc, exact=False)
    chain = sw.forward_down(xg, wgc, wuc, wdc, exact=True)
    ref = _ref64(x, wg, wu, wd)
    e_tc, e_up = _check_closer(tc, chain, ref, f"B={b}")
    assert e_tc < e_up, (e_tc, e_up)
    if b >= 64:  # the default takes the tensor cores from 64 rows on
        assert torch.equal(sw.forward_down(xg, wgc, wuc, wdc), tc)
    else:
        assert torch.equal(sw.forward_down(xg, wgc, wuc, wdc), chain)


def test_swiglu_forward_down_tensor_cores_biases():
    _, sw = _mods()
    b = 96
    x, w, _, wg, wu, wd = ops_inputs(b)
    g = torch.Generator().manual_seed(11)
    bg, bu = (0.1 * torch.randn(3072, generator=g)).half(), (0.1 * torch.randn(3072, generator=g)).half()
    bd = (0.1 * torch.randn(1024, generator=g)).half()
    args = [t.cuda() for t in (wg, wu, wd, bg, bu, bd)]
    xg = x.cuda().view(b, 1, 1024)
    tc = sw.forward_down(xg, *args, exact=False)
    chain = sw.forward_down(xg, *args, exact=True)
    _check_closer(tc, chain, _ref64(x, wg, wu, wd, bg, bu, bd), "biases")


@pytest.mark.parametrize("b", [64, 256])
def test_rmsnorm_forward_down_tensor_cores(b):
    rn, sw = _mods()
    x, w, resid, wg, wu, wd = ops_inputs(b)
    args = [t.cuda() for t in (wg, wu, wd)]
    out_tc, normed_tc, rms_tc = sw.rmsnorm_forward_down(x.cuda(), w.cuda(), OPS_CASE["eps"], *args,
                                                        exact=False)
    out_ch, normed_ch, rms_ch = sw.rmsnorm_forward_down(x.cuda(), w.cuda(), OPS_CASE["eps"], *args,
                                                        exact=True)
    # The RMSNorm half is the same kernel either way.
    assert torch.equal(normed_tc, normed_ch) and torch.equal(rms_tc, rms_ch)
    _check_closer(out_tc, out_ch, _ref64(normed_ch.cpu(), wg, wu, wd), f"rmsnorm B={b}")
    # Against upstream's own operators where the golden file holds them.
    g = _golden()
    if f"swd_out_{b}" in g.files:
        up = _h(g[f"swd_out_{b}"]).view(b, 1024)
        assert float((out_tc.cpu().float() - up.float()).abs().max()) < 5e-2
