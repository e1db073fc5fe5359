"""The tcgen05 GEMM (qwen_b200_gemm_f16, include/qwen_b200_batched.h) against a
plain PyTorch fp32 reference of the same op, for every fused epilogue, with
rows and columns that are not multiples of the 128 x BN tile.

Tolerances (fp16 inputs, fp32 accumulation in a different order than the
reference): fp32 outputs within 1e-3 + 1e-3 * |ref|; fp16 outputs within
1 fp16 ulp of the rounded reference plus the same fp32 slack; argmax exact
on rows whose top-2 reference margin exceeds 1e-3.
"""
import ctypes

import pytest
import torch

from decode_helpers import last_error, lib

pytestmark = pytest.mark.gpu

EPI_F16, EPI_F32, EPI_F32_RES16, EPI_SWIGLU, EPI_F16_RES32, EPI_ARGMAX = range(6)


def _fn():
    f = lib().qwen_b200_gemm_f16
    vp, i = ctypes.c_void_p, ctypes.c_int
    f.restype = i
    f.argtypes = [i, vp, vp, vp, vp, vp, i, i, i, i, i, vp]
    w = lib().qwen_b200_gemm_argmax_workspace
    w.restype = ctypes.c_longlong
    w.argtypes = [i, i]
    return f, w


def gemm(epi, a, b, res=None, ldo=None, k_splits=1):
    f, wsz = _fn()
    M, K = a.shape
    N = b.shape[0]
    if epi == EPI_ARGMAX:
        out = torch.empty(M, dtype=torch.int32, device="cuda")
    elif epi == EPI_SWIGLU:
        out = torch.empty(M, N // 2, dtype=torch.float16, device="cuda")
    elif epi in (EPI_F32, EPI_F32_RES16):
        out = torch.empty(M, ldo or N, dtype=torch.float32, device="cuda")
    else:
        out = torch.empty(M, ldo or N, dtype=torch.float16, device="cuda")
    ws = torch.empty(max(16, wsz(M, N), k_splits * M * N * 4), dtype=torch.uint8, device="cuda")
    rc = f(epi, a.data_ptr(), b.data_ptr(), out.data_ptr(), res.data_ptr() if res is not None else None,
           ws.data_ptr(), M, N, K, ldo or N, k_splits,
           ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    if rc:
        raise RuntimeError(last_error())
    torch.cuda.synchronize()
    return out


def ref_mm(a, b):
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        return a.float() @ b.float().t()
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev


def silu_half_ref(x16: torch.Tensor) -> torch.Tensor:
    """fp16 SiLU with the upstream decode kernel's rounding steps
    (megakernel.cu:141-154), evaluated with torch fp16 ops on the GPU."""
    log2e = torch.tensor(1.44269504088896340736, dtype=torch.float16, device=x16.device)
    t = (-x16) * log2e
    e = torch.exp2(t.float()).half()
    d = (1.0 + e.float()).half()
    r = (1.0 / d.float()).half()
    return x16 * r


def _inputs(M, N, K, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    a = torch.randn(M, K, generator=g, device="cuda").half()
    b = (0.05 * torch.randn(N, K, generator=g, device="cuda")).half()
    return a, b


def _close16(out, ref32, what):
    ref16 = ref32.half()
    ulp = (ref16.float().abs().clamp_min(6e-5) * 2.0 ** -10)
    err = (out.float() - ref32).abs()
    bad = err > ulp + 1e-3 + 1e-3 * ref32.abs()
    assert not bool(bad.any()), f"{what}: max err {float(err.max())}"


SHAPES = [(1, 64, 64), (100, 80, 1024), (256, 1024, 2048), (200, 4096, 1024), (256, 6144, 1024),
          (130, 1024, 3072)]


@pytest.mark.parametrize("M,N,K", SHAPES)
def test_gemm_f16_and_f32(M, N, K):
    a, b = _inputs(M, N, K, M + N + K)
    ref = ref_mm(a, b)
    _close16(gemm(EPI_F16, a, b), ref, "f16")
    o32 = gemm(EPI_F32, a, b)
    assert torch.allclose(o32, ref, atol=1e-3, rtol=1e-3), float((o32 - ref).abs().max())


@pytest.mark.parametrize("M,N,K", [(256, 1024, 2048), (77, 1024, 3072)])
def test_gemm_residual_epilogues(M, N, K):
    a, b = _inputs(M, N, K, 5)
    ref = ref_mm(a, b)
    r16 = torch.randn(M, N, device="cuda").half()
    o = gemm(EPI_F32_RES16, a, b, res=r16)
    assert torch.allclose(o, ref + r16.float(), atol=1e-3, rtol=1e-3)
    r32 = torch.randn(M, N, device="cuda")
    o = gemm(EPI_F16_RES32, a, b, res=r32)
    _close16(o, ref + r32, "f16+res32")


@pytest.mark.parametrize("M", [1, 256])
def test_gemm_swiglu_epilogue(M):
    N, K = 6144, 1024
    a, b = _inputs(M, N, K, 11)
    ref = ref_mm(a, b)
    gate, up = ref[:, 0::2], ref[:, 1::2]
    want = (silu_half_ref(gate.half()).float() * up).half()
    out = gemm(EPI_SWIGLU, a, b)
    # a gate that rounds to the neighbouring fp16 value moves silu by ~1 ulp
    err = (out.float() - want.float()).abs()
    tol = 2 * want.float().abs().clamp_min(6e-5) * 2.0 ** -10 + 2e-3 * up.abs() + 1e-3
    assert not bool((err > tol).any()), float(err.max())
    assert float((out == want).float().mean()) > 0.95


@pytest.mark.parametrize("M,N", [(256, 151936), (3, 4096), (129, 1040)])
def test_gemm_argmax_epilogue(M, N):
    K = 1024
    a, b = _inputs(M, N, K, 3)
    ref = ref_mm(a, b)
    top2 = torch.topk(ref, 2, dim=1)
    margin = top2.values[:, 0] - top2.values[:, 1]
    got = gemm(EPI_ARGMAX, a, b).long()
    sel = margin > 1e-3
    assert bool(sel.any())
    assert torch.equal(got[sel], top2.indices[sel, 0])


@pytest.mark.parametrize("M,N,K,splits", [(256, 1024, 2048, 4), (256, 1024, 3072, 4), (77, 1024, 3072, 3),
                                          (5, 64, 128, 2)])
def test_gemm_split_k(M, N, K, splits):
    a, b = _inputs(M, N, K, 17)
    ref = ref_mm(a, b)
    r16 = torch.randn(M, N, device="cuda").half()
    o = gemm(EPI_F32_RES16, a, b, res=r16, k_splits=splits)
    assert torch.allclose(o, ref + r16.float(), atol=1e-3, rtol=1e-3)
    r32 = torch.randn(M, N, device="cuda")
    _close16(gemm(EPI_F16_RES32, a, b, res=r32, k_splits=splits), ref + r32, "split f16+res32")
    _close16(gemm(EPI_F16, a, b, k_splits=splits), ref, "split f16")
    assert torch.allclose(gemm(EPI_F32, a, b, k_splits=splits), ref, atol=1e-3, rtol=1e-3)


@pytest.mark.parametrize("M,N,K,splits", [(256, 1024, 2048, 4), (256, 1024, 3072, 4), (77, 1024, 3072, 3),
                                          (5, 64, 128, 2)])
def test_cluster_split_k_equals_workspace_split_k(M, N, K, splits):
    """Split-K added inside a thread-block cluster (workspace NULL) gives the
    same bits as the partials-in-global-memory path."""
    f, _ = _fn()
    a, b = _inputs(M, N, K, 23)
    for epi, odt, rdt in ((EPI_F32_RES16, torch.float32, torch.float16), (EPI_F16_RES32, torch.float16, torch.float32),
                          (EPI_F32, torch.float32, None), (EPI_F16, torch.float16, None)):
        res = torch.randn(M, N, device="cuda").to(rdt) if rdt is not None else None
        outs = []
        for ws in (torch.empty(splits * M * N * 4, dtype=torch.uint8, device="cuda"), None):
            out = torch.empty(M, N, dtype=odt, device="cuda")
            rc = f(epi, a.data_ptr(), b.data_ptr(), out.data_ptr(), res.data_ptr() if res is not None else None,
                   ws.data_ptr() if ws is not None else None, M, N, K, N, splits,
                   ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
            assert rc == 0, last_error()
            torch.cuda.synchronize()
            outs.append(out)
        assert torch.equal(outs[0], outs[1]), epi


def test_gemm_rejects_bad_shapes():
    f, _ = _fn()
    a = torch.zeros(4, 100, dtype=torch.float16, device="cuda")
    rc = f(EPI_F16, a.data_ptr(), a.data_ptr(), a.data_ptr(), None, None, 4, 4, 100, 4, 1, None)
    code, msg = last_error()
    assert rc != 0 and rc == code and "multiple" in msg


def gemm_tiled(epi, a, b, bn, res=None, k_splits=1, workspace=True):
    f = lib().qwen_b200_gemm_f16_tiled
    vp, i = ctypes.c_void_p, ctypes.c_int
    f.restype = i
    f.argtypes = [i, vp, vp, vp, vp, vp, i, i, i, i, i, i, vp]
    M, K = a.shape
    N = b.shape[0]
    if epi == EPI_SWIGLU:
        out = torch.empty(M, N // 2, dtype=torch.float16, device="cuda")
    elif epi in (EPI_F32, EPI_F32_RES16):
        out = torch.empty(M, N, dtype=torch.float32, device="cuda")
    else:
        out = torch.empty(M, N, dtype=torch.float16, device="cuda")
    ws = torch.empty(max(16, k_splits * M * N * 4), dtype=torch.uint8, device="cuda") if workspace else None
    rc = f(epi, a.data_ptr(), b.data_ptr(), out.data_ptr(), res.data_ptr() if res is not None else None,
           ws.data_ptr() if ws is not None else None, M, N, K, N, k_splits, bn,
           ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    if rc:
        raise RuntimeError(last_error())
    torch.cuda.synchronize()
    return out


@pytest.mark.parametrize("bn", [64, 128, 256])
@pytest.mark.parametrize("M,N,K", [(256, 4096, 1024), (130, 1024, 3072), (7, 256, 128)])
def test_gemm_tile_widths(bn, M, N, K):
    """Every tile width gives the reference result (256 columns: one
    128 x 256 accumulator per CTA, 48 KB ring stages)."""
    a, b = _inputs(M, N, K, bn + M)
    ref = ref_mm(a, b)
    _close16(gemm_tiled(EPI_F16, a, b, bn), ref, f"bn {bn}")
    r32 = torch.randn(M, N, device="cuda")
    ks = min(4, K // 64)
    _close16(gemm_tiled(EPI_F16_RES32, a, b, bn, res=r32, k_splits=ks), ref + r32, f"bn {bn} split")
    _close16(gemm_tiled(EPI_F16, a, b, bn, k_splits=ks, workspace=False), ref, f"bn {bn} cluster split")


@pytest.mark.parametrize("bn", [128, 256])
def test_swiglu_after_split_k(bn):
    """The SwiGLU epilogue after a split-K reduction (cluster and partials
    forms give the same bits as each other and as the unsplit GEMM, up to the
    fp32 summation order of the slices)."""
    M, N, K = 256, 6144, 1024
    a, b = _inputs(M, N, K, 31)
    one = gemm_tiled(EPI_SWIGLU, a, b, bn)
    cl = gemm_tiled(EPI_SWIGLU, a, b, bn, k_splits=2, workspace=False)
    part = gemm_tiled(EPI_SWIGLU, a, b, bn, k_splits=2)
    assert torch.equal(cl, part)
    ref = ref_mm(a, b)
    gate, up = ref[:, 0::2], ref[:, 1::2]
    want = (silu_half_ref(gate.half()).float() * up).half()
    for out in (one, cl):
        err = (out.float() - want.float()).abs()
        tol = 2 * want.float().abs().clamp_min(6e-5) * 2.0 ** -10 + 2e-3 * up.abs() + 1e-3
        assert not bool((err > tol).any()), float(err.max())


@pytest.mark.parametrize("M,N", [(1, 151936), (129, 18992), (256, 151936), (300, 4160)])
def test_persistent_lm_head_argmax_matches_tile_kernel(M, N):
    """The lm_head path (qwen_b200_lmhead_argmax: one persistent CTA per SM
    over all tiles, double-buffered accumulators) gives the same tokens as the
    one-tile-per-CTA EPI_ARGMAX GEMM, bit for bit (same per-tile MMA order,
    lowest index among equal values), and the fp32 reference's token where
    the top two logits are apart.  Shapes: a single row, ragged column tiles
    (an 8-way vocabulary shard), three row tiles."""
    K = 1024
    a, b = _inputs(M, N, K, 41)
    want = gemm(EPI_ARGMAX, a, b)
    f = lib().qwen_b200_lmhead_argmax
    f.restype = ctypes.c_int
    f.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_longlong,
                  ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
    wsz = lib().qwen_b200_lmhead_argmax_workspace
    wsz.restype = ctypes.c_longlong
    wsz.argtypes = [ctypes.c_int, ctypes.c_int]
    ws = torch.empty(max(16, wsz(M, N)), dtype=torch.uint8, device="cuda")
    val = torch.empty(M, dtype=torch.float32, device="cuda")
    idx = torch.empty(M, dtype=torch.int32, device="cuda")
    rc = f(a.data_ptr(), b.data_ptr(), M, N, 0, val.data_ptr(), idx.data_ptr(), ws.data_ptr(),
           ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    if rc:
        raise RuntimeError(last_error())
    torch.cuda.synchronize()
    assert torch.equal(idx, want)
    ref = ref_mm(a, b)
    top2 = torch.topk(ref, 2, dim=1)
    sel = (top2.values[:, 0] - top2.values[:, 1]) > 1e-3
    assert torch.equal(idx.long()[sel], top2.indices[sel, 0])
    assert torch.allclose(val, ref.gather(1, idx.long().view(-1, 1)).view(-1), atol=2e-3, rtol=2e-3)
