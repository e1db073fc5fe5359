"""launch_ldg_generate_nosync_static_ws (the non-allocating variant of
launch_ldg_generate_nosync, include/qwen_b200.h) against the allocating
launcher, through the C ABI.

Collected last on purpose: it must pass both alone and after every other test
has used the allocating launchers in the same process.  Both launchers run the
same kernel on the same inputs, so tokens must be equal, and the final-normed
hidden (as logits) and the K/V rows written must agree within the decode
tolerances of decode_helpers.
"""
import ctypes

import pytest
import torch

from decode_helpers import LOGIT_ATOL, CAbiDecoder, last_error, lib, logits_from_norm

pytestmark = pytest.mark.gpu

START = 1100  # 18 attention splits per KV head at this context length
STEPS = 8


def _static_ws_fn():
    f = lib().launch_ldg_generate_nosync_static_ws
    vp, i = ctypes.c_void_p, ctypes.c_int
    f.restype = i
    f.argtypes = [i, i] + [vp] * 20 + [i, i, i, ctypes.c_float, vp]
    return f


def _generate_static_ws(dec: CAbiDecoder, token: int, pos: int, n: int) -> list[int]:
    rc = _static_ws_fn()(int(token), int(n), *dec._ptrs(), dec.out.data_ptr(), dec.L, int(pos),
                         dec.max_seq, dec.scale, dec._stream())
    code, msg = last_error()
    assert rc == code
    if rc:
        raise RuntimeError(f"launch_ldg_generate_nosync_static_ws: {msg}")
    torch.cuda.synchronize(dec.dev)
    return dec.out[:n].cpu().tolist()


def _seeded_pair(weights, num_layers):
    g = torch.Generator().manual_seed(77)
    kc = torch.zeros(num_layers, 8, 2048, 128, dtype=torch.float16)
    vc = torch.zeros_like(kc)
    kc[:, :, :START] = torch.randn(num_layers, 8, START, 128, generator=g).half()
    vc[:, :, :START] = (0.5 * torch.randn(num_layers, 8, START, 128, generator=g)).half()
    a = CAbiDecoder(weights, num_layers)
    b = CAbiDecoder(weights, num_layers)
    for d in (a, b):
        d.kc.copy_(kc)
        d.vc.copy_(vc)
    return a, b


def _agree(a: CAbiDecoder, b: CAbiDecoder, pos: int, n: int, what: str):
    la = logits_from_norm(a.norm, a.w["embed_weight"])
    lb = logits_from_norm(b.norm, a.w["embed_weight"])
    diff = float((la - lb).abs().max())
    assert diff <= LOGIT_ATOL, f"{what}: logits differ by {diff}"
    kd = float((a.kc[:, :, pos:pos + n].float() - b.kc[:, :, pos:pos + n].float()).abs().max())
    vd = float((a.vc[:, :, pos:pos + n].float() - b.vc[:, :, pos:pos + n].float()).abs().max())
    assert kd <= 5e-2 and vd <= 5e-2, f"{what}: KV differ by k={kd} v={vd}"


def test_static_ws_matches_allocating_launcher_two_calls(weights_28l):
    a, b = _seeded_pair(weights_28l, 28)
    first = 4242
    # call 1: set-up on first use, then a launch
    ta = a.generate(first, START, STEPS)
    tb = _generate_static_ws(b, first, START, STEPS)
    assert tb == ta, (ta, tb)
    assert -1 not in tb
    _agree(a, b, START, STEPS, "call 1")
    # call 2: continues from the last token on the same caches
    ta2 = a.generate(ta[-1], START + STEPS, STEPS)
    tb2 = _generate_static_ws(b, tb[-1], START + STEPS, STEPS)
    assert tb2 == ta2, (ta2, tb2)
    assert -1 not in tb2
    _agree(a, b, START + STEPS, STEPS, "call 2")


def test_static_ws_rejects_bad_arguments(weights_2l):
    d = CAbiDecoder(weights_2l, 2)
    d.out.fill_(-7)
    rc = _static_ws_fn()(1, 4, *d._ptrs(), d.out.data_ptr(), 2, 2046, d.max_seq, d.scale,
                         d._stream())
    code, msg = last_error()
    assert rc != 0 and rc == code and "max_seq_len" in msg, (rc, msg)
    torch.cuda.synchronize()
    assert int(d.out[0].item()) == -7  # nothing was launched
