"""launch_ldg_generate_nosync_static_ws (the non-allocating variant of
launch_ldg_generate_nosync, include/qwen_b200.h) against the allocating
launcher, through the C ABI.

Collected last on purpose: it must pass both alone and after every other test
has used the allocating launchers in the same process.  Both launchers run the
same kernel on the same inputs, so tokens must be equal, and the final-normed
hidden (as logits) and the K/V rows written must agree within the decode
tolerances of decode_helpers.

The static-workspace calls run on a non-blocking torch stream, as a caller
with its own streams would: the one-time set-up of the first call must be
ordered before the launch on that stream.  A second test repeats the check in
a fresh process where nothing else ran first, and also asserts that the
static path neither set up the allocating launchers' workspace nor changed
the device's free memory or torch's allocation during its second call.
"""
import ctypes
import os
import subprocess
import sys

import pytest
import torch

from decode_helpers import LOGIT_ATOL, CAbiDecoder, last_error, lib, logits_from_norm

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))

START = 1100  # 18 attention splits per KV head at this context length
STEPS = 8


def _static_ws_fn():
    f = lib().launch_ldg_generate_nosync_static_ws
    vp, i = ctypes.c_void_p, ctypes.c_int
    f.restype = i
    f.argtypes = [i, i] + [vp] * 20 + [i, i, i, ctypes.c_float, vp]
    return f


def _launch_static_ws(dec: CAbiDecoder, token: int, pos: int, n: int) -> None:
    rc = _static_ws_fn()(int(token), int(n), *dec._ptrs(), dec.out.data_ptr(), dec.L, int(pos),
                         dec.max_seq, dec.scale, dec._stream())
    code, msg = last_error()
    assert rc == code
    if rc:
        raise RuntimeError(f"launch_ldg_generate_nosync_static_ws: {msg}")


def _generate_static_ws(dec: CAbiDecoder, token: int, pos: int, n: int) -> list[int]:
    _launch_static_ws(dec, token, pos, n)
    torch.cuda.synchronize(dec.dev)
    return dec.out[:n].cpu().tolist()


def _workspace_info(device: int) -> tuple[int, int]:
    f = lib().qwen_b200_workspace_info
    f.restype = ctypes.c_int
    f.argtypes = [ctypes.c_int, ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_int)]
    a, b = ctypes.c_int(-1), ctypes.c_int(-1)
    assert f(device, ctypes.byref(a), ctypes.byref(b)) == 0
    return a.value, b.value


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
    side = torch.cuda.Stream()
    # call 1: set-up on first use, then a launch
    ta = a.generate(first, START, STEPS)
    with torch.cuda.stream(side):
        tb = _generate_static_ws(b, first, START, STEPS)
    assert tb == ta, (ta, tb)
    assert -1 not in tb
    _agree(a, b, START, STEPS, "call 1")
    # call 2: continues from the last token on the same caches
    ta2 = a.generate(ta[-1], START + STEPS, STEPS)
    with torch.cuda.stream(side):
        tb2 = _generate_static_ws(b, tb[-1], START + STEPS, STEPS)
    assert tb2 == ta2, (ta2, tb2)
    assert -1 not in tb2
    _agree(a, b, START + STEPS, STEPS, "call 2")
    assert lib().qwen_b200_device_status(torch.cuda.current_device(), None) == 0


# Run in a fresh process by the test below: the static path first, on a
# non-blocking stream, with nothing else having touched the library.
_FRESH = r"""
import sys, torch
sys.path.insert(0, sys.argv[1])
import conftest  # noqa: F401  (import paths)
from qwen_weights import synthetic_weights
from decode_helpers import lib
import test_zz_no_alloc as T
torch.cuda.set_device(0)
a, b = T._seeded_pair(synthetic_weights(seed=7, num_layers=2), 2)
first, S, N = 4242, T.START, T.STEPS
assert T._workspace_info(0) == (0, 0)
side = torch.cuda.Stream()
with torch.cuda.stream(side):
    tb = T._generate_static_ws(b, first, S, N)                 # call 1: set-up + launch
    assert T._workspace_info(0) == (0, 1), T._workspace_info(0)
    torch.cuda.synchronize()
    free0, alloc0 = torch.cuda.mem_get_info()[0], torch.cuda.memory_allocated()
    T._launch_static_ws(b, tb[-1], S + N, N)                  # call 2
    torch.cuda.synchronize()
    free1, alloc1 = torch.cuda.mem_get_info()[0], torch.cuda.memory_allocated()
    assert (free1, alloc1) == (free0, alloc0), (free0, free1, alloc0, alloc1)
    assert T._workspace_info(0) == (0, 1), T._workspace_info(0)
    tb2 = b.out[:N].cpu().tolist()
assert lib().qwen_b200_device_status(0, None) == 0
ta = a.generate(first, S, N)                                   # the allocating launcher
ta2 = a.generate(ta[-1], S + N, N)
assert (tb, tb2) == (ta, ta2), (ta, tb, ta2, tb2)
assert -1 not in tb + tb2
print("FRESH-OK")
"""


def test_static_ws_fresh_process_allocates_nothing():
    r = subprocess.run([sys.executable, "-c", _FRESH, HERE], capture_output=True, text=True,
                       timeout=600, cwd=HERE)
    assert r.returncode == 0 and "FRESH-OK" in r.stdout, r.stdout[-2000:] + r.stderr[-4000:]


def test_static_ws_rejects_bad_arguments(weights_2l):
    d = CAbiDecoder(weights_2l, 2)
    d.out.fill_(-7)
    rc = _static_ws_fn()(1, 4, *d._ptrs(), d.out.data_ptr(), 2, 2046, d.max_seq, d.scale,
                         d._stream())
    code, msg = last_error()
    assert rc != 0 and rc == code and "max_seq_len" in msg, (rc, msg)
    torch.cuda.synchronize()
    assert int(d.out[0].item()) == -7  # nothing was launched
