"""The C-ABI library loads and exports every symbol include/*.h declares, the
extension module reports the upstream ABI version, and the launchers reject
bad arguments on the host (no GPU needed: validation precedes any CUDA call)."""
import ctypes
import glob
import os
import re

import pytest

from conftest import PKG, ROOT

LIB = os.path.join(PKG, "libqwen_b200.so")


def _declared_functions():
    names = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        text = open(h).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        text = re.sub(r"//[^\n]*", "", text)
        for m in re.finditer(r"^[A-Za-z_][\w \t\*]*?\b([A-Za-z_]\w*)\s*\([^;{]*\)\s*;", text, flags=re.M):
            if not m.group(0).lstrip().startswith(("typedef", "#")):
                names.add(m.group(1))
    return sorted(names)


def test_header_declares_the_upstream_launchers():
    names = _declared_functions()
    assert "launch_ldg_decode_direct" in names
    assert "launch_ldg_generate_nosync" in names


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(LIB)
    missing = [n for n in _declared_functions() if not hasattr(lib, n)]
    assert not missing, missing


def test_workspace_info_before_any_launch():
    """No launcher ran in this process: neither per-device workspace exists
    (host-side query, no CUDA call)."""
    lib = ctypes.CDLL(LIB)
    a, b = ctypes.c_int(-1), ctypes.c_int(-1)
    assert lib.qwen_b200_workspace_info(0, ctypes.byref(a), ctypes.byref(b)) == 0
    assert (a.value, b.value) == (0, 0)
    assert lib.qwen_b200_workspace_info(64, None, None) == -1


def test_abi_version():
    lib = ctypes.CDLL(LIB)
    assert lib.qwen_b200_abi_version() == 2
    import qwen_megakernel_C
    assert qwen_megakernel_C.abi_version() == 2


def _call_decode(lib, num_layers=28, position=0, max_seq=2048, token=1):
    vp = ctypes.c_void_p
    f = lib.launch_ldg_decode_direct
    f.restype = None
    f.argtypes = [ctypes.c_int] + [vp] * 20 + [ctypes.c_int] * 3 + [ctypes.c_float, vp]
    dummy = [vp(16 * (i + 1)) for i in range(20)]
    f(token, *dummy, num_layers, position, max_seq, 0.088, vp(0))
    buf = ctypes.create_string_buffer(512)
    lib.qwen_b200_last_error.restype = ctypes.c_int
    rc = lib.qwen_b200_last_error(buf, 512)
    return rc, buf.value.decode()


@pytest.mark.parametrize("kw,pattern", [
    (dict(num_layers=0), "num_layers"),
    (dict(position=2048), "max_seq_len"),
    (dict(position=-1), "max_seq_len"),
    (dict(token=151936), "token id"),
    (dict(token=-5), "token id"),
])
def test_launcher_rejects_bad_arguments(kw, pattern):
    rc, msg = _call_decode(ctypes.CDLL(LIB), **kw)
    assert rc != 0 and pattern in msg, (rc, msg)


def _ops_lib():
    lib = ctypes.CDLL(LIB)
    vp, i, ll = ctypes.c_void_p, ctypes.c_int, ctypes.c_longlong
    lib.qwen_b200_swiglu_forward.restype = i
    lib.qwen_b200_swiglu_forward.argtypes = [vp] * 8 + [ll, i, i, vp]
    lib.qwen_b200_rmsnorm_forward.restype = i
    lib.qwen_b200_rmsnorm_forward.argtypes = [vp] * 5 + [ll, i, ctypes.c_float, vp]
    lib.qwen_b200_swiglu_forward_down_workspace.restype = ll
    lib.qwen_b200_swiglu_forward_down_workspace.argtypes = [ll, i]
    return lib


@pytest.mark.parametrize("rows,hidden,inter,misalign,pattern", [
    (4, 1004, 3072, False, "multiples of 8"),
    (4, 1024, 3070, False, "multiples of 8"),
    (-1, 1024, 3072, False, "rows"),
    (4, 1024, 3072, True, "16-byte aligned"),
])
def test_swiglu_rejects_bad_arguments(rows, hidden, inter, misalign, pattern):
    lib = _ops_lib()
    p = [ctypes.c_void_p(4096 * (k + 1) + (8 if misalign and k == 0 else 0)) for k in range(8)]
    p[3] = p[4] = ctypes.c_void_p(0)  # no biases
    rc = lib.qwen_b200_swiglu_forward(*p, rows, hidden, inter, None)
    buf = ctypes.create_string_buffer(512)
    assert rc != 0 and lib.qwen_b200_last_error(buf, 512) == rc
    assert pattern in buf.value.decode(), buf.value


def test_ops_workspace_and_empty_calls():
    lib = _ops_lib()
    # activations (4 bytes per element) + the down projection's K slices
    # (12 bytes per element), each rounded up to 256 bytes
    assert lib.qwen_b200_swiglu_forward_down_workspace(3, 3072) == 3 * 3072 * 4 + 3 * 3072 * 12
    assert lib.qwen_b200_swiglu_forward_down_workspace(3, 40) == 512 + 1536
    # Empty inputs are a no-op (no CUDA call), even with null pointers.
    assert lib.qwen_b200_swiglu_forward(*([None] * 8), 0, 1024, 3072, None) == 0
    assert lib.qwen_b200_rmsnorm_forward(*([None] * 5), 0, 1024, 1e-6, None) == 0


def test_extension_error_messages_with_numbers():
    """An error message that formats a number must raise, not crash: the
    extensions are built with the system C++ compiler, whose runtime matches
    the libstdc++ torch loads."""
    import torch
    import swiglu_fused
    w = torch.zeros(1024, 3072, dtype=torch.float16)
    with pytest.raises(RuntimeError, match="got 2 dimensions"):
        swiglu_fused.forward(torch.zeros(2, 1024, dtype=torch.float16), w, w)
