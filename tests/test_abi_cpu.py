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
