"""Helpers for the decode parity tests: a ctypes driver of the C ABI in
include/qwen_b200.h (torch supplies only device memory and the stream) and
the comparison rules stated by the acceptance criteria.

Tolerances (floating point, fp16 decode):
* greedy token ids must match the oracle's wherever the oracle's top-1/top-2
  logit margin exceeds MARGIN = 1e-2;
* logits (final-normed hidden @ tied lm_head^T, fp32) within LOGIT_ATOL = 3e-2
  max-abs of the oracle's.
"""
from __future__ import annotations

import ctypes
import math
import os

import torch

from conftest import PKG

MARGIN = 1e-2
LOGIT_ATOL = 3e-2

_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        L = ctypes.CDLL(os.path.join(PKG, "libqwen_b200.so"))
        vp, i, f = ctypes.c_void_p, ctypes.c_int, ctypes.c_float
        L.launch_ldg_decode_direct.restype = None
        L.launch_ldg_decode_direct.argtypes = [i, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp,
                                               vp, vp, vp, vp, vp, vp, vp, vp, i, i, i, f, vp]
        L.launch_ldg_generate_nosync.restype = None
        L.launch_ldg_generate_nosync.argtypes = [i, i, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp,
                                                 vp, vp, vp, vp, vp, vp, vp, vp, vp, i, i, i, f, vp]
        L.qwen_b200_last_error.restype = i
        L.qwen_b200_last_error.argtypes = [ctypes.c_char_p, i]
        L.qwen_b200_device_status.restype = i
        L.qwen_b200_device_status.argtypes = [i, ctypes.POINTER(ctypes.c_uint64)]
        L.qwen_b200_selftest_wait_timeout.restype = i
        L.qwen_b200_selftest_wait_timeout.argtypes = [ctypes.c_longlong, vp]
        L.qwen_b200_set_wait_timeout_ns.restype = None
        L.qwen_b200_set_wait_timeout_ns.argtypes = [ctypes.c_longlong]
        L.qwen_b200_abi_version.restype = i
        _lib = L
    return _lib


def last_error() -> tuple[int, str]:
    buf = ctypes.create_string_buffer(512)
    rc = lib().qwen_b200_last_error(buf, 512)
    return rc, buf.value.decode()


def pack_table(layer_weights, device) -> torch.Tensor:
    ptrs = []
    for li in range(len(layer_weights) // 11):
        ptrs += [t.data_ptr() for t in layer_weights[li * 11: li * 11 + 11]] + [0]
    t = torch.zeros(len(ptrs) + 2, dtype=torch.int64, device=device)
    off = ((16 - t.data_ptr() % 16) % 16) // 8
    t = t[off: off + len(ptrs)]
    t.copy_(torch.tensor(ptrs, dtype=torch.int64))
    return t


class CAbiDecoder:
    """Drives launch_ldg_decode_direct / launch_ldg_generate_nosync with the
    buffers the upstream Decoder allocates (Model/Qwen06B_architecture.py:220-255)."""

    def __init__(self, weights_cpu: dict, num_layers: int, device="cuda", max_seq=2048):
        self.dev = torch.device(device)
        self.w = {k: ([t.to(self.dev) for t in v] if isinstance(v, list) else v.to(self.dev))
                  for k, v in weights_cpu.items() if k != "lm_head_weight"}
        self.w["lm_head_weight"] = self.w["embed_weight"]
        self.L = num_layers
        self.max_seq = max_seq
        self.table = pack_table(self.w["layer_weights"][: num_layers * 11], self.dev)
        f16, f32, i32 = (dict(dtype=d, device=self.dev) for d in (torch.float16, torch.float32, torch.int32))
        self.kc = torch.zeros(num_layers, 8, max_seq, 128, **f16)
        self.vc = torch.zeros_like(self.kc)
        self.hidden = torch.empty(1024, **f16)
        self.act = torch.empty(2048, **f32)
        self.res = torch.empty(1024, **f32)
        self.q = torch.empty(2048, **f16)
        self.k = torch.empty(1024, **f16)
        self.v = torch.empty(1024, **f16)
        self.attn = torch.empty(2048, **f16)
        self.inter = torch.empty(3072, **f32)
        self.norm = torch.empty(1024, **f32)
        self.bvals = torch.empty(4096, **f32)
        self.bidx = torch.empty(4096, **i32)
        self.out = torch.empty(2048, **i32)
        self.scale = 1.0 / math.sqrt(128)

    def _ptrs(self):
        w = self.w
        return [w["embed_weight"].data_ptr(), self.table.data_ptr(), w["final_norm_weight"].data_ptr(),
                w["lm_head_weight"].data_ptr(), w["cos_table"].data_ptr(), w["sin_table"].data_ptr(),
                self.kc.data_ptr(), self.vc.data_ptr(), self.hidden.data_ptr(), self.act.data_ptr(),
                self.res.data_ptr(), self.q.data_ptr(), self.k.data_ptr(), self.v.data_ptr(),
                self.attn.data_ptr(), self.inter.data_ptr(), self.norm.data_ptr(),
                self.bvals.data_ptr(), self.bidx.data_ptr()]

    def _stream(self):
        return ctypes.c_void_p(torch.cuda.current_stream(self.dev).cuda_stream)

    def step(self, token: int, pos: int) -> int:
        p = self._ptrs()
        lib().launch_ldg_decode_direct(int(token), self.out.data_ptr(), *p, self.L, int(pos),
                                       self.max_seq, self.scale, self._stream())
        rc, msg = last_error()
        if rc:
            raise RuntimeError(f"launch_ldg_decode_direct: {msg}")
        torch.cuda.synchronize(self.dev)
        return int(self.out[0].item())

    def generate(self, token: int, pos: int, n: int) -> list[int]:
        p = self._ptrs()
        lib().launch_ldg_generate_nosync(int(token), int(n), *p, self.out.data_ptr(), self.L,
                                         int(pos), self.max_seq, self.scale, self._stream())
        rc, msg = last_error()
        if rc:
            raise RuntimeError(f"launch_ldg_generate_nosync: {msg}")
        torch.cuda.synchronize(self.dev)
        return self.out[:n].cpu().tolist()


def logits_from_norm(norm_out: torch.Tensor, embed: torch.Tensor) -> torch.Tensor:
    """fp32 logits = norm_out @ E^T, on the embedding's device, TF32 off."""
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        x = norm_out.to(embed.device, torch.float32)
        return (embed.float() @ x).cpu()
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev


def check_step(ref_logits: torch.Tensor, got_logits: torch.Tensor, got_token: int,
               where: str) -> tuple[float, float]:
    """Applies the token and logit rules; returns (max-abs diff, margin)."""
    top2 = torch.topk(ref_logits, 2)
    margin = float(top2.values[0] - top2.values[1])
    ref_tok = int(top2.indices[0])
    diff = float((ref_logits - got_logits).abs().max())
    assert diff <= LOGIT_ATOL, f"{where}: logits max-abs diff {diff:.4g} > {LOGIT_ATOL}"
    if margin > MARGIN:
        assert got_token == ref_tok, (f"{where}: token {got_token} != reference {ref_tok} "
                                      f"(margin {margin:.4g})")
    return diff, margin
