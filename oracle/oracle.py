"""ctypes front end of the CPU oracle (``oracle/liboracle.so``).

TEST INFRASTRUCTURE, NOT PRODUCT CODE: imported only by ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline/reference arm, as
the checker.  The C restatement it wraps is documented in ``oracle.c``; each C
function cites the upstream file:line it follows.

Parity pinning: the oracle is checked against outputs of the upstream
implementation itself (its CUDA megakernel and Tools operators, built from the
unmodified upstream sources by ``oracle/build_ref.py`` and run on a B200 by
``tests/golden/make_golden.py``), committed as fixtures in ``tests/golden/``,
and against HF ``Qwen3ForCausalLM`` in fp32 (the comparator the upstream
project itself uses, ``Model/benchmark.py:128-246``).
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")

H, I_SZ, NQ, NKV, HD, VOCAB = 1024, 3072, 16, 8, 128, 151936
QS, KVS = NQ * HD, NKV * HD

_lib = None


def build() -> str:
    """Compile liboracle.so with the committed Makefile (idempotent)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        src = os.path.join(HERE, "oracle.c")
        if not os.path.exists(LIB_PATH) or os.path.getmtime(LIB_PATH) < os.path.getmtime(src):
            build()
        L = ctypes.CDLL(LIB_PATH)
        vp, i, f = ctypes.c_void_p, ctypes.c_int, ctypes.c_float
        L.oracle_decode_step.restype = i
        L.oracle_decode_step.argtypes = [i, i, vp, vp, i, vp, vp, vp, vp, vp, vp, i, f,
                                         vp, vp, vp, vp, vp, i]
        L.oracle_lm_head_argmax.restype = None
        L.oracle_lm_head_argmax.argtypes = [vp, i, vp, i, i, vp, vp, i]
        L.oracle_rmsnorm.restype = None
        L.oracle_rmsnorm.argtypes = [vp, vp, vp, vp, vp, i, i, f]
        L.oracle_swiglu_forward.restype = None
        L.oracle_swiglu_forward.argtypes = [vp, vp, vp, vp, vp, i, i, i, vp, vp, vp, i]
        L.oracle_swiglu_forward_down.restype = None
        L.oracle_swiglu_forward_down.argtypes = [vp, vp, vp, vp, vp, vp, vp, i, i, i, vp, i]
        L.oracle_silu_half.restype = f
        L.oracle_silu_half.argtypes = [f]
        _lib = L
    return _lib


def _ptr(t: torch.Tensor | None) -> int | None:
    if t is None:
        return None
    assert t.device.type == "cpu" and t.is_contiguous()
    return t.data_ptr()


class OracleModel:
    """Stateful CPU decoder: same weights, KV layout and step semantics as the
    upstream ``Decoder.step`` (``Model/Qwen06B_architecture.py:279-333``)."""

    def __init__(self, weights: dict, num_layers: int | None = None,
                 max_seq_len: int = 2048, nthreads: int = 0):
        self.w = {k: ([t.cpu().contiguous() for t in v] if isinstance(v, list)
                      else v.cpu().contiguous()) for k, v in weights.items()}
        lw = self.w["layer_weights"]
        self.num_layers = num_layers or len(lw) // 11
        assert len(lw) >= self.num_layers * 11
        ptrs = [t.data_ptr() for t in lw[: self.num_layers * 11]]
        self._ptr_table = (ctypes.c_void_p * len(ptrs))(*ptrs)
        self.max_seq_len = max_seq_len
        self.nthreads = nthreads
        shape = (self.num_layers, NKV, max_seq_len, HD)
        self.k_cache = torch.zeros(shape, dtype=torch.float16)
        self.v_cache = torch.zeros(shape, dtype=torch.float16)
        self.position = 0
        self.attn_scale = 1.0 / float(np.sqrt(HD))

    def reset(self) -> None:
        self.position = 0
        self.k_cache.zero_()
        self.v_cache.zero_()

    def step(self, token: int, want_logits: bool = False, want_debug: bool = False) -> dict:
        hidden = torch.empty(H, dtype=torch.float16)
        norm = torch.empty(H, dtype=torch.float32)
        logits = torch.empty(VOCAB, dtype=torch.float32) if want_logits else None
        attn = torch.empty(self.num_layers * QS, dtype=torch.float16) if want_debug else None
        qkv = torch.empty(self.num_layers * (QS + 2 * KVS), dtype=torch.float16) if want_debug else None
        w = self.w
        tok = lib().oracle_decode_step(
            int(token), int(self.position), _ptr(w["embed_weight"]), self._ptr_table,
            self.num_layers, _ptr(w["final_norm_weight"]), _ptr(w["lm_head_weight"]),
            _ptr(w["cos_table"]), _ptr(w["sin_table"]), _ptr(self.k_cache), _ptr(self.v_cache),
            self.max_seq_len, self.attn_scale, _ptr(hidden), _ptr(norm), _ptr(logits),
            _ptr(attn), _ptr(qkv), self.nthreads)
        if tok < 0:
            raise ValueError(f"oracle rejected token={token} position={self.position}")
        self.position += 1
        out = dict(token=tok, hidden=hidden, norm_out=norm)
        if want_logits:
            out["logits"] = logits
        if want_debug:
            out["attn"] = attn.view(self.num_layers, QS)
            out["qkv"] = qkv.view(self.num_layers, QS + 2 * KVS)
        return out

    def generate(self, first_token: int, num_steps: int) -> list[int]:
        """Greedy tokens, as ``generate_nosync`` returns them (megakernel.cu:1247-1314)."""
        toks, t = [], first_token
        for _ in range(num_steps):
            t = self.step(t)["token"]
            toks.append(t)
        return toks


def lm_head_argmax(x: torch.Tensor, embed: torch.Tensor, row0: int = 0, row1: int | None = None,
                   nthreads: int = 0) -> tuple[torch.Tensor, torch.Tensor]:
    x = x.to(torch.float16).contiguous().cpu()
    row1 = embed.shape[0] if row1 is None else row1
    b = x.shape[0]
    val = torch.empty(b, dtype=torch.float32)
    idx = torch.empty(b, dtype=torch.int32)
    lib().oracle_lm_head_argmax(_ptr(x), b, _ptr(embed.contiguous().cpu()), row0, row1,
                                _ptr(val), _ptr(idx), nthreads)
    return val, idx


def rmsnorm_forward(x: torch.Tensor, w: torch.Tensor, eps: float,
                    residual: torch.Tensor | None = None):
    """``rmsnorm.forward`` (Tools/rmsnorm/rmsnorm.cu:123-133); updates residual in place."""
    x = x.contiguous()
    rows, cols = x.numel() // x.shape[-1], x.shape[-1]
    out = torch.empty_like(x)
    rms = torch.empty(rows, dtype=torch.float32)
    lib().oracle_rmsnorm(_ptr(x), _ptr(w.contiguous()), _ptr(residual), _ptr(out), _ptr(rms),
                         rows, cols, float(eps))
    return out, rms


def _opt(t: torch.Tensor | None) -> torch.Tensor | None:
    return None if t is None else t.cpu().contiguous()


def swiglu_forward(x: torch.Tensor, wg: torch.Tensor, wu: torch.Tensor,
                   b_gate: torch.Tensor | None = None, b_up: torch.Tensor | None = None,
                   nthreads: int = 0):
    """``swiglu_fused.forward`` (swiglu.cu:316-361): x [B,S,H], W [H,I], biases [I] or None."""
    b, s, h = x.shape
    inter = wg.shape[1]
    out = torch.empty(b, s, inter, dtype=torch.float16)
    gc, uc = torch.empty_like(out), torch.empty_like(out)
    bg, bu = _opt(b_gate), _opt(b_up)
    lib().oracle_swiglu_forward(_ptr(x.contiguous()), _ptr(wg.contiguous()), _ptr(wu.contiguous()),
                                _ptr(bg), _ptr(bu), b * s, h, inter, _ptr(out), _ptr(gc), _ptr(uc),
                                nthreads)
    return out, gc, uc


def swiglu_forward_down(x: torch.Tensor, wg: torch.Tensor, wu: torch.Tensor, wd: torch.Tensor,
                        b_gate: torch.Tensor | None = None, b_up: torch.Tensor | None = None,
                        b_down: torch.Tensor | None = None, nthreads: int = 0) -> torch.Tensor:
    """``swiglu_fused.forward_down`` (swiglu.cu:413-464): Wg, Wu [H,I], Wd [I,H], biases or None."""
    b, s, h = x.shape
    inter = wg.shape[1]
    out = torch.empty(b, s, h, dtype=torch.float16)
    bg, bu, bd = _opt(b_gate), _opt(b_up), _opt(b_down)
    lib().oracle_swiglu_forward_down(_ptr(x.contiguous()), _ptr(wg.contiguous()),
                                     _ptr(wu.contiguous()), _ptr(wd.contiguous()), _ptr(bg),
                                     _ptr(bu), _ptr(bd), b * s, h, inter, _ptr(out), nthreads)
    return out
