"""Temperature / top-k / top-p sampling on the GPU (C ABI include/qwen_b200_sample.h).

No upstream counterpart: upstream decodes greedily only (``README.md:691-692``).
The filters follow the transformers logits warpers that upstream's benchmark
uses through ``generate()`` (temperature, then top-k, then top-p); the draw is
Gumbel-max over a Philox counter stream, so a (seed, offset, row key) triple
always gives the same token.
"""
from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass

import torch

_PKG = os.path.dirname(os.path.abspath(__file__))
_lib = None


@dataclass
class SamplingParams:
    """temperature 0 (or top_k 1) is greedy; top_k 0 and top_p 1 switch a filter off."""
    temperature: float = 1.0
    top_k: int = 0
    top_p: float = 1.0
    seed: int = 0


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        path = os.path.join(_PKG, "libqwen_b200.so")
        if not os.path.exists(path):
            raise RuntimeError(f"{path} is missing: build it with qwen0.6b_b200/build.py")
        L = ctypes.CDLL(path)
        vp, i, ll, ull, f = ctypes.c_void_p, ctypes.c_int, ctypes.c_longlong, ctypes.c_ulonglong, ctypes.c_float
        L.qwen_b200_sample.restype = i
        L.qwen_b200_sample.argtypes = [vp, ll, i, i, f, i, f, ull, ull, vp, vp, vp, vp, vp]
        L.qwen_b200_sample_set_cluster.restype = None
        L.qwen_b200_sample_set_cluster.argtypes = [i]
        L.qwen_b200_last_error.restype = i
        L.qwen_b200_last_error.argtypes = [ctypes.c_char_p, i]
        _lib = L
    return _lib


def _check(rc: int, what: str) -> None:
    if rc:
        buf = ctypes.create_string_buffer(512)
        lib().qwen_b200_last_error(buf, 512)
        raise RuntimeError(f"{what} failed (code {rc}): {buf.value.decode()}")


def set_cluster_path(enable: bool) -> None:
    """Cluster-of-8-CTAs-per-row path (default) or one CTA per row (same results)."""
    lib().qwen_b200_sample_set_cluster(1 if enable else 0)


def sample(logits: torch.Tensor, params: SamplingParams, offset: int = 0,
           out: torch.Tensor | None = None, row_seq: torch.Tensor | None = None,
           row_pos: torch.Tensor | None = None, kept_min: torch.Tensor | None = None) -> torch.Tensor:
    """Tokens (device int32 [rows]) drawn from fp32 logits [rows, ld] (or [vocab]).
    Enqueued on the current stream; no host synchronisation."""
    lg = logits if logits.dim() == 2 else logits.view(1, -1)
    if not (lg.is_cuda and lg.dtype == torch.float32 and lg.stride(1) == 1):
        raise ValueError("logits must be a CUDA float32 tensor with unit column stride")
    rows, vocab = lg.shape
    out = torch.empty(rows, dtype=torch.int32, device=lg.device) if out is None else out
    for t in (row_seq, row_pos):
        if t is not None and (t.dtype != torch.int32 or t.numel() < rows or not t.is_contiguous()):
            raise ValueError("row_seq / row_pos must be contiguous int32 tensors with one entry per row")
    ptr = lambda t: t.data_ptr() if t is not None else None  # noqa: E731
    stream = torch.cuda.current_stream(lg.device).cuda_stream
    with torch.cuda.device(lg.device):
        _check(lib().qwen_b200_sample(
            lg.data_ptr(), lg.stride(0), rows, vocab, float(params.temperature), int(params.top_k),
            float(params.top_p), int(params.seed) & 0xFFFFFFFFFFFFFFFF, int(offset) & 0xFFFFFFFFFFFFFFFF,
            ptr(row_seq), ptr(row_pos), out.data_ptr(), ptr(kept_min), ctypes.c_void_p(stream)), "sample")
    return out
