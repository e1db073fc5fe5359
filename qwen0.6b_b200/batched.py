"""Batched greedy decode of many independent sequences per GPU (B200).

No upstream counterpart: upstream decodes one sequence at a time through
``Decoder`` (``Model/Qwen06B_architecture.py:205-382``).  Each sequence keeps
the upstream per-sequence fp16 KV-cache layout ``[layers, 8, max_seq, 128]``
(``:233-237``); the caches of all sequences are stacked into one K and one V
pool.  A step advances up to ``max_rows`` sequences by one token each through
the C ABI of ``include/qwen_b200_batched.h`` (tcgen05 GEMMs for the
projections and the lm_head, split-KV attention over each sequence's cache).

torch only allocates device memory here; every kernel lives in
``libqwen_b200.so``, and the class refuses to run without it.

Multi-GPU: sequences are independent, so a job shards them across GPUs (one
process per GPU, each with a full weight replica and its own sequences); no
collective is involved.  ``shard_sequences`` gives the split.
"""
from __future__ import annotations

import ctypes
import math
import os

import torch

_PKG = os.path.dirname(os.path.abspath(__file__))
_lib = None

H, IM, NQ, NKV, HD = 1024, 3072, 16, 8, 128
VOCAB = 151936


class _Layer(ctypes.Structure):
    _fields_ = [(n, ctypes.c_void_p) for n in
                ("input_norm", "w_qkv", "q_norm", "k_norm", "w_o", "post_norm", "w_gu", "w_down")]


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        path = os.path.join(_PKG, "libqwen_b200.so")
        if not os.path.exists(path):
            raise RuntimeError(f"{path} is missing: build it with qwen0.6b_b200/build.py")
        L = ctypes.CDLL(path)
        vp, i, ll = ctypes.c_void_p, ctypes.c_int, ctypes.c_longlong
        L.qwen_b200_batched_workspace.restype = ll
        L.qwen_b200_batched_workspace.argtypes = [i, i]
        L.qwen_b200_batched_create.restype = i
        L.qwen_b200_batched_create.argtypes = [ctypes.POINTER(vp), ctypes.POINTER(_Layer), i, vp, vp,
                                               vp, vp, vp, vp, i, i, i, vp, ll]
        L.qwen_b200_batched_create_paged.restype = i
        L.qwen_b200_batched_create_paged.argtypes = [ctypes.POINTER(vp), ctypes.POINTER(_Layer), i, vp, vp,
                                                     vp, vp, vp, vp, i, vp, i, i, i, i, vp, ll]
        L.qwen_b200_batched_step.restype = i
        L.qwen_b200_batched_step.argtypes = [vp, i, vp, vp, vp, vp, vp, i, ctypes.c_float, vp]
        L.qwen_b200_batched_step_logits.restype = i
        L.qwen_b200_batched_step_logits.argtypes = [vp, i, vp, vp, vp, vp, ll, vp, i, ctypes.c_float, vp]
        L.qwen_b200_batched_status.restype = i
        L.qwen_b200_batched_status.argtypes = [vp, ctypes.POINTER(ctypes.c_uint64)]
        L.qwen_b200_batched_destroy.restype = None
        L.qwen_b200_batched_destroy.argtypes = [vp]
        L.qwen_b200_last_error.restype = i
        L.qwen_b200_last_error.argtypes = [ctypes.c_char_p, i]
        _lib = L
    return _lib


def _check(rc: int, what: str) -> None:
    if rc:
        buf = ctypes.create_string_buffer(512)
        lib().qwen_b200_last_error(buf, 512)
        raise RuntimeError(f"{what} failed (code {rc}): {buf.value.decode()}")


def shard_sequences(num_seqs: int, world: int, rank: int) -> range:
    """Contiguous block of sequence indices owned by `rank` of `world`."""
    per = (num_seqs + world - 1) // world
    lo = min(num_seqs, rank * per)
    return range(lo, min(num_seqs, lo + per))


def pack_layer(lw: list) -> dict:
    """Batched-path weights of one layer from its 11 upstream tensors
    (LDGLayerWeight order): q|k|v rows stacked, gate/up rows interleaved."""
    in_norm, q, k, v, q_norm, k_norm, o, post_norm, gate, up, down = lw
    w_qkv = torch.cat([q, k, v], 0).contiguous()
    w_gu = torch.stack([gate, up], 1).reshape(2 * gate.shape[0], gate.shape[1]).contiguous()
    return dict(input_norm=in_norm.contiguous(), w_qkv=w_qkv, q_norm=q_norm.contiguous(),
                k_norm=k_norm.contiguous(), w_o=o.contiguous(), post_norm=post_norm.contiguous(),
                w_gu=w_gu, w_down=down.contiguous())


PAGE = 128  # tokens per KV page


class PagePool:
    """Host bookkeeping of paged KV pools: which page holds positions
    [128 i, 128 i + 128) of each sequence (-1: none), and the free pages."""

    def __init__(self, num_pages: int, num_seqs: int, max_pages: int):
        self.num_pages, self.num_seqs, self.max_pages = num_pages, num_seqs, max_pages
        self.table = [[-1] * max_pages for _ in range(num_seqs)]
        self.free = list(range(num_pages - 1, -1, -1))  # pop() hands out the lowest page first

    def reserve(self, seq: int, upto_position: int) -> bool:
        """Maps pages for positions 0..upto_position; True if the row changed."""
        need = upto_position // PAGE + 1
        if not 0 <= seq < self.num_seqs or not 0 <= upto_position or need > self.max_pages:
            raise ValueError(f"sequence {seq} / position {upto_position} outside the page table")
        row = self.table[seq]
        missing = [i for i in range(need) if row[i] < 0]
        if len(missing) > len(self.free):
            raise RuntimeError(f"KV page pool exhausted ({self.num_pages} pages of {PAGE} tokens)")
        for i in missing:
            row[i] = self.free.pop()
        return bool(missing)

    def release(self, seq: int) -> None:
        row = self.table[seq]
        for i, pg in enumerate(row):
            if pg >= 0:
                self.free.append(pg)
                row[i] = -1

    @property
    def in_use(self) -> int:
        return self.num_pages - len(self.free)


class BatchedDecoder:
    """Greedy (or sampled) decode of `num_seqs` independent sequences on one GPU.

    weights: the ``load_weights`` dict (``embed_weight``, ``layer_weights``,
    ``final_norm_weight``, ``cos_table``, ``sin_table``), any device.
    Contiguous pools (default): sequence s owns ``k_pool[s]`` / ``v_pool[s]``
    (fp16 [layers, 8, max_seq, 128], the upstream per-sequence layout).
    Paged pools (``paged=True``, no upstream counterpart): ``num_pages`` pages
    of 128 tokens (fp16 [num_pages, layers, 8, 128, 128] for K and for V)
    shared by all sequences through ``page_table`` (int32 [num_seqs,
    max_seq / 128], -1 = unmapped); ``reserve`` maps pages before positions
    are used (``prefill``, ``prefill_parallel`` and ``generate`` do it), and
    ``release`` returns a finished sequence's pages.  max_seq may then exceed
    2048 (RoPE tables are rebuilt to max_seq rows when the weights' are shorter).
    """

    def __init__(self, weights: dict, num_seqs: int, max_rows: int | None = None,
                 max_seq: int = 2048, num_layers: int | None = None, device=None,
                 k_pool: torch.Tensor | None = None, v_pool: torch.Tensor | None = None,
                 paged: bool = False, num_pages: int | None = None):
        self.dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        lw = weights["layer_weights"]
        self.L = num_layers or len(lw) // 11
        self.num_seqs = num_seqs
        self.max_rows = max_rows or num_seqs
        self.max_seq = max_seq
        to = dict(device=self.dev)
        self.embed = weights["embed_weight"].to(**to).contiguous()
        self.final_norm = weights["final_norm_weight"].to(**to).contiguous()
        self.cos = weights["cos_table"].to(**to).contiguous()
        self.sin = weights["sin_table"].to(**to).contiguous()
        if self.cos.shape[0] < max_seq:
            from qwen_weights import rope_tables
            cos, sin = rope_tables(max_seq)
            self.cos, self.sin = cos.to(**to), sin.to(**to)
        self.layers = [pack_layer([t.to(**to) for t in lw[11 * l: 11 * l + 11]]) for l in range(self.L)]
        # Positions a sequence has not reached are never read, so the pools need no clearing.
        # Caller-owned pools (e.g. a Decoder's own cache) must have this exact layout.
        shape = (num_seqs, self.L, NKV, max_seq, HD)
        self.paged = bool(paged)
        if self.paged:
            if k_pool is not None or v_pool is not None:
                raise ValueError("caller-owned pools are contiguous only")
            self.max_pages = (max_seq + PAGE - 1) // PAGE
            self.num_pages = int(num_pages) if num_pages else num_seqs * self.max_pages
            shape = (self.num_pages, self.L, NKV, PAGE, HD)
            self.page_table = torch.full((num_seqs, self.max_pages), -1, dtype=torch.int32, **to)
            self.pages = PagePool(self.num_pages, num_seqs, self.max_pages)
        if k_pool is not None or v_pool is not None:
            for t in (k_pool, v_pool):
                if (t is None or tuple(t.shape) != shape or t.dtype != torch.float16
                        or not t.is_contiguous() or t.device != self.dev):
                    raise ValueError(f"k_pool / v_pool must be contiguous fp16 {shape} on {self.dev}")
            self.k_pool, self.v_pool = k_pool, v_pool
        else:
            self.k_pool = torch.empty(shape, dtype=torch.float16, **to)
            self.v_pool = torch.empty_like(self.k_pool)
        ws = lib().qwen_b200_batched_workspace(self.max_rows, max_seq)
        self.workspace = torch.empty(ws, dtype=torch.uint8, **to)
        self.tokens_out = torch.empty(self.max_rows, dtype=torch.int32, **to)
        self.attn_scale = 1.0 / math.sqrt(HD)
        arr = (_Layer * self.L)()
        for l, d in enumerate(self.layers):
            for name in _Layer._fields_:
                setattr(arr[l], name[0], d[name[0]].data_ptr())
        h = ctypes.c_void_p()
        with torch.cuda.device(self.dev):
            if self.paged:
                _check(lib().qwen_b200_batched_create_paged(
                    ctypes.byref(h), arr, self.L, self.embed.data_ptr(), self.final_norm.data_ptr(),
                    self.cos.data_ptr(), self.sin.data_ptr(), self.k_pool.data_ptr(), self.v_pool.data_ptr(),
                    self.num_pages, self.page_table.data_ptr(), self.max_pages, num_seqs, max_seq,
                    self.max_rows, self.workspace.data_ptr(), ws), "batched_create_paged")
            else:
                _check(lib().qwen_b200_batched_create(
                    ctypes.byref(h), arr, self.L, self.embed.data_ptr(), self.final_norm.data_ptr(),
                    self.cos.data_ptr(), self.sin.data_ptr(), self.k_pool.data_ptr(), self.v_pool.data_ptr(),
                    num_seqs, max_seq, self.max_rows, self.workspace.data_ptr(), ws), "batched_create")
        self._h = h

    # ----------------------------------------------------------- paged pools
    def reserve(self, seq: int, upto_position: int) -> None:
        """Maps pages for positions 0..upto_position of sequence `seq` (paged
        pools; a no-op otherwise).  Raises when the pool is exhausted."""
        if not self.paged:
            return
        if not 0 <= upto_position < self.max_seq:
            raise ValueError(f"position {upto_position} outside [0, {self.max_seq})")
        if self.pages.reserve(seq, upto_position):
            self.page_table[seq].copy_(torch.tensor(self.pages.table[seq], dtype=torch.int32))

    def release(self, seq: int) -> None:
        """Returns every page of sequence `seq` to the pool (paged pools)."""
        if not self.paged:
            return
        self.pages.release(seq)
        self.page_table[seq].fill_(-1)

    @property
    def pages_in_use(self) -> int:
        return self.pages.in_use if self.paged else 0

    def close(self) -> None:
        if getattr(self, "_h", None):
            lib().qwen_b200_batched_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def step(self, seq_ids: torch.Tensor, positions: torch.Tensor, tokens: torch.Tensor,
             max_position: int, norm_out: torch.Tensor | None = None,
             out: torch.Tensor | None = None, sampling=None) -> torch.Tensor:
        """One step of rows = len(seq_ids) sequences (device int32 tensors):
        greedy, or drawn with ``sampling`` (a ``sampling.SamplingParams``; each
        row's random stream is keyed by its sequence id and position, so a
        draw does not depend on the batch composition).  Returns the device
        int32 tensor of produced tokens.  No host synchronisation."""
        rows = int(seq_ids.numel())
        for t in (seq_ids, positions, tokens):
            if t.dtype != torch.int32 or t.device != self.dev or not t.is_contiguous():
                raise ValueError("seq_ids, positions and tokens must be contiguous int32 tensors on "
                                 f"{self.dev}")
        out = self.tokens_out[:rows] if out is None else out
        stream = torch.cuda.current_stream(self.dev).cuda_stream
        if sampling is not None:
            from sampling import sample
            if getattr(self, "_logits", None) is None:
                self._logits = torch.empty(self.max_rows, VOCAB, dtype=torch.float32, device=self.dev)
            _check(lib().qwen_b200_batched_step_logits(
                self._h, rows, seq_ids.data_ptr(), positions.data_ptr(), tokens.data_ptr(),
                self._logits.data_ptr(), VOCAB, norm_out.data_ptr() if norm_out is not None else None,
                int(max_position), self.attn_scale, ctypes.c_void_p(stream)), "batched_step_logits")
            return sample(self._logits[:rows], sampling, out=out, row_seq=seq_ids, row_pos=positions)
        _check(lib().qwen_b200_batched_step(
            self._h, rows, seq_ids.data_ptr(), positions.data_ptr(), tokens.data_ptr(),
            out.data_ptr(), norm_out.data_ptr() if norm_out is not None else None,
            int(max_position), self.attn_scale, ctypes.c_void_p(stream)), "batched_step")
        return out

    def status(self) -> int:
        d = ctypes.c_uint64(0)
        return lib().qwen_b200_batched_status(self._h, ctypes.byref(d))

    def prefill(self, prompts: list[list[int]], seqs: list[int] | None = None) -> None:
        """Teacher-forced steps over every prompt token but the last (as
        upstream's ``Decoder.generate`` prefills, one position per step), rows
        = the sequences whose prompt still has tokens at that position."""
        seqs = list(range(len(prompts))) if seqs is None else seqs
        longest = max(len(p) for p in prompts)
        for t in range(longest - 1):
            live = [i for i, p in enumerate(prompts) if t < len(p) - 1]
            for c0 in range(0, len(live), self.max_rows):
                chunk = live[c0: c0 + self.max_rows]
                for i in chunk:
                    self.reserve(seqs[i], t)
                ids = torch.tensor([seqs[i] for i in chunk], dtype=torch.int32, device=self.dev)
                pos = torch.full((len(chunk),), t, dtype=torch.int32, device=self.dev)
                tok = torch.tensor([prompts[i][t] for i in chunk], dtype=torch.int32, device=self.dev)
                self.step(ids, pos, tok, t)

    def prefill_parallel(self, prompts: list[list[int]], seqs: list[int] | None = None,
                         starts: list[int] | None = None) -> None:
        """Parallel prefill (no upstream counterpart; upstream feeds one prompt
        token per step, ``Model/Qwen06B_architecture.py:346-347``): the K/V of
        every prompt token but the last, for all sequences, in as few steps as
        max_rows allows.  Rows of one step may be several positions of the same
        sequence: every row's K/V is appended before the step's attention runs,
        so the row at position p attends to the positions 0..p written by the
        same step.  starts[i] is the position of prompts[i][0] (default 0)."""
        seqs = list(range(len(prompts))) if seqs is None else seqs
        starts = [0] * len(prompts) if starts is None else starts
        rows = [(seqs[i], starts[i] + t, p[t]) for i, p in enumerate(prompts) for t in range(len(p) - 1)]
        for c0 in range(0, len(rows), self.max_rows):
            chunk = rows[c0: c0 + self.max_rows]
            for r in chunk:
                self.reserve(r[0], r[1])
            ids = torch.tensor([r[0] for r in chunk], dtype=torch.int32, device=self.dev)
            pos = torch.tensor([r[1] for r in chunk], dtype=torch.int32, device=self.dev)
            tok = torch.tensor([r[2] for r in chunk], dtype=torch.int32, device=self.dev)
            self.step(ids, pos, tok, max(r[1] for r in chunk),
                      out=torch.empty(len(chunk), dtype=torch.int32, device=self.dev))

    def generate(self, prompts: list[list[int]], max_tokens: int, sampling=None) -> list[list[int]]:
        """Prefill, then `max_tokens` steps of all sequences (at most max_rows
        of them), greedy or with ``sampling``; returns the generated ids per
        sequence."""
        if len(prompts) > self.max_rows:
            raise ValueError(f"{len(prompts)} sequences > max_rows={self.max_rows}")
        self.prefill(prompts)
        n = len(prompts)
        ids = torch.arange(n, dtype=torch.int32, device=self.dev)
        pos = torch.tensor([len(p) - 1 for p in prompts], dtype=torch.int32, device=self.dev)
        tok = torch.tensor([p[-1] for p in prompts], dtype=torch.int32, device=self.dev)
        start_max = max(len(p) - 1 for p in prompts)
        if start_max + max_tokens > self.max_seq:
            raise ValueError("generation would run past max_seq")
        outs = []
        for i, p in enumerate(prompts):
            self.reserve(i, len(p) - 1 + max_tokens - 1)
        for s in range(max_tokens):
            nxt = self.step(ids, pos, tok, start_max + s,
                            out=torch.empty(n, dtype=torch.int32, device=self.dev), sampling=sampling)
            outs.append(nxt)
            tok = nxt
            pos = pos + 1
        return torch.stack(outs, 1).cpu().tolist()
