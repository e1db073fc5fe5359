"""Vocabulary-sharded tied lm_head + greedy argmax across GPUs.

No upstream counterpart: upstream evaluates the whole 151,936 x 1024 lm_head
on one GPU and reduces it with its two argmax phases
(``Tools/megakernel/megakernel.cu:1001-1144``).  Here each rank holds a
contiguous block of vocabulary rows, computes its rows' logits on the tensor
cores with a fused per-row (max, index) reduction
(``qwen_b200_lmhead_argmax``), the ranks exchange one (value, index) pair per
hidden row with an all-gather (NCCL over NVLink on GPUs), and a small kernel
picks the largest value, lowest index on ties (``qwen_b200_argmax_pick``).  A
vocabulary row's dot product does not depend on the shard that holds it, so
the result equals the single-GPU argmax bit for bit.

torch is the plumbing (device memory, the process group); the compute is in
``libqwen_b200.so``.
"""
from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from batched import lib as _batched_lib

VOCAB = 151936
HIDDEN = 1024


def _lib():
    L = _batched_lib()
    if not getattr(L, "_lmhead_ready", False):
        vp, i, ll = ctypes.c_void_p, ctypes.c_int, ctypes.c_longlong
        L.qwen_b200_lmhead_argmax_workspace.restype = ll
        L.qwen_b200_lmhead_argmax_workspace.argtypes = [i, i]
        L.qwen_b200_lmhead_argmax.restype = i
        L.qwen_b200_lmhead_argmax.argtypes = [vp, vp, i, i, ll, vp, vp, vp, vp]
        L.qwen_b200_argmax_pick.restype = i
        L.qwen_b200_argmax_pick.argtypes = [vp, vp, i, i, vp, vp]
        L._lmhead_ready = True
    return L


def _check(rc: int, what: str) -> None:
    if rc:
        buf = ctypes.create_string_buffer(512)
        _lib().qwen_b200_last_error(buf, 512)
        raise RuntimeError(f"{what} failed (code {rc}): {buf.value.decode()}")


def shard_rows(vocab: int, world: int, rank: int) -> tuple[int, int]:
    """[lo, hi) vocabulary rows of `rank`: equal blocks rounded up to a
    multiple of 16 rows (the GEMM's column granularity), the last block takes
    the remainder."""
    per = -(-vocab // world)
    per = -(-per // 16) * 16
    lo = min(vocab, rank * per)
    return lo, min(vocab, lo + per)


def exchange_pairs(val: torch.Tensor, idx: torch.Tensor, group=None) -> tuple[torch.Tensor, torch.Tensor]:
    """All-gather every rank's (fp32 value, int32 index) per row; returns
    values [world, rows] and indices [world, rows] in rank order."""
    world = dist.get_world_size(group)
    packed = torch.stack([val.contiguous().view(torch.int32), idx.contiguous()])
    parts = [torch.empty_like(packed) for _ in range(world)]
    dist.all_gather(parts, packed, group=group)
    allp = torch.stack(parts)
    return allp[:, 0].contiguous().view(torch.float32), allp[:, 1].contiguous()


class ShardedLMHead:
    """This rank's block of the tied lm_head and the cross-rank greedy pick.

    embed: the full [151936, 1024] fp16 embedding (any device; only this
    rank's rows are kept on `device`), or None with `shard` given directly.
    """

    def __init__(self, embed: torch.Tensor | None, world: int, rank: int, device=None,
                 max_rows: int = 256, group=None, shard: torch.Tensor | None = None):
        self.dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.world, self.rank, self.group = world, rank, group
        self.lo, self.hi = shard_rows(VOCAB, world, rank)
        if shard is None:
            shard = embed[self.lo:self.hi]
        if tuple(shard.shape) != (self.hi - self.lo, HIDDEN) or shard.dtype != torch.float16:
            raise ValueError(f"shard must be fp16 [{self.hi - self.lo}, {HIDDEN}]")
        self.weight = shard.to(self.dev).contiguous()
        self.max_rows = max_rows
        ws = _lib().qwen_b200_lmhead_argmax_workspace(max_rows, self.hi - self.lo)
        self.workspace = torch.empty(max(16, ws), dtype=torch.uint8, device=self.dev)
        self.val = torch.empty(max_rows, dtype=torch.float32, device=self.dev)
        self.idx = torch.empty(max_rows, dtype=torch.int32, device=self.dev)
        self.tokens = torch.empty(max_rows, dtype=torch.int32, device=self.dev)

    def _stream(self):
        return ctypes.c_void_p(torch.cuda.current_stream(self.dev).cuda_stream)

    def local(self, hidden: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        """(max logit, global index) of this rank's vocabulary rows, per row of
        hidden fp16 [rows, 1024]."""
        rows = hidden.shape[0]
        if rows > self.max_rows or hidden.dtype != torch.float16 or not hidden.is_contiguous():
            raise ValueError(f"hidden must be contiguous fp16 [<= {self.max_rows}, {HIDDEN}]")
        _check(_lib().qwen_b200_lmhead_argmax(
            hidden.data_ptr(), self.weight.data_ptr(), rows, self.hi - self.lo, self.lo,
            self.val.data_ptr(), self.idx.data_ptr(), self.workspace.data_ptr(), self._stream()),
            "lmhead_argmax")
        return self.val[:rows], self.idx[:rows]

    def pick(self, vals: torch.Tensor, idxs: torch.Tensor) -> torch.Tensor:
        world, rows = vals.shape
        out = self.tokens[:rows]
        _check(_lib().qwen_b200_argmax_pick(vals.data_ptr(), idxs.data_ptr(), world, rows,
                                            out.data_ptr(), self._stream()), "argmax_pick")
        return out

    def argmax(self, hidden: torch.Tensor) -> torch.Tensor:
        """Greedy token per row over the whole vocabulary (all ranks call it
        together; every rank returns the same tokens)."""
        val, idx = self.local(hidden)
        if self.world == 1:
            vals, idxs = val.view(1, -1), idx.view(1, -1)
        else:
            vals, idxs = exchange_pairs(val, idx, self.group)
        return self.pick(vals, idxs)
