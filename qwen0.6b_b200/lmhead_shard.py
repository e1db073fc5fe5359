"""Vocabulary-sharded tied lm_head + greedy argmax across GPUs.

No upstream counterpart: upstream evaluates the whole 151,936 x 1024 lm_head
on one GPU and reduces it with its two argmax phases
(``Tools/megakernel/megakernel.cu:1001-1144``).  Here each rank holds a
contiguous block of vocabulary rows, computes its rows' logits on the tensor
cores with a fused per-row (max, index) reduction
(``qwen_b200_lmhead_argmax``), and the ranks exchange one (value, index) pair
per hidden row.  Two exchanges:

* ``exchange="peer"`` (default on GPUs): one kernel per rank stores its pairs
  straight into every rank's receive buffer over NVLink (CUDA IPC mappings,
  plain 8-byte stores tagged with a per-call epoch) and picks the token from
  its own buffer once all ranks' pairs are in (``qwen_b200_argmax_exchange``):
  one launch, no collective library call;
* ``exchange="nccl"``: an all-gather through torch.distributed (NCCL over
  NVLink; gloo on CPU for the host-logic tests), then a pick kernel
  (``qwen_b200_argmax_pick``).

Either way the largest value wins, lowest index on ties.  A vocabulary row's
dot product does not depend on the shard that holds it, so the result equals
the single-GPU argmax bit for bit.

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
        L.qwen_b200_peer_buffer_bytes.restype = ll
        L.qwen_b200_peer_buffer_bytes.argtypes = [i, i]
        L.qwen_b200_peer_buffer_create.restype = i
        L.qwen_b200_peer_buffer_create.argtypes = [ll, ctypes.POINTER(vp), vp]
        L.qwen_b200_peer_buffer_open.restype = i
        L.qwen_b200_peer_buffer_open.argtypes = [vp, ctypes.POINTER(vp)]
        L.qwen_b200_peer_buffer_close.restype = i
        L.qwen_b200_peer_buffer_close.argtypes = [vp, i]
        L.qwen_b200_argmax_exchange.restype = i
        L.qwen_b200_argmax_exchange.argtypes = [vp, vp, vp, i, i, i, ctypes.c_uint, ll, vp, vp, vp]
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
                 max_rows: int = 256, group=None, shard: torch.Tensor | None = None,
                 exchange: str = "peer", timeout_ns: int = 2_000_000_000):
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
        if exchange not in ("peer", "nccl"):
            raise ValueError("exchange must be 'peer' or 'nccl'")
        self.exchange = exchange if (world > 1 and self.dev.type == "cuda") else "nccl"
        self.timeout_ns = int(timeout_ns)
        self.status = torch.zeros(1, dtype=torch.int64, device=self.dev)
        self._own = None
        self._peers = None
        self._epoch = 0  # peer buffers: opened by the first exchange (all ranks together)

    # --------------------------------------------------------- peer buffers
    def _open_peer_buffers(self) -> None:
        """Own receive buffer (cudaMalloc'd, cleared) and its IPC handle; the
        handles travel through torch.distributed; every peer's buffer is
        opened on this device."""
        L = _lib()
        nbytes = L.qwen_b200_peer_buffer_bytes(self.world, self.max_rows)
        handle = ctypes.create_string_buffer(64)
        own = ctypes.c_void_p()
        with torch.cuda.device(self.dev):
            _check(L.qwen_b200_peer_buffer_create(nbytes, ctypes.byref(own), handle), "peer_buffer_create")
        self._own = own
        handles = [None] * self.world
        dist.all_gather_object(handles, bytes(handle.raw), group=self.group)
        ptrs = []
        opened = []
        with torch.cuda.device(self.dev):
            for q, h in enumerate(handles):
                if q == self.rank:
                    ptrs.append(own.value)
                    continue
                p = ctypes.c_void_p()
                _check(L.qwen_b200_peer_buffer_open(ctypes.create_string_buffer(h, 64), ctypes.byref(p)),
                       "peer_buffer_open")
                ptrs.append(p.value)
                opened.append(p)
        self._peers = (ctypes.c_void_p * self.world)(*ptrs)
        self._opened = opened
        dist.barrier(group=self.group)

    def close(self) -> None:
        """Unmaps the peers' buffers, waits for every rank to do the same,
        then frees this rank's buffer (all ranks call it together)."""
        if self._own is None:
            return
        L = _lib()
        torch.cuda.synchronize(self.dev)
        with torch.cuda.device(self.dev):
            for p in self._opened:
                L.qwen_b200_peer_buffer_close(p, 1)
        dist.barrier(group=self.group)
        with torch.cuda.device(self.dev):
            L.qwen_b200_peer_buffer_close(self._own, 0)
        self._own = None
        self._peers = None

    def device_status(self) -> int:
        """0, or the packed (1 << 32 | rank << 24 | row) of an exchange wait that gave up."""
        return int(self.status.item())

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
        together, with the same number of rows; every rank returns the same
        tokens)."""
        val, idx = self.local(hidden)
        if self.world == 1:
            return self.pick(val.view(1, -1), idx.view(1, -1))
        if self.exchange == "peer":
            if self._peers is None:
                self._open_peer_buffers()
            rows = val.shape[0]
            self._epoch += 1
            out = self.tokens[:rows]
            _check(_lib().qwen_b200_argmax_exchange(
                val.data_ptr(), idx.data_ptr(), self._peers, self.world, self.rank, rows,
                self._epoch, self.timeout_ns, out.data_ptr(), self.status.data_ptr(), self._stream()),
                "argmax_exchange")
            return out
        vals, idxs = exchange_pairs(val, idx, self.group)
        return self.pick(vals, idxs)
