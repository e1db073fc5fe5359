"""Host logic of the vocabulary-sharded lm_head (qwen0.6b_b200/lmhead_shard.py)
on CPU: the shard boundaries, and the pair exchange over a real process group
(gloo, world size 2) followed by the pick rule, against the unsharded argmax.
The per-shard (max, index) pairs are produced here by torch on CPU; on GPUs
the kernel produces them (tests/test_lmhead_gpu.py)."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from lmhead_shard import VOCAB, exchange_pairs, shard_rows


def test_shard_rows_cover_the_vocabulary():
    for world in (1, 2, 3, 4, 8):
        spans = [shard_rows(VOCAB, world, r) for r in range(world)]
        assert spans[0][0] == 0 and spans[-1][1] == VOCAB
        for (a, b), (c, _) in zip(spans, spans[1:]):
            assert b == c
        assert all((hi - lo) % 16 == 0 and hi > lo for lo, hi in spans)
    assert shard_rows(VOCAB, 8, 3) == (3 * 18992, 4 * 18992)


def pick(vals, idxs):
    """Reference rule: largest value, lowest index among equal values."""
    best_v, best_i = vals[0].clone(), idxs[0].clone()
    for w in range(1, vals.shape[0]):
        v, i = vals[w], idxs[w]
        take = (v > best_v) | ((v == best_v) & (i < best_i))
        best_v = torch.where(take, v, best_v)
        best_i = torch.where(take, i, best_i)
    return best_i


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        _rank_body(rank, world, q)
    except Exception as e:  # reported to the parent instead of a silent exit
        q.put((rank, "error", repr(e)))
    finally:
        dist.destroy_process_group()


def _rank_body(rank, world, q):
    vocab, rows = 64 * world, 5
    g = torch.Generator().manual_seed(0)
    logits = torch.randn(rows, vocab, generator=g)
    # A tie across the two shards in row 0: the lower index must win.
    logits[0, 3] = logits[0, 64 + 7] = 100.0
    lo, hi = shard_rows(vocab, world, rank)
    local = logits[:, lo:hi]
    val = local.max(dim=1).values.float()
    # max() may return any index of equal values: take the lowest.
    idx = torch.tensor([int((local[r] == val[r]).nonzero()[0]) for r in range(rows)], dtype=torch.int32) + lo
    vals, idxs = exchange_pairs(val, idx)
    got = pick(vals, idxs)
    want = [int((logits[r] == logits[r].max()).nonzero()[0]) for r in range(rows)]
    q.put((rank, got.tolist(), want))


def test_exchange_and_pick_world2_gloo():
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for _, got, want in results:
        assert got != "error", want
        assert got == want
        assert got[0] == 3
