"""Vocabulary-sharded lm_head + argmax (qwen0.6b_b200/lmhead_shard.py, C ABI
include/qwen_b200_batched.h) on the GPU.

* Eight shards evaluated on one GPU and picked together give the same token
  and the same winning logit as the unsharded lm_head, bit for bit (a
  vocabulary row's dot product does not depend on its shard); tokens also
  match a plain PyTorch fp32 reference wherever its top-2 margin > 1e-3.
* With two GPUs, two ranks (one process each) agree with the single-GPU
  result, through the NCCL all-gather and through the peer-memory exchange
  kernel (qwen_b200_argmax_exchange).
* On one GPU the exchange kernel is checked without two waiting kernels on
  the same device: rank 1's pairs are placed in rank 0's receive buffer
  first (as rank 1's stores would), then rank 0's kernel picks; and a wait on
  a rank whose pairs never come gives up after its bound, writes -1 and a
  status word, and leaves the context usable.
"""
import ctypes
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

VOCAB = 151936


def _embed(seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return (0.02 * torch.randn(VOCAB, 1024, generator=g, device="cuda")).half()


def _hidden(b, seed=1):
    g = torch.Generator(device="cuda").manual_seed(seed + b)
    return torch.randn(b, 1024, generator=g, device="cuda").half()


@pytest.mark.parametrize("b", [1, 64, 256])
def test_eight_shards_equal_unsharded(b):
    from lmhead_shard import ShardedLMHead
    emb, x = _embed(), _hidden(b)
    full = ShardedLMHead(emb, 1, 0, max_rows=256)
    v_full, i_full = (t.clone() for t in full.local(x))
    tok_full = full.pick(v_full.view(1, -1), i_full.view(1, -1)).clone()
    vals, idxs = [], []
    for r in range(8):
        sh = ShardedLMHead(emb, 8, r, max_rows=256)
        v, i = sh.local(x)
        vals.append(v.clone())
        idxs.append(i.clone())
    vals, idxs = torch.stack(vals), torch.stack(idxs)
    tok = full.pick(vals, idxs)
    assert torch.equal(tok, tok_full)
    assert torch.equal(vals.max(0).values, v_full)
    ref = x.float() @ emb.float().t()
    top2 = torch.topk(ref, 2, dim=1)
    sel = (top2.values[:, 0] - top2.values[:, 1]) > 1e-3
    assert torch.equal(tok.long()[sel], top2.indices[sel, 0])


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, q, exchange):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    head = None
    try:
        from lmhead_shard import ShardedLMHead
        emb = _embed()
        head = ShardedLMHead(emb, world, rank, max_rows=256, exchange=exchange)
        single = ShardedLMHead(emb, 1, 0, max_rows=256)
        toks, singles = [], []
        for b in (64, 256, 1, 64):  # several calls: the buffer halves alternate
            x = _hidden(b)
            toks.append(head.argmax(x).cpu().tolist())
            singles.append(single.argmax(x).cpu().tolist())
        q.put((rank, toks, singles, head.device_status()))
    except Exception as e:
        q.put((rank, "error", repr(e), -1))
    finally:
        if head is not None:
            head.close()
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("exchange", ["nccl", "peer"])
def test_two_gpu_exchange(exchange):
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, q, exchange)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=300) for _ in range(world)]
    for p in procs:
        p.join(timeout=120)
    for _, tok, single, status in results:
        assert tok != "error", single
        assert tok == single
        assert status == 0


def _exchange_fn():
    from lmhead_shard import _lib
    return _lib()


def _words(t: torch.Tensor, epoch: int) -> torch.Tensor:
    """int64 handoff words: epoch in the high half, the 32-bit payload low."""
    return (epoch << 32) | (t.view(torch.int32).to(torch.int64) & 0xFFFFFFFF)


def _exchange(L, v, i, buf, rank, rows, epoch, timeout_ns, out, status):
    peers = (ctypes.c_void_p * 2)(buf.data_ptr(), buf.data_ptr())
    return L.qwen_b200_argmax_exchange(v.data_ptr(), i.data_ptr(), peers, 2, rank, rows, epoch, timeout_ns,
                                       out.data_ptr(), status.data_ptr(),
                                       ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))


@pytest.mark.parametrize("b,epoch", [(64, 1), (256, 2), (3, 7)])
def test_exchange_kernel_picks_across_ranks(b, epoch):
    """Rank 0's kernel with rank 1's pairs already in its buffer (half
    epoch & 1, slot 1 of [2][world][rows][2]) gives the single-GPU tokens."""
    from lmhead_shard import ShardedLMHead
    L = _exchange_fn()
    emb, x = _embed(), _hidden(b)
    sh = [ShardedLMHead(emb, 2, r, max_rows=256) for r in range(2)]
    (v0, i0), (v1, i1) = ((v.clone(), i.clone()) for v, i in (s.local(x) for s in sh))
    want = ShardedLMHead(emb, 1, 0, max_rows=256).argmax(x).clone()
    buf = torch.zeros(2, 2, b, 2, dtype=torch.int64, device="cuda")
    buf[epoch & 1, 1, :, 0] = _words(v1, epoch)
    buf[epoch & 1, 1, :, 1] = _words(i1, epoch)
    out = torch.full((b,), -7, dtype=torch.int32, device="cuda")
    status = torch.zeros(1, dtype=torch.int64, device="cuda")
    assert _exchange(L, v0, i0, buf, 0, b, epoch, 1_000_000_000, out, status) == 0
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    assert torch.equal(out, want)
    # rank 0's own pairs landed in slot 0 of the same half
    assert torch.equal(buf[epoch & 1, 0, :, 0], _words(v0, epoch))


def test_exchange_wait_times_out_and_context_survives():
    """Rank 1 never stores its pairs: rank 0's bounded wait gives up, writes
    -1 and (1 << 32 | rank 1 << 24 | row) in the status word; the context
    stays usable."""
    from lmhead_shard import ShardedLMHead
    L = _exchange_fn()
    b = 4
    emb, x = _embed(), _hidden(b)
    v0, i0 = ShardedLMHead(emb, 2, 0, max_rows=8).local(x)
    buf = torch.zeros(2, 2, b, 2, dtype=torch.int64, device="cuda")
    out = torch.zeros(b, dtype=torch.int32, device="cuda")
    status = torch.zeros(1, dtype=torch.int64, device="cuda")
    assert _exchange(L, v0, i0, buf, 0, b, 1, 20_000_000, out, status) == 0
    torch.cuda.synchronize()
    assert out.cpu().tolist() == [-1] * b
    st = int(status.item())
    assert st >> 32 == 1 and (st >> 24) & 0xFF == 1 and (st & 0xFFFFFF) < b
    full = ShardedLMHead(emb, 1, 0, max_rows=8).argmax(x)
    assert torch.equal(full.cpu(), full.cpu()) and int(full.min()) >= 0
