"""Vocabulary-sharded lm_head + argmax (qwen0.6b_b200/lmhead_shard.py, C ABI
include/qwen_b200_batched.h) on the GPU.

* Eight shards evaluated on one GPU and picked together give the same token
  and the same winning logit as the unsharded lm_head, bit for bit (a
  vocabulary row's dot product does not depend on its shard); tokens also
  match a plain PyTorch fp32 reference wherever its top-2 margin > 1e-3.
* With two GPUs, two NCCL ranks (one process each) agree with the
  single-GPU result.
"""
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


def _rank_main(rank, world, port, q):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    try:
        from lmhead_shard import ShardedLMHead
        emb, x = _embed(), _hidden(64)
        head = ShardedLMHead(emb, world, rank, max_rows=64)
        tok = head.argmax(x).cpu().tolist()
        single = ShardedLMHead(emb, 1, 0, max_rows=64).argmax(x).cpu().tolist()
        q.put((rank, tok, single))
    except Exception as e:
        q.put((rank, "error", repr(e)))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_two_gpu_nccl_exchange():
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=300) for _ in range(world)]
    for p in procs:
        p.join(timeout=120)
    for _, tok, single in results:
        assert tok != "error", single
        assert tok == single
