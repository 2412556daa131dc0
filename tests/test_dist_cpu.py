"""Multi-rank logic on CPU: world_size-2 gloo process groups.

* DiT head sharding: each rank computes its K/V head groups (the oracle stands
  in for the GPU kernel here) and the all-gather + permute must reproduce the
  unsharded operator exactly.
* Request sharding (the decode bench): every rank owns a full batch and the
  reported value is total bytes over the max rank time.
* Failure: a rank that never joins makes the others' collective fail with an
  error inside a short timeout instead of hanging.
"""
import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _oracle_compute(q, k, v, mask, scale=None, **_):
    import oracle

    D = q.shape[-1]
    out = oracle.flash_attn_ext(q.numpy(), k.numpy(), v.numpy(), None if mask is None else mask.numpy(),
                                scale=D ** -0.5 if scale is None else scale)
    return torch.from_numpy(out)


def _worker_heads(rank, world, port, result_q):
    import sys

    sys.path[:0] = [ROOT, os.path.join(ROOT, "acestep.cpp_b200")]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    from acefa.dist import head_shard, sharded_attention

    g = torch.Generator().manual_seed(42)
    B, Hq, Hkv, S, D = 2, 8, 4, 40, 64
    q = torch.randn(B, Hq, S, D, generator=g)
    k = torch.randn(B, Hkv, S, D, generator=g).half()
    v = torch.randn(B, Hkv, S, D, generator=g).half()
    m = torch.zeros(B, 1, S, S)
    m[..., 30:] = float("-inf")
    m = m.half()
    sh = head_shard(Hq, Hkv, world, rank)
    out = sharded_attention(q[:, sh.hq0:sh.hq1].contiguous(), k[:, sh.hk0:sh.hk1].contiguous(),
                            v[:, sh.hk0:sh.hk1].contiguous(), m, world, compute=_oracle_compute)
    full = _oracle_compute(q, k, v, m)
    result_q.put((rank, float((out - full).abs().max())))
    dist.barrier()
    dist.destroy_process_group()


def test_head_sharded_dit_attention_gloo():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker_heads, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = [q.get(timeout=120) for _ in ps]
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, err in res:
        assert err == 0.0, (rank, err)


def test_head_shard_partition():
    from acefa.dist import head_shard

    for world in (1, 2, 4, 8):
        shards = [head_shard(16, 8, world, r) for r in range(world)]
        assert shards[0].hq0 == 0 and shards[-1].hq1 == 16
        for a, b in zip(shards, shards[1:]):
            assert a.hq1 == b.hq0 and a.hk1 == b.hk0
        for s in shards:
            assert (s.hq1 - s.hq0) == 2 * (s.hk1 - s.hk0)  # whole GQA groups
    with pytest.raises(ValueError):
        head_shard(16, 8, 3, 0)


def _worker_bench(rank, world, port, result_q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    # each rank reports its own elapsed time; the job's time is the max
    ms = torch.tensor([10.0 + 5.0 * rank])
    dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    result_q.put((rank, float(ms.item())))
    dist.barrier()
    dist.destroy_process_group()


def test_request_sharding_uses_max_rank_time():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker_bench, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = dict(q.get(timeout=120) for _ in ps)
    for p in ps:
        p.join(timeout=60)
    assert res == {0: 15.0, 1: 15.0}


def _worker_missing(rank, world, port, result_q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=3))
        t = torch.ones(1)
        dist.all_reduce(t)
        result_q.put((rank, "completed"))
    except Exception as e:  # the missing peer surfaces as an error, not a hang
        result_q.put((rank, type(e).__name__))


def test_missing_rank_fails_fast():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    p = ctx.Process(target=_worker_missing, args=(0, 2, port, q))  # rank 1 never starts
    p.start()
    rank, what = q.get(timeout=120)
    p.join(timeout=60)
    assert what != "completed"
