"""Head-sharded DiT attention on 2 GPUs (skipped with fewer): the output
assembled by the NCCL all-gather and by the kernels' own P2P stores into every
rank's buffer both equal the single-GPU operator on the same inputs."""
import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
pytestmark = pytest.mark.gpu


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, result_q):
    import sys

    sys.path[:0] = [ROOT, os.path.join(ROOT, "acestep.cpp_b200")]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    import acefa
    from acefa.dist import MirroredShardedOp, ShardedOp, head_shard

    g = torch.Generator().manual_seed(42 + 1000 * 4)
    B, Hq, Hkv, S, D = 2, 16, 16, 1500, 128
    q = torch.randn(B, Hq, S, D, generator=g).to(dev)
    k = torch.randn(B, Hkv, S, D, generator=g).half().to(dev)
    v = torch.randn(B, Hkv, S, D, generator=g).half().to(dev)
    qi = torch.arange(S)[:, None]
    kj = torch.arange(S)[None, :]
    m = torch.where((qi - kj).abs() <= 128, 0.0, float("-inf")).half().reshape(1, 1, S, S).to(dev)
    sh = head_shard(Hq, Hkv, world, rank)
    op = ShardedOp(q[:, sh.hq0:sh.hq1].contiguous(), k[:, sh.hk0:sh.hk1].contiguous(),
                   v[:, sh.hk0:sh.hk1].contiguous(), m, world)
    out = op()
    full = acefa.flash_attn_ext(q, k, v, m)
    torch.cuda.synchronize()
    err_gather = float((out - full).abs().max())
    # P2P path: each kernel stores its rows into both GPUs' output buffers
    mop = MirroredShardedOp(q[:, sh.hq0:sh.hq1].contiguous(), k[:, sh.hk0:sh.hk1].contiguous(),
                            v[:, sh.hk0:sh.hk1].contiguous(), m, world)
    mop.out.fill_(float("nan"))
    torch.cuda.synchronize()
    dist.barrier()  # no peer writes into this buffer before the fill is done
    errs = []
    for _ in range(3):
        o2 = mop()
        torch.cuda.synchronize()
        errs.append(float((o2 - full).abs().max()))
        dist.barrier()  # readers done before the peers' next call overwrites
    mop.close()
    result_q.put((rank, max([err_gather] + errs)))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_head_sharded_dit_nccl_2gpu():
    ctx = mp.get_context("spawn")
    result_q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_worker, args=(r, 2, port, result_q)) for r in range(2)]
    for p in ps:
        p.start()
    res = [result_q.get(timeout=120) for _ in ps]
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, err in res:
        assert err == 0.0, (rank, err)  # same kernel, same rows: bit-identical
