"""The N-sharded stack's host plumbing on world_size-2 gloo CPU ranks: weight row shards, chunked
all-gathers into column slabs and the slab layout the next linear reads.  A dense fp32 stand-in
replaces the shard GEMM (this checks the distributed bookkeeping, not the kernel)."""
import os
import sys

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _weights_dense(b, name, qtype, n, k, r, p):
    g = torch.Generator().manual_seed(b * 16 + ("qkv", "out", "up", "down").index(name))
    w = torch.randn(n, k, generator=g) / k ** 0.5
    n_loc = n // p
    return w[r * n_loc:(r + 1) * n_loc].contiguous(), None


def _stand_in(x_slabs, packed, row_exp, qtype, n, out):
    x = torch.cat(list(x_slabs.float()), dim=1)  # [M, K] from [S, M, K/S]
    out.copy_((x @ packed.T).to(out.dtype))
    return out


def _worker(rank, world, port, q):
    sys.path[:0] = [ROOT, os.path.join(ROOT, "mac-kernels-public_b200")]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from qlin.sharded import ShardedStack
        torch.manual_seed(0)
        x = torch.randn(64, 128).to(torch.float16)
        st = ShardedStack(blocks=2, tokens=64, hidden=128, chunks=2, device=torch.device("cpu"), op=_stand_in,
                          weights=_weights_dense)
        outs = st.forward(x)
        y = torch.cat([torch.cat(list(o.float()), dim=1) for o in outs], dim=0)  # [tokens, hidden]
        q.put((rank, y))
    finally:
        dist.destroy_process_group()


def _dense_reference(x):
    from qlin.sharded import layers
    h = x
    for b in range(2):
        outs = {}
        for name, qtype, n, k in layers(128):
            w, _ = _weights_dense(b, name, qtype, n, k, 0, 1)
            src = {"qkv": h, "out": h, "up": outs.get("out"), "down": outs.get("up")}[name]
            outs[name] = (src.float() @ w.T).to(torch.float16)
        h = outs["down"]
    return h.float()


def test_two_rank_sharded_stack_matches_dense():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29500 + os.getpid() % 1000
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    torch.manual_seed(0)
    x = torch.randn(64, 128).to(torch.float16)
    ref = _dense_reference(x)
    for r in (0, 1):
        assert torch.allclose(got[r], ref, rtol=2e-2, atol=2e-2), (got[r] - ref).abs().max()
    assert torch.equal(got[0], got[1])
