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


def _base_dense(b, base, hidden):
    rows, cols = {"qkv": (3, 1), "out": (1, 1), "up": (4, 1), "down": (1, 4)}[base]
    g = torch.Generator().manual_seed(b * 16 + ("qkv", "out", "up", "down").index(base))
    return torch.randn(rows * hidden, cols * hidden, generator=g) / (cols * hidden) ** 0.5


def _weights_dense(b, name, base, qtype, n_loc, k, rows):
    w = _base_dense(b, base, k if base != "down" else k // 4)[rows]
    assert w.shape == (n_loc, k)
    return w.contiguous(), None


def _stand_in(x_slabs, packed, row_exp, qtype, n, out):
    x = torch.cat(list(x_slabs.float()), dim=1)  # [M, K] from [S, M, K/S]
    out.copy_((x @ packed.T).to(out.dtype))
    return out


def _worker(rank, world, port, q, gather):
    sys.path[:0] = [ROOT, os.path.join(ROOT, "mac-kernels-public_b200")]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from qlin.sharded import ShardedStack
        torch.manual_seed(0)
        x = torch.randn(64, 128).to(torch.float16)
        st = ShardedStack(blocks=2, tokens=64, hidden=128, chunks=2, device=torch.device("cpu"), op=_stand_in,
                          weights=_weights_dense, gather=gather)
        outs = st.forward(x)
        y = torch.cat([torch.cat(list(o.float()), dim=1) for o in outs], dim=0)  # [tokens, hidden]
        # a numpy copy pickles by value: a torch tensor would be passed as a file descriptor that
        # the parent fetches from this process, which may have exited by then
        q.put((rank, y.numpy().copy()))
    finally:
        dist.destroy_process_group()


def _dense_reference(x, gather):
    """The block chain on one device: QKV, out (reading V for attention's output, or the block input
    when every output is gathered), MLP up and down."""
    h = x
    hid = x.shape[1]
    for b in range(2):
        w = {base: _base_dense(b, base, hid) for base in ("qkv", "out", "up", "down")}
        qkv = (h.float() @ w["qkv"].T).to(torch.float16)
        attn = qkv[:, 2 * hid:] if gather == "consumed" else h
        out = (attn.float() @ w["out"].T).to(torch.float16)
        up = (out.float() @ w["up"].T).to(torch.float16)
        h = (up.float() @ w["down"].T).to(torch.float16)
    return h.float()


def _free_port():
    """A TCP port on 127.0.0.1 that nothing listens on right now (the OS picks it)."""
    import socket
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        return sk.getsockname()[1]


@pytest.mark.parametrize("gather", ["consumed", "all"])
def test_two_rank_sharded_stack_matches_dense(gather):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q, gather)) for r in range(2)]
    for p in procs:
        p.start()
    got = {r: torch.from_numpy(y) for r, y in (q.get(timeout=120) for _ in procs)}
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    torch.manual_seed(0)
    x = torch.randn(64, 128).to(torch.float16)
    ref = _dense_reference(x, gather)
    for r in (0, 1):
        assert torch.allclose(got[r], ref, rtol=2e-2, atol=2e-2), (got[r] - ref).abs().max()
    assert torch.equal(got[0], got[1])


def test_head_grouped_qkv_rows():
    """Rank r of p holds the Q, K and V rows of its own heads; the shards of all ranks together
    hold every row once."""
    from qlin.sharded import layers, shard_rows
    hid, p = 128, 4
    for gather in ("consumed", "all"):
        seen = []
        for r in range(p):
            for name, base, _, n, _, _, _, _ in layers(hid, gather, p):
                rows = shard_rows(name, base, hid, r, p)
                assert len(rows) == n // p
                if base == "qkv":
                    seen.append(rows)
        rows = torch.cat(seen)
        assert torch.equal(rows.sort().values, torch.arange(3 * hid))
    v = shard_rows("v", "qkv", hid, 1, p)
    assert torch.equal(v, torch.arange(2 * hid + 32, 2 * hid + 64))
