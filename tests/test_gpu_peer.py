"""GPU checks of the sharded linear fused with its all-gather (qlin_gguf_linear_allgather).

One GPU: two "ranks" whose gathered buffers and flag pads are both local, with the other rank's
flag preset so no wait is pending: the epilogue must store identical tiles into both buffers
(equal to the unfused slab linear, bit for bit), leave other slabs alone, and advance the pads.
A wait on a flag that nothing sets must run out after its limit with QLIN_ETIMEOUT, leave the
output untouched, and keep the context usable.
Two or more GPUs (skipped otherwise): the peer-transport stack equals the NCCL-transport stack.
"""
import os

import numpy as np
import pytest
import torch

from oracle import qlin_oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def qlin():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    import qlin as q
    return q


def _pads(world):
    pads = torch.zeros(world, 16, dtype=torch.int32, device="cuda")  # 64-byte PeerSync per rank
    return pads, [pads[r].data_ptr() for r in range(world)]


def _weights(qlin, qtype, n, k, seed):
    raw = torch.from_numpy(O.random_gguf_blocks(qtype, n, k, seed=seed)).cuda()
    return raw, *qlin.repack_gguf(raw, qtype, (n, k))


@pytest.mark.parametrize("m,k", [(600, 256), (64, 2048)])  # single-pass epilogue; split-K finalize
def test_two_destinations_on_one_gpu(qlin, m, k):
    qtype, n, world = 12, 256, 2
    raw, packed, row_exp = _weights(qlin, qtype, n, k, seed=m)
    pads, sync = _pads(world)
    pads[0, 1] = 1000  # the other rank's flag in rank 0's pad: its kernels "finished" long ago
    bufs = [torch.zeros(world, m, n, dtype=torch.float16, device="cuda") for _ in range(world)]
    y_ranks = [b[0].data_ptr() for b in bufs]  # rank 0's slab in each rank's buffer
    g = torch.Generator().manual_seed(k)
    for call in range(2):
        x = torch.randn(1, m, k, generator=g).to(torch.float16).cuda()
        qlin.gguf_linear_allgather(x, packed, row_exp, qtype, n, y_ranks, sync, 0)
        want = qlin.gguf_linear_slabs(x, packed, row_exp, qtype, n)
        torch.cuda.synchronize()
        assert qlin.device_status() == (0, 0)
        for b in bufs:
            assert torch.equal(b[0], want)
            assert not b[1].any()
        p = pads.cpu().numpy()
        assert p[0, 8] == 0 and p[0, 9] == call + 1  # arrived reset, epoch counted
        assert p[0, 0] == call + 1 and p[1, 0] == call + 1  # published in both pads
        assert p[1, 9] == 0


def test_wait_runs_out_and_context_stays_usable(qlin):
    qtype, m, n, k, world = 8, 300, 128, 256, 2
    raw, packed, row_exp = _weights(qlin, qtype, n, k, seed=5)
    pads, sync = _pads(world)
    pads[0, 9] = 1  # rank 0 reached epoch 1; nothing ever sets rank 1's flag
    y = torch.zeros(world, world, m, n, dtype=torch.float16, device="cuda")
    x = torch.randn(1, m, k, generator=torch.Generator().manual_seed(2)).to(torch.float16).cuda()
    qlin.gguf_linear_allgather(x, packed, row_exp, qtype, n, [y[0, 0].data_ptr(), y[1, 0].data_ptr()], sync, 0,
                               timeout_ms=100)
    torch.cuda.synchronize()
    code, where = qlin.device_status()
    assert code == 4 and (where & 0xFF) == 6, (code, where)
    assert not y.any()
    # the context still runs work
    got = qlin.gguf_linear_slabs(x, packed, row_exp, qtype, n)
    want = qlin.gguf_linear(x[0], raw, qtype, (n, k))
    assert torch.equal(got, want)
    assert qlin.device_status() == (0, 0)


def _stack_worker(rank, world, port, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    import datetime
    torch.cuda.set_device(rank)
    torch.distributed.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                                         device_id=torch.device("cuda", rank))
    from qlin.sharded import ShardedStack
    dev = torch.device("cuda", rank)
    x = torch.randn(512, 1024, generator=torch.Generator().manual_seed(4)).to(torch.float16).to(dev)
    res = {}
    for transport, chunks in (("nccl", 1), ("peer", 1), ("nccl", 2), ("peer", 2)):
        st = ShardedStack(blocks=3, tokens=512, hidden=1024, chunks=chunks, device=dev, seed=9, transport=transport)
        outs = st.forward(x)
        y = torch.cat([o.permute(1, 0, 2).reshape(o.shape[1], -1) for o in outs], dim=0)
        if transport == "peer":
            st.capture(x)
            y2 = st.replay()
            y2 = torch.cat([o.permute(1, 0, 2).reshape(o.shape[1], -1) for o in y2], dim=0)
            torch.cuda.synchronize()
            assert torch.equal(y, y2)
        res[(transport, chunks)] = y.cpu()
        st.close()
    import qlin
    assert qlin.device_status() == (0, 0)
    torch.save(res, os.path.join(out_dir, f"r{rank}.pt"))
    torch.distributed.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_peer_stack_equals_nccl_stack(tmp_path):
    import socket
    import torch.multiprocessing as mp
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    mp.start_processes(_stack_worker, args=(2, port, str(tmp_path)), nprocs=2, start_method="spawn")
    r0, r1 = torch.load(tmp_path / "r0.pt"), torch.load(tmp_path / "r1.pt")
    for chunks in (1, 2):
        base = r0[("nccl", chunks)]
        assert torch.isfinite(base.float()).all()
        for res in (r0, r1):
            for transport in ("nccl", "peer"):
                got = res[(transport, chunks)]
                assert torch.equal(got, base), (transport, chunks, (got.float() - base.float()).abs().max().item())
    # a different chunking changes the GEMMs' K-split plan (fp32 summation order) only
    a, b = r0[("nccl", 1)].float(), r0[("nccl", 2)].float()
    assert ((a - b).norm() / a.norm()).item() < 1e-2
