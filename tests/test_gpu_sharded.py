"""GPU checks of the slab operand and the sharded MMDiT stack on one GPU.

* qlin_gguf_linear_slabs on an activation split into column slabs equals the ordinary GGUF linear
  on the concatenated activation (same kernel, same K order: identical bits).
* The stack on one rank equals a chain of gguf_linear calls over the same weights."""
import pytest
import torch

from oracle import qlin_oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def qlin():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    import qlin as q
    return q


@pytest.mark.parametrize("qtype,slabs", [(12, 2), (14, 4), (8, 3)])
def test_slab_operand_equals_row_major(qlin, qtype, slabs):
    m, n, k = 200, 256, 768 if qtype != 14 else 1536
    if (k // slabs) % 64:
        pytest.skip("slab width must be a multiple of 64")
    g = torch.Generator().manual_seed(qtype + slabs)
    x = torch.randn(m, k, generator=g).to(torch.float16).cuda()
    raw = torch.from_numpy(O.random_gguf_blocks(qtype, n, k, seed=qtype)).cuda()
    packed, row_exp = qlin.repack_gguf(raw, qtype, (n, k))
    want = qlin.gguf_linear(x, raw, qtype, (n, k))
    xs = x.view(m, slabs, k // slabs).permute(1, 0, 2).contiguous()  # [slabs, m, k/slabs]
    got = qlin.gguf_linear_slabs(xs, packed, row_exp, qtype, n)
    assert torch.equal(got, want)


@pytest.mark.parametrize("gather", ["consumed", "all"])
def test_stack_on_one_gpu_equals_linear_chain(qlin, gather):
    from qlin.sharded import ShardedStack, base_weight, layers
    dev = torch.device("cuda", 0)
    hidden, tokens = 256, 384
    st = ShardedStack(blocks=2, tokens=tokens, hidden=hidden, chunks=2, device=dev, seed=3, gather=gather)
    x = torch.randn(tokens, hidden, generator=torch.Generator().manual_seed(1)).to(torch.float16).to(dev)
    outs = st.forward(x)
    got = torch.cat([o[0] for o in outs], dim=0)
    h = x
    for b in range(2):
        res = {"x": h}
        for name, base, qtype, n, k, src, col0, _ in layers(hidden, gather, 1):
            raw = base_weight(3, b, base, hidden, dev)
            # chunk by chunk, as the stack runs it (the same GEMM plan, hence identical sums)
            inp = res[src][:, col0:col0 + k]
            res[name] = torch.cat([qlin.gguf_linear(c, raw, qtype, (n, k)) for c in inp.split(tokens // 2)])
        h = res["down"]
    assert torch.isfinite(got).all()
    assert torch.equal(got, h)
