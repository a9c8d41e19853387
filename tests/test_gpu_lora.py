"""Unmerged LoRA fused into the linears as extra K stages (bf16 operands, fp32 accumulator):
y = linear(x) + scale * (x . down^T) . up^T against float64, for the INT8 ConvRot and GGUF paths,
ranks that are and are not multiples of 64, K splits (small M) and CTA pairs (large M), and the
fallback beside the layer above rank 256."""
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


def _lora(n, k, rank, seed, dtype):
    g = torch.Generator().manual_seed(seed)
    down = (torch.randn(rank, k, generator=g) / k ** 0.5).to(dtype)
    up = (torch.randn(n, rank, generator=g) * 0.02).to(dtype)
    return down, up


def _side(x, down, up, scale):
    return scale * (x.double().numpy() @ down.double().numpy().T) @ up.double().numpy().T


@pytest.mark.parametrize("m,n", [(33, 512), (600, 1024)])
@pytest.mark.parametrize("rank", [16, 100, 256])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_int8_linear_fused_lora(qlin, m, n, rank, dtype):
    k = 1024
    x, q, s, b = O.cfg_int8_convrot(m, k, n, seed=rank + m)
    x = x.to(dtype)
    down, up = _lora(n, k, rank, m, dtype)
    ref = O.int8_convrot_linear_ref(x.float().numpy(), q.numpy(), s.float().numpy(), b.float().numpy(), group=128)
    ref = ref + _side(x, down, up, 0.75)
    y = qlin.int8_linear(x.cuda(), q.cuda(), s.cuda(), b.cuda(), dtype, convrot=True, convrot_groupsize=128,
                         lora_down=down.cuda(), lora_up=up.cuda(), lora_scale=0.75)
    tol = 2e-3 if dtype == torch.float16 else 8e-3
    assert O.max_abs_rel(y.float().cpu().numpy(), ref) <= tol, O.max_abs_rel(y.float().cpu().numpy(), ref)
    code, where = qlin.device_status()
    assert code == 0, where


@pytest.mark.parametrize("qtype", [8, 12, 14, 3, 13, 11])
@pytest.mark.parametrize("m", [20, 700])
def test_gguf_linear_fused_lora(qlin, qtype, m):
    n, k, rank = 512, 768, 64
    g = torch.Generator().manual_seed(qtype * 10 + m)
    x = torch.randn(m, k, generator=g).to(torch.float16)
    raw = O.random_gguf_blocks(qtype, n, k, seed=qtype)
    w = O.gguf_dequantize(raw, qtype, n, k)
    down, up = _lora(n, k, rank, qtype, torch.float16)
    ref = O.linear_f64(x.float().numpy(), w) + _side(x, down, up, 1.0)
    y = qlin.gguf_linear(x.cuda(), torch.from_numpy(raw).cuda(), qtype, (n, k), lora_down=down.cuda(),
                         lora_up=up.cuda(), lora_scale=1.0)
    assert O.max_abs_rel(y.float().cpu().numpy(), ref) <= 2e-3, O.max_abs_rel(y.float().cpu().numpy(), ref)


def test_rank_above_256_runs_beside(qlin):
    m, n, k, rank = 40, 256, 512, 300
    x, q, s, b = O.cfg_int8_convrot(m, k, n, seed=1)
    down, up = _lora(n, k, rank, 2, torch.float16)
    ref = O.int8_convrot_linear_ref(x.float().numpy(), q.numpy(), s.float().numpy(), b.float().numpy(), group=128)
    ref = ref + _side(x, down, up, 0.5)
    y = qlin.int8_linear(x.cuda(), q.cuda(), s.cuda(), b.cuda(), torch.float16, convrot=True, convrot_groupsize=128,
                         lora_down=down.cuda(), lora_up=up.cuda(), lora_scale=0.5)
    assert O.max_abs_rel(y.float().cpu().numpy(), ref) <= 3e-3


@pytest.mark.parametrize("path", ["int8", "gguf"])
def test_fused_lora_launches_no_library_gemm(qlin, path, monkeypatch):
    """The fused LoRA computes t = x . down^T itself: no torch / cuBLAS / CUTLASS GEMM is called or
    launched, every GEMM-like kernel of the call belongs to libqlin."""
    m, n, k, rank = 300, 512, 1024, 64
    x, q, s, b = O.cfg_int8_convrot(m, k, n, seed=4)
    down, up = _lora(n, k, rank, 5, torch.bfloat16)
    raw = torch.from_numpy(O.random_gguf_blocks(8, n, k, seed=6)).cuda()
    xd, qd, sd, bd, dd, ud = x.cuda().bfloat16(), q.cuda(), s.cuda(), b.cuda(), down.cuda(), up.cuda()

    def call():
        if path == "int8":
            return qlin.int8_linear(xd, qd, sd, bd, torch.bfloat16, convrot=True, convrot_groupsize=128,
                                    lora_down=dd, lora_up=ud, lora_scale=0.5)
        return qlin.gguf_linear(xd, raw, 8, (n, k), bias=bd, lora_down=dd, lora_up=ud, lora_scale=0.5)

    call()  # repack / warm-up outside the profiled call
    torch.cuda.synchronize()

    def forbidden(*a, **kw):
        raise AssertionError("library GEMM called on the fused LoRA path")

    monkeypatch.setattr(torch, "mm", forbidden)
    monkeypatch.setattr(torch, "matmul", forbidden)
    monkeypatch.setattr(torch.nn.functional, "linear", forbidden)
    with torch.profiler.profile(activities=[torch.profiler.ProfilerActivity.CUDA]) as prof:
        y = call()
        torch.cuda.synchronize()
    monkeypatch.undo()
    names = [e.name for e in prof.events() if e.device_type == torch.autograd.DeviceType.CUDA]
    gemmish = [nm for nm in names if any(t in nm.lower() for t in ("gemm", "cutlass", "cublas", "xmma", "nvjet"))]
    assert gemmish and all("qlin" in nm for nm in gemmish), gemmish
    ref = O.int8_convrot_linear_ref(x.bfloat16().float().numpy(), q.numpy(), s.float().numpy(), b.float().numpy(),
                                    group=128) if path == "int8" else \
        O.linear_f64(x.bfloat16().float().numpy(), O.gguf_dequantize(raw.cpu().numpy(), 8, n, k), b.float().numpy())
    ref = ref + _side(x.bfloat16(), down, up, 0.5)
    assert O.max_abs_rel(y.float().cpu().numpy(), ref) <= 8e-3
