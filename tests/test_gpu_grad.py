"""GPU parity of the input gradient for frozen packed weights (int8_linear_grad_input,
w4a8_linear_grad_input and the *_trainable autograd wrappers) through the C-ABI, against the
float64 restatement dx = dy . W: max |dx - ref| / max |ref| within 2e-3 for fp16 and fp32
outputs and 8e-3 for bf16 (the forward's tolerances)."""
import os

import numpy as np
import pytest
import torch

from oracle import qlin_oracle as O

pytestmark = pytest.mark.gpu
TOL = {torch.float16: 2e-3, torch.bfloat16: 8e-3, torch.float32: 2e-3}
GOLD = os.path.join(os.path.dirname(__file__), "golden", "kitchen_w4a8.npz")


@pytest.fixture(scope="module")
def qlin():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    import qlin as q
    return q


def _weights(n, k, seed):
    g = torch.Generator().manual_seed(seed)
    q = torch.randint(-127, 128, (n, k), generator=g, dtype=torch.int32).to(torch.int8)
    s = (torch.randn(n, generator=g).abs() * 0.02 / 127).to(torch.float16)
    return q, s, g


def _check_status(qlin):
    code, where = qlin.device_status(reset=True)
    assert code == 0, f"a kernel timed out waiting (where={where:#x})"


@pytest.mark.parametrize("m,n,k", [(1, 200, 256), (2, 64, 512), (37, 300, 512), (300, 1000, 768), (700, 520, 1024)])
@pytest.mark.parametrize("group", [0, 32, 64, 128, 256])
def test_int8_grad_input_matches_fp64(qlin, m, n, k, group):
    q, s, g = _weights(n, k, seed=m + n + group)
    dy = torch.randn(m, n, generator=g).to(torch.float16)
    ref = O.int8_grad_input(dy.double().numpy(), q.numpy(), s.float().numpy(), group)
    dx = qlin.int8_linear_grad_input(dy.cuda(), q.cuda(), s.cuda(), group > 0, group or 256)
    assert dx.dtype == torch.float16 and dx.shape == (m, k)
    got = dx.float().cpu().numpy()
    assert np.isfinite(got).all()
    assert O.max_abs_rel(got, ref) <= TOL[torch.float16], O.max_abs_rel(got, ref)
    _check_status(qlin)


@pytest.mark.parametrize("dy_dtype,out_dtype,scale_dtype", [
    (torch.bfloat16, torch.bfloat16, torch.float32), (torch.float32, torch.float32, torch.float16),
    (torch.float16, torch.float32, torch.float32), (torch.float32, torch.bfloat16, torch.float16)])
def test_int8_grad_input_dtypes(qlin, dy_dtype, out_dtype, scale_dtype):
    m, n, k = 45, 130, 512
    q, s, g = _weights(n, k, seed=3)
    s = s.to(scale_dtype)
    dy = (torch.randn(m, n, generator=g) * 2e-5).to(dy_dtype)  # training-scale gradients
    ref = O.int8_grad_input(dy.double().numpy(), q.numpy(), s.double().numpy(), 128)
    dx = qlin.int8_linear_grad_input(dy.cuda(), q.cuda(), s.cuda(), True, 128, out_dtype=out_dtype)
    assert dx.dtype == out_dtype
    assert O.max_abs_rel(dx.float().cpu().numpy(), ref) <= TOL[out_dtype]


def test_int8_grad_input_shapes_and_edges(qlin):
    n, k = 96, 256
    q, s, g = _weights(n, k, seed=5)
    qd, sd = q.cuda(), s.cuda()
    # N-d and non-contiguous dy
    dy = torch.randn(3, 4, 2 * n, generator=g).to(torch.float16).cuda()[..., ::2]
    dx = qlin.int8_linear_grad_input(dy, qd, sd, True, 256)
    assert dx.shape == (3, 4, k)
    ref = O.int8_grad_input(dy.reshape(-1, n).double().cpu().numpy(), q.numpy(), s.float().numpy(), 256)
    assert O.max_abs_rel(dx.reshape(-1, k).float().cpu().numpy(), ref) <= 2e-3
    # a scalar scale broadcasts
    dx1 = qlin.int8_linear_grad_input(dy, qd, torch.tensor([0.01], device="cuda"), False)
    ref1 = O.int8_grad_input(dy.reshape(-1, n).double().cpu().numpy(), q.numpy(), np.full(n, 0.01), 0)
    assert O.max_abs_rel(dx1.reshape(-1, k).float().cpu().numpy(), ref1) <= 2e-3
    # empty token dimension and empty contraction
    assert qlin.int8_linear_grad_input(torch.empty(0, n, dtype=torch.float16, device="cuda"), qd, sd).shape == (0, k)
    q0 = torch.empty(0, k, dtype=torch.int8, device="cuda")
    z = qlin.int8_linear_grad_input(torch.empty(5, 0, dtype=torch.float16, device="cuda"), q0,
                                    torch.empty(0, device="cuda"))
    assert z.shape == (5, k) and bool((z == 0).all())
    # zero rows of dy give zero rows of dx
    dyz = torch.zeros(4, n, dtype=torch.float16, device="cuda")
    assert bool((qlin.int8_linear_grad_input(dyz, qd, sd, True, 128) == 0).all())
    _check_status(qlin)


def test_int8_trainable_gradients(qlin):
    m, n, k = 64, 192, 512
    q, s, g = _weights(n, k, seed=9)
    qd, sd = q.cuda(), s.cuda()
    x = torch.randn(m, k, generator=g).to(torch.float16).cuda().requires_grad_(True)
    b = (torch.randn(n, generator=g) * 0.01).to(torch.float16).cuda().requires_grad_(True)
    y = qlin.int8_linear_trainable(x, qd, sd, b, True, 256)
    assert torch.equal(y.detach(), qlin.int8_linear(x.detach(), qd, sd, b.detach(), convrot=True, convrot_groupsize=256))
    dy = torch.randn(m, n, generator=g).to(torch.float16).cuda()
    y.backward(dy)
    assert torch.equal(x.grad, qlin.int8_linear_grad_input(dy, qd, sd, True, 256, out_dtype=torch.float16))
    assert torch.allclose(b.grad.float(), dy.float().sum(0), rtol=1e-3, atol=1e-2)
    assert q.grad is None


@pytest.mark.parametrize("fmt,bits", [("w4a8", 4), ("w6a8", 6)])
def test_w4a8_grad_input_matches_fp64(qlin, fmt, bits):
    z = np.load(GOLD)
    q = torch.from_numpy(z[f"{fmt}_q"]).cuda()
    s_rel = torch.from_numpy(z[f"{fmt}_s_rel"]).view(torch.float8_e4m3fn).cuda()
    s_ch = torch.from_numpy(z[f"{fmt}_s_channel"]).cuda()
    cb = torch.from_numpy(z["w4a8_codebook"]).cuda() if fmt == "w4a8" else None
    n, k = 96, 1024
    w = O.dequantize_kitchen_w4a8(z[f"{fmt}_q"], z[f"{fmt}_s_rel"], z[f"{fmt}_s_channel"], k, bits, 16,
                                  None if cb is None else z["w4a8_codebook"], 256)
    dy = torch.randn(33, n, generator=torch.Generator().manual_seed(bits)).to(torch.float16)
    ref = dy.double().numpy() @ np.asarray(w, dtype=np.float64)
    dx = qlin.w4a8_linear_grad_input(dy.cuda(), q, s_rel, s_ch, cb, None, 16, 256, torch.float16)
    assert O.max_abs_rel(dx.float().cpu().numpy(), ref) <= 2e-3
    x = torch.randn(33, k, dtype=torch.float16, device="cuda", requires_grad=True)
    qlin.w4a8_linear_trainable(x, q, s_rel, s_ch, cb, None, None, 16, 256).backward(dy.cuda())
    assert torch.equal(x.grad, dx)
    with pytest.raises(NotImplementedError):
        qlin.w4a8_linear_grad_input(dy.cuda(), q, s_rel, s_ch, cb, torch.zeros(k // 16, n, device="cuda"), 16, 256)


@pytest.mark.parametrize("pad", [0, 4, 8])
def test_int8_grad_input_abi_row_pitch(qlin, pad):
    """dx written with a row pitch of k + pad through the C ABI (pad 4: rows not 16-byte aligned,
    so the rotation stores element by element; pad 8: aligned rows, vector stores); the padding
    columns stay untouched."""
    from qlin import _lib
    m, n, k = 33, 200, 256
    q, s, g = _weights(n, k, seed=11)
    dy = torch.randn(m, n, generator=g).to(torch.float16)
    qd, sd, dyd = q.cuda(), s.cuda(), dy.cuda()
    qt = qlin._grad.grad_weight(qd)
    ld = k + pad
    dx = torch.full((m, ld), 7.0, dtype=torch.float16, device="cuda")
    nws = _lib.lib.qlin_int8_linear_grad_input_workspace(m, n, k, 128)
    ws = torch.empty(nws, dtype=torch.uint8, device="cuda")
    rc = _lib.lib.qlin_int8_linear_grad_input(dyd.data_ptr(), 1, m, n, n, qt.data_ptr(), k, sd.data_ptr(), 1, 128,
                                              dx.data_ptr(), 1, ld, ws.data_ptr(), nws,
                                              torch.cuda.current_stream().cuda_stream)
    assert rc == 0, _lib.lib.qlin_last_error()
    ref = O.int8_grad_input(dy.double().numpy(), q.numpy(), s.float().numpy(), 128)
    assert O.max_abs_rel(dx[:, :k].float().cpu().numpy(), ref) <= 2e-3
    if pad:
        assert bool((dx[:, k:] == 7.0).all())
    # a workspace one byte short is refused before any launch
    rc = _lib.lib.qlin_int8_linear_grad_input(dyd.data_ptr(), 1, m, n, n, qt.data_ptr(), k, sd.data_ptr(), 1, 128,
                                              dx.data_ptr(), 1, ld, ws.data_ptr(), nws - 1,
                                              torch.cuda.current_stream().cuda_stream)
    assert rc == 2


@pytest.mark.parametrize("group", [32, 64, 128])
@pytest.mark.parametrize("out_dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("m,n,k", [(2048, 1024, 3072), (4096, 512, 1408)])  # CTA pairs; 11 tiles: single CTAs
def test_fused_rotation_equals_separate_pass(qlin, group, out_dtype, m, n, k):
    """With a 2-byte dx, no K split and groups up to 128 the GEMM epilogue rotates dx's rows
    itself; a row pitch that is not a multiple of 8 elements takes the fp32 output + separate
    rotation pass instead.  Both apply the same butterflies to the same fp32 values, so they agree
    bit for bit."""
    from qlin import _lib
    q, s, g = _weights(n, k, seed=group)
    dy = torch.randn(m, n, generator=g).to(torch.float16).cuda()
    qd, sd = q.cuda(), s.cuda()
    qt = qlin._grad.grad_weight(qd)
    nws = _lib.lib.qlin_int8_linear_grad_input_workspace(m, n, k, group)
    ws = torch.empty(nws, dtype=torch.uint8, device="cuda")
    code = 1 if out_dtype == torch.float16 else 2
    outs, rotate_launches = [], []
    for ld in (k, k + 4):
        dx = torch.zeros(m, ld, dtype=out_dtype, device="cuda")
        torch.cuda.synchronize()
        with torch.profiler.profile(activities=[torch.profiler.ProfilerActivity.CUDA]) as prof:
            rc = _lib.lib.qlin_int8_linear_grad_input(dy.data_ptr(), 1, m, n, n, qt.data_ptr(), k, sd.data_ptr(), 1,
                                                      group, dx.data_ptr(), code, ld, ws.data_ptr(), nws,
                                                      torch.cuda.current_stream().cuda_stream)
            torch.cuda.synchronize()
        assert rc == 0, _lib.lib.qlin_last_error()
        rotate_launches.append(sum(1 for e in prof.events() if "grad_rotate_kernel" in e.name))
        outs.append(dx[:, :k].clone())
    assert rotate_launches == [0, 1]  # fused in the epilogue, then the separate pass
    assert torch.equal(outs[0], outs[1])
    ref = O.int8_grad_input(dy.double().cpu().numpy(), q.numpy(), s.float().numpy(), group)
    assert O.max_abs_rel(outs[0].float().cpu().numpy(), ref) <= TOL[out_dtype]
    _check_status(qlin)
