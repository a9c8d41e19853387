"""GPU parity of the W4A8 / W6A8 kind::i8 path through the C-ABI.

* int32 accumulation bit-exact: integer activations whose row maximum is 127 quantize with scale
  exactly 1, so with power-of-two group scales the fp32 output must equal the exact integer
  result of the CPU oracle bit for bit (each group's int32 sum is checked through its own scale).
* Random data: fp16 outputs within max-abs-rel 2e-3 of the float64 reference computed from the
  same per-token INT8 activations (oracle.grouped_linear_a8).
"""
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


def _pack(wq, bits, layout):
    if bits == 4:
        return O.pack_w4_uniform(wq).view(np.uint8)
    if layout == 0:
        return O.pack_w6_interleaved(wq)
    return O.pack_codes_kitchen(np.asarray(wq, np.int32) + 32, 6).view(np.uint8)


@pytest.mark.parametrize("bits,layout", [(4, 0), (6, 0), (6, 1)])
@pytest.mark.parametrize("group", [32, 64, 128, 256])
def test_int32_accumulation_bit_exact(qlin, bits, layout, group):
    m, n, k = 40, 256, 512
    rng = np.random.default_rng(bits * 100 + group)
    x = rng.integers(-127, 128, (m, k)).astype(np.float32)
    x[:, 7] = 127.0  # every row's absmax is 127 -> activation scale exactly 1
    lo, hi = (-8, 8) if bits == 4 else (-32, 32)
    wq = rng.integers(lo, hi, (n, k)).astype(np.int8)
    groups = k // group
    s = np.ldexp(1.0, -(np.arange(groups) % 3))[None, :].repeat(n, 0).astype(np.float16)  # 1, 1/2, 1/4, ...
    p = O.int_group_partials(x.astype(np.int64), wq, group)  # [groups, m, n] exact
    want = np.zeros((m, n))
    for g in range(groups):
        want += p[g] * float(s[0, g])
    xt = torch.from_numpy(x).to(torch.float16).cuda()
    w = torch.from_numpy(_pack(wq, bits, layout).copy()).cuda()
    y = qlin.w4a8_linear(xt, w, torch.from_numpy(s).cuda(), bits=bits, group_size=group, layout=layout,
                         out_dtype=torch.float32)
    got = y.cpu().numpy().astype(np.float64)
    assert np.array_equal(got, want), np.abs(got - want).max()
    code, where = qlin.device_status()
    assert code == 0, where


@pytest.mark.parametrize("bits", [4, 6])
def test_per_channel_scales_bit_exact(qlin, bits):
    m, n, k = 33, 192, 1024
    rng = np.random.default_rng(3 + bits)
    x = rng.integers(-127, 128, (m, k)).astype(np.float32)
    x[:, 0] = -127.0
    lo, hi = (-8, 8) if bits == 4 else (-32, 32)
    wq = rng.integers(lo, hi, (n, k)).astype(np.int8)
    s = np.ldexp(1.0, -rng.integers(0, 4, n)).astype(np.float32)
    want = (x.astype(np.int64) @ wq.astype(np.int64).T).astype(np.float64) * s[None, :]
    y = qlin.w4a8_linear(torch.from_numpy(x).half().cuda(), torch.from_numpy(_pack(wq, bits, 0).copy()).cuda(),
                         torch.from_numpy(s).cuda(), bits=bits, group_size=0, out_dtype=torch.float32)
    assert np.array_equal(y.cpu().numpy().astype(np.float64), want)


@pytest.mark.parametrize("bits,group", [(4, 128), (6, 64)])
@pytest.mark.parametrize("m", [1, 5, 33, 130, 300])
def test_random_matches_fp64_reference(qlin, bits, group, m):
    n, k = 320, 1536
    g = torch.Generator().manual_seed(m * 7 + bits)
    x = torch.randn(m, k, generator=g).to(torch.float16)
    lo, hi = (-8, 8) if bits == 4 else (-32, 32)
    wq = torch.randint(lo, hi, (n, k), generator=g, dtype=torch.int32).numpy().astype(np.int8)
    s = (torch.randn(n, k // group, generator=g).abs() * 0.02 / (7 if bits == 4 else 31)).to(torch.float16)
    b = (torch.randn(n, generator=g) * 0.01).to(torch.float16)
    ref, _, _ = O.grouped_linear_a8(x.numpy(), wq, s.numpy(), group, b.float().numpy())
    y = qlin.w4a8_linear(x.cuda(), torch.from_numpy(_pack(wq, bits, 0).copy()).cuda(), s.cuda(), bits=bits,
                         group_size=group, bias=b.cuda())
    assert y.dtype == torch.float16
    got = y.float().cpu().numpy()
    assert np.isfinite(got).all()
    assert O.max_abs_rel(got, ref) <= 2e-3, O.max_abs_rel(got, ref)


def test_bf16_input_rotation_and_ragged_n(qlin):
    m, n, k, group = 70, 200, 1024, 128
    g = torch.Generator().manual_seed(5)
    x = torch.randn(m, k, generator=g).to(torch.bfloat16)
    wq = torch.randint(-8, 8, (n, k), generator=g, dtype=torch.int32).numpy().astype(np.int8)
    s = (torch.randn(n, k // group, generator=g).abs() * 0.003).to(torch.float16)
    xr = torch.from_numpy(O.rotate_rows(x.float().numpy(), 256)).to(torch.bfloat16)  # rotated, rounded to x's dtype
    ref, _, _ = O.grouped_linear_a8(xr, wq, s.numpy(), group)
    y = qlin.w4a8_linear(x.cuda(), torch.from_numpy(_pack(wq, 4, 0).copy()).cuda(), s.cuda(), bits=4, group_size=group,
                         rotate_group=256, out_dtype=torch.float32)
    # bf16 rounding of the rotated activations differs from the fp16 reference quantizer only in
    # rare codes; the output tolerance absorbs it
    assert O.max_abs_rel(y.cpu().numpy(), ref) <= 1e-2


def test_rejects_bad_shapes(qlin):
    x = torch.randn(4, 100, device="cuda", dtype=torch.float16)
    w = torch.zeros(128, 50, dtype=torch.uint8, device="cuda")
    with pytest.raises(NotImplementedError):
        qlin.w4a8_linear(x, w, torch.ones(128, 1, dtype=torch.float16, device="cuda"), bits=4, group_size=100)


@pytest.mark.parametrize("bits,layout", [(4, 0), (6, 0), (6, 1)])
@pytest.mark.parametrize("group", [64, 128, 256, 0])
@pytest.mark.parametrize("m", [100, 300])
def test_pair_kernel_int32_exact(qlin, bits, layout, group, m):
    """Token counts above 64 run on CTA pairs (256 weight rows, 128- or 256-token tiles, decoded
    weights in shared memory): every group's int32 sum exact through its power-of-two scale, for
    groups of 64 (two per 128-deep stage), 128, 256 (two stages per group) and per-channel scales;
    N = 320 leaves the odd CTA of the last pair past the last weight row."""
    n, k = 320, 1024
    rng = np.random.default_rng(bits * 1000 + group + m)
    x = rng.integers(-127, 128, (m, k)).astype(np.float32)
    x[:, 3] = 127.0  # activation scale exactly 1
    lo, hi = (-8, 8) if bits == 4 else (-32, 32)
    wq = rng.integers(lo, hi, (n, k)).astype(np.int8)
    if group:
        groups = k // group
        s = np.ldexp(1.0, -((np.arange(n)[:, None] + np.arange(groups)[None, :]) % 3)).astype(np.float16)
        want = np.zeros((m, n))
        p = O.int_group_partials(x.astype(np.int64), wq, group)
        for g in range(groups):
            want += p[g] * s[:, g][None, :].astype(np.float64)
    else:
        s = np.ldexp(1.0, -rng.integers(0, 4, n)).astype(np.float32)
        want = (x.astype(np.int64) @ wq.astype(np.int64).T).astype(np.float64) * s[None, :]
    y = qlin.w4a8_linear(torch.from_numpy(x).half().cuda(), torch.from_numpy(_pack(wq, bits, layout).copy()).cuda(),
                         torch.from_numpy(s).cuda(), bits=bits, group_size=group, layout=layout,
                         out_dtype=torch.float32)
    got = y.cpu().numpy().astype(np.float64)
    assert np.isfinite(got).all()
    assert np.array_equal(got, want), np.abs(got - want).max()
    code, where = qlin.device_status()
    assert code == 0, where
