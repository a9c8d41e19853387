"""The kitchen's AsymW4A8Int8Layout (symmetric) on the GPU: the int8 weight grid bit-identical
with the reference's own CPU port (golden fixtures from modal/weight_error_app.py:326-336), the
decode-only entry point against the fixtures' decoded rows, and the linear against float64."""
import os

import numpy as np
import pytest
import torch

from oracle import qlin_oracle as O

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(__file__), "golden", "kitchen_w4a8.npz")


@pytest.fixture(scope="module")
def qlin():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    import qlin as q
    return q


def _case(z, fmt):
    q = torch.from_numpy(z[f"{fmt}_q"]).cuda()
    s_rel = torch.from_numpy(z[f"{fmt}_s_rel"]).view(torch.float8_e4m3fn).cuda()
    s_ch = torch.from_numpy(z[f"{fmt}_s_channel"]).cuda()
    cb = torch.from_numpy(z["w4a8_codebook"]).cuda() if fmt == "w4a8" else None
    return q, s_rel, s_ch, cb


@pytest.mark.parametrize("fmt", ["w4a8", "w6a8"])
def test_grid_bit_identical_with_reference_port(qlin, fmt):
    z = np.load(GOLD)
    q, s_rel, s_ch, cb = _case(z, fmt)
    from qlin._w4a8 import kitchen_grid
    grid = kitchen_grid(q, s_rel, cb, 16)
    assert np.array_equal(grid.cpu().numpy(), z[f"{fmt}_grid"])


@pytest.mark.parametrize("fmt", ["w4a8", "w6a8"])
def test_dequantize_matches_reference_port(qlin, fmt):
    z = np.load(GOLD)
    q, s_rel, s_ch, cb = _case(z, fmt)
    w = qlin.dequantize_w4a8_int8_weight(q, s_rel, s_ch, cb, None, 16, 256, torch.float32)
    ref = z[f"{fmt}_deq16"]
    assert np.abs(w[:16].cpu().numpy() - ref).max() <= 1e-5 * np.abs(ref).max()


@pytest.mark.parametrize("fmt,bits", [("w4a8", 4), ("w6a8", 6)])
@pytest.mark.parametrize("m", [1, 40, 300])
def test_linear_matches_fp64(qlin, fmt, bits, m):
    z = np.load(GOLD)
    q, s_rel, s_ch, cb = _case(z, fmt)
    n, k = 96, 1024
    g = torch.Generator().manual_seed(m)
    x = torch.randn(m, k, generator=g).to(torch.float16)
    b = (torch.randn(n, generator=g) * 0.01).to(torch.float16)
    w = O.dequantize_kitchen_w4a8(z[f"{fmt}_q"], z[f"{fmt}_s_rel"], z[f"{fmt}_s_channel"], k, bits, 16,
                                  None if cb is None else z["w4a8_codebook"], 256)
    ref = O.linear_f64(x.float().numpy(), w, b.float().numpy())
    y = qlin.w4a8_int8_linear(x.cuda(), q, s_rel, s_ch, cb, None, b.cuda(), 16, 256)
    assert y.dtype == torch.float16
    assert O.max_abs_rel(y.float().cpu().numpy(), ref) <= 2e-3


def test_asymmetric_correction_declines(qlin):
    z = np.load(GOLD)
    q, s_rel, s_ch, cb = _case(z, "w4a8")
    with pytest.raises(NotImplementedError):
        qlin.w4a8_int8_linear(torch.randn(4, 1024, device="cuda", dtype=torch.float16), q, s_rel, s_ch, cb,
                              torch.zeros(96, device="cuda"))


def _random_kitchen(n, k, bits, seed, codebook):
    """Seeded packed codes at checkpoint widths: uniform codes, finite positive e4m3 s_rel
    (bytes 0x20..0x5F: 2^-4 .. 15), fp32 s_channel, and a sorted 16-level codebook for 4 bits."""
    rng = np.random.default_rng(seed)
    lo = 1 if bits == 6 else 0
    codes = rng.integers(lo, 1 << bits, size=(n, k))
    q = O.pack_codes_kitchen(codes, bits)
    s_rel = rng.integers(0x20, 0x60, size=(n, k // 16)).astype(np.uint8)
    s_ch = (np.abs(rng.standard_normal(n)) * 1e-3 + 1e-4).astype(np.float32)
    cb = np.sort(rng.uniform(-8, 8, 16)).astype(np.float32) if codebook else None
    return q, s_rel, s_ch, cb


@pytest.mark.parametrize("bits,codebook", [(4, True), (4, False), (6, False)])
@pytest.mark.parametrize("n,k", [(12288, 3072), (3072, 12288)])
def test_grid_and_linear_at_checkpoint_widths(qlin, bits, codebook, n, k):
    """Qwen-Image / Wan MLP widths: the int8 grid is bit-identical with the oracle's restatement of
    the reference port's decode over the whole tensor, and the linear (H4-256 rotation) meets the
    fp64 tolerance."""
    q, s_rel, s_ch, cb = _random_kitchen(n, k, bits, seed=n + k + bits, codebook=codebook)
    from qlin._w4a8 import kitchen_grid
    cb_t = None if cb is None else torch.from_numpy(cb).cuda()
    grid = kitchen_grid(torch.from_numpy(q).cuda(), torch.from_numpy(s_rel).view(torch.float8_e4m3fn).cuda(), cb_t, 16)
    want = O.kitchen_int8_grid(q, s_rel, k, bits, 16, cb)
    assert np.array_equal(grid.cpu().numpy(), want)
    m = 96
    g = torch.Generator().manual_seed(k)
    x = torch.randn(m, k, generator=g).to(torch.float16)
    w = O.dequantize_kitchen_w4a8(q, s_rel, s_ch, k, bits, 16, cb, 256)
    ref = O.linear_f64(x.float().numpy(), w)
    y = qlin.w4a8_int8_linear(x.cuda(), torch.from_numpy(q).cuda(),
                              torch.from_numpy(s_rel).view(torch.float8_e4m3fn).cuda(),
                              torch.from_numpy(s_ch).cuda(), cb_t, None, None, 16, 256)
    assert O.max_abs_rel(y.float().cpu().numpy(), ref) <= 2e-3


@pytest.mark.parametrize("bits,k,group,codebook", [(4, 48, 16, True), (4, 96, 32, False), (6, 64, 16, False),
                                                   (6, 96, 32, False), (4, 1024, 16, False), (6, 1024, 64, False)])
def test_grid_every_scale_code_and_both_kernels(qlin, bits, k, group, codebook):
    """Every finite e4m3 group-scale code (subnormals, +-448, negative scales) and codes over the full
    range, through both grid kernels (32 values per thread when K is a multiple of 32 and the group 16
    or a multiple of 32, else 16 per thread): bit-identical with the oracle."""
    rng = np.random.default_rng(bits * 1000 + k + group)
    n = 37
    codes = rng.integers(0, 1 << bits, size=(n, k))
    q = O.pack_codes_kitchen(codes, bits)
    finite = np.array([b for b in range(256) if (b & 0x7F) != 0x7F], dtype=np.uint8)
    s_rel = rng.choice(finite, size=(n, k // group)).astype(np.uint8)
    cb = np.sort(rng.uniform(-8, 8, 16)).astype(np.float32) if codebook else None
    from qlin._w4a8 import kitchen_grid
    grid = kitchen_grid(torch.from_numpy(q).cuda(), torch.from_numpy(s_rel).view(torch.float8_e4m3fn).cuda(),
                        None if cb is None else torch.from_numpy(cb).cuda(), group)
    want = O.kitchen_int8_grid(q, s_rel, k, bits, group, cb)
    assert np.array_equal(grid.cpu().numpy(), want)
