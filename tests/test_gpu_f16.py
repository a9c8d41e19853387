"""GPU parity of the weight-only (kind::f16) path through the C-ABI: GGUF decode bit-exact with
gguf-py 0.19.0 via the oracle, GGUF and INT8 ConvRot linears within the north-star tolerance
(max |y - ref| / max |ref| <= 2e-3 for fp16 outputs, against a float64 reference)."""
import numpy as np
import pytest
import torch

import checks as C
from oracle import qlin_oracle as O

pytestmark = pytest.mark.gpu

TOL = {torch.float16: 2e-3, torch.bfloat16: 8e-3, torch.float32: 2e-3}


@pytest.fixture(scope="module")
def qlin():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    import qlin as q
    return q


def _check_status(qlin):
    code, where = qlin.device_status(reset=True)
    assert code == 0, f"a kernel timed out waiting (where={where:#x})"


ALL_TYPES = sorted(O.GGUF_TYPES)


@pytest.mark.parametrize("qtype", ALL_TYPES)
@pytest.mark.parametrize("out_dtype", [torch.float32, torch.float16, torch.bfloat16])
def test_gguf_dequantize_bit_exact(qlin, qtype, out_dtype):
    name, qk, ts = O.GGUF_TYPES[qtype]
    raw = O.random_gguf_blocks(qtype, 40, 768 if qk == 256 else 544, seed=qtype)
    n, k = 40, (768 if qk == 256 else 544)
    flat = raw.reshape(-1, ts)
    offs = O.GGUF_SCALE_FIELDS[name][0]
    for i, v in enumerate([0.0, 65504.0, -65504.0, 2.0 ** -24, -(2.0 ** -20), 6.1e-5]):
        for off in offs:
            flat[i, off:off + 2] = np.array([v], dtype=np.float16).view(np.uint8)
    ref = O.gguf_dequantize(raw, qtype, n, k)
    got = qlin.dequantize_gguf(torch.from_numpy(raw).cuda(), qtype, (n, k), out_dtype).cpu()
    want = torch.from_numpy(ref).to(out_dtype)
    assert torch.equal(got.view(-1).float().isnan(), want.view(-1).float().isnan())
    assert torch.equal(got.float().nan_to_num(), want.float().nan_to_num())
    if out_dtype == torch.float32:
        assert np.array_equal(got.numpy().view(np.uint32), ref.view(np.uint32))
    _check_status(qlin)


@pytest.mark.parametrize("qtype", [11, 12, 13, 23])
def test_gguf_dequantize_rows_straddling_blocks(qlin, qtype):
    raw = O.random_gguf_blocks(qtype, 3, 1024, seed=5)  # 12 superblocks
    ref = O.gguf_dequantize(raw, qtype, 6, 512)
    got = qlin.dequantize_gguf(torch.from_numpy(raw).cuda(), qtype, (6, 512), torch.float32).cpu().numpy()
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))


@pytest.mark.parametrize("qtype", ALL_TYPES)
def test_gguf_repack_row_exponents(qlin, qtype):
    n, k = 200, 1024
    raw = O.random_gguf_blocks(qtype, n, k, seed=11 + qtype)
    packed, rexp = qlin.repack_gguf(torch.from_numpy(raw).cuda(), qtype, (n, k))
    want = O.gguf_row_exponent(O.gguf_row_bound(raw, qtype, n, k))
    got = rexp.cpu().numpy()
    assert got.shape[0] == 256
    assert np.array_equal(got[:n], want)
    assert np.all(got[n:] == 0)


EXACT_DECODE = (2, 6, 8, 20)  # Q4_0, Q5_0, Q8_0, IQ4_NL: RN16(w * 2^-e), one rounding


@pytest.mark.parametrize("qtype", ALL_TYPES)
def test_gguf_decoded_weights_through_the_linear(qlin, qtype):
    """One-hot activation rows pull single decoded weights through the linear (fp32 output, no
    bias; adding zeros is exact): the identity over all K columns runs the tensor-core GEMM, one
    row the small-M kernel and two rows the GEMM's split-K path.  Types decoded with one rounding must give RN16(w * 2^-e) * 2^e
    bit for bit; the others stay within two fp16 rounding steps at the row's largest weight."""
    n, k = 256, 512
    raw = O.random_gguf_blocks(qtype, n, k, seed=70 + qtype)
    w = O.gguf_dequantize(raw, qtype, n, k).T
    raw_d = torch.from_numpy(raw).cuda()
    eye = torch.eye(k, dtype=torch.float16)
    for rows in (slice(0, k), slice(37, 38), slice(37, 39)):
        y = qlin.gguf_linear(eye[rows].cuda(), raw_d, qtype, (n, k), out_dtype=torch.float32).cpu().numpy()
        if qtype in EXACT_DECODE:
            C.onehot_exact(O.GGUF_TYPES[qtype][0], y, raw, qtype, n, k, rows)  # +0 and -0 alike
        else:
            tol = np.abs(w).max(axis=0) * 2.0 ** -9
            assert np.all(np.abs(y - w[rows]) <= tol), (qtype, np.abs(y - w[rows]).max())
    _check_status(qlin)


def _gguf_case(qtype, m, n, k, seed, x_dtype=torch.float16, bias=True, scale=None):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(m, k, generator=g).to(x_dtype)
    raw = O.random_gguf_blocks(qtype, n, k, seed=seed, scale=scale)
    b = (torch.randn(n, generator=g) * 0.1).to(torch.float16) if bias else None
    w = O.gguf_dequantize(raw, qtype, n, k)
    ref = O.linear_f64(x.float().numpy(), w, None if b is None else b.float().numpy())
    return x, raw, b, ref


@pytest.mark.parametrize("qtype", ALL_TYPES)
@pytest.mark.parametrize("m", [1, 7, 16, 33, 130, 300])
def test_gguf_linear_matches_fp64(qlin, qtype, m):
    n, k = 384, 1024
    x, raw, b, ref = _gguf_case(qtype, m, n, k, seed=m * 31 + qtype)
    y = qlin.gguf_linear(x.cuda(), torch.from_numpy(raw).cuda(), qtype, (n, k), bias=None if b is None else b.cuda())
    assert y.dtype == torch.float16 and y.shape == (m, n)
    got = y.float().cpu().numpy()
    assert np.isfinite(got).all()
    assert O.max_abs_rel(got, ref) <= 2e-3, O.max_abs_rel(got, ref)
    _check_status(qlin)


@pytest.mark.parametrize("qtype", ALL_TYPES)
@pytest.mark.parametrize("m", [600, 1000])
def test_gguf_linear_cta_pairs_match_fp64(qlin, qtype, m):
    """Token tiles of 192 / 256 over an even number of 128-row weight tiles: the two-CTA
    (cta_group::2) kernels, several tiles per CTA pair, a ragged last token tile."""
    n, k = 512, 768 if O.GGUF_TYPES[qtype][1] == 256 else 640
    x, raw, b, ref = _gguf_case(qtype, m, n, k, seed=m + qtype)
    y = qlin.gguf_linear(x.cuda(), torch.from_numpy(raw).cuda(), qtype, (n, k), bias=b.cuda())
    got = y.float().cpu().numpy()
    assert np.isfinite(got).all()
    assert O.max_abs_rel(got, ref) <= 2e-3, O.max_abs_rel(got, ref)
    _check_status(qlin)


@pytest.mark.parametrize("qtype", [8, 12, 3, 7, 13, 23])
@pytest.mark.parametrize("x_dtype,out_dtype", [(torch.bfloat16, torch.bfloat16), (torch.float16, torch.float32),
                                               (torch.float32, torch.float16)])
def test_gguf_linear_dtypes_and_ragged_n(qlin, qtype, x_dtype, out_dtype):
    m, n, k = 45, 200, 768 if O.GGUF_TYPES[qtype][1] == 256 else 800
    x, raw, b, ref = _gguf_case(qtype, m, n, k, seed=7, x_dtype=x_dtype)
    y = qlin.gguf_linear(x.cuda(), torch.from_numpy(raw).cuda(), qtype, (n, k), bias=b.cuda(), out_dtype=out_dtype)
    assert y.dtype == out_dtype
    assert O.max_abs_rel(y.float().cpu().numpy(), ref) <= TOL[out_dtype]


def test_gguf_linear_large_activations_and_scales(qlin):
    # H3-scale activations (|x| ~ 3e4) against large block scales: the row exponents keep the fp16
    # operands finite.
    m, n, k = 64, 256, 512
    g = torch.Generator().manual_seed(3)
    x = (torch.randn(m, k, generator=g) * 1e4).clamp(-6e4, 6e4).to(torch.float16)
    raw = O.random_gguf_blocks(8, n, k, seed=3, scale=30.0)
    w = O.gguf_dequantize(raw, 8, n, k)
    ref = O.linear_f64(x.float().numpy(), w)
    y = qlin.gguf_linear(x.cuda(), torch.from_numpy(raw).cuda(), 8, (n, k), out_dtype=torch.float32)
    got = y.cpu().numpy()
    assert np.isfinite(got).all()
    assert O.max_abs_rel(got, ref) <= 2e-3


def test_gguf_linear_nd_input_and_empty(qlin):
    n, k = 128, 512
    raw = torch.from_numpy(O.random_gguf_blocks(2, n, k, seed=1)).cuda()
    x = torch.randn(2, 5, k, device="cuda", dtype=torch.float16)
    y = qlin.gguf_linear(x, raw, 2, (n, k))
    assert y.shape == (2, 5, n)
    y2 = qlin.gguf_linear(x.reshape(10, k), raw, 2, (n, k))
    assert torch.equal(y.reshape(10, n), y2)
    e = qlin.gguf_linear(torch.empty(0, k, device="cuda", dtype=torch.float16), raw, 2, (n, k))
    assert e.shape == (0, n)


@pytest.mark.parametrize("group", [0, 128, 256])
@pytest.mark.parametrize("m,n", [(1, 320), (16, 320), (100, 320), (256, 320), (256, 512), (768, 1024)])
def test_int8_convrot_linear_matches_fp64(qlin, group, m, n):
    k = 1024
    x, q, s, b = O.cfg_int8_convrot(m, k, n, seed=m + group)
    ref = O.int8_convrot_linear_ref(x.float().numpy(), q.numpy(), s.float().numpy(), b.float().numpy(),
                                    group=group or 128, convrot=group > 0)
    y = qlin.int8_linear(x.cuda(), q.cuda(), s.cuda(), b.cuda(), torch.float16, convrot=group > 0,
                         convrot_groupsize=group or 256)
    got = y.float().cpu().numpy()
    assert np.isfinite(got).all()
    assert O.max_abs_rel(got, ref) <= 2e-3, O.max_abs_rel(got, ref)
    _check_status(qlin)


@pytest.mark.parametrize("x_dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("scale_dtype", [torch.float32, torch.float16])
def test_int8_linear_dtypes_and_scale_shapes(qlin, x_dtype, scale_dtype):
    m, n, k = 77, 256, 768
    x, q, s, b = O.cfg_int8_convrot(m, k, n, seed=5)
    x = x.to(x_dtype)
    ref = O.int8_convrot_linear_ref(x.float().numpy(), q.numpy(), s.float().numpy(), None, group=256)
    y = qlin.int8_linear(x.cuda(), q.cuda(), s.to(scale_dtype).reshape(n, 1).cuda(), None, torch.float32,
                         convrot=True, convrot_groupsize=256)
    assert O.max_abs_rel(y.cpu().numpy(), ref) <= 2e-3


def test_int8_linear_extreme_rows(qlin):
    # rows with an outlier of 16000, tiny rows (2^-26) and zero rows
    m, n, k = 48, 128, 512
    g = torch.Generator().manual_seed(9)
    x = torch.randn(m, k, generator=g)
    x[0, 3] = 16000.0
    x[1] *= 2.0 ** -26
    x[2] = 0
    x = x.to(torch.float16)
    q = torch.randint(-127, 128, (n, k), generator=g, dtype=torch.int32).to(torch.int8)
    s = torch.full((n,), 1e-3)
    ref = O.int8_convrot_linear_ref(x.float().numpy(), q.numpy(), s.numpy(), None, group=128)
    y = qlin.int8_linear(x.cuda(), q.cuda(), s.cuda(), None, torch.float32, convrot=True, convrot_groupsize=128)
    got = y.cpu().numpy()
    assert np.isfinite(got).all()
    assert np.all(got[2] == 0)
    for r in range(m):  # per-row check so the tiny row is held to its own scale
        if np.abs(ref[r]).max() > 0:
            assert O.max_abs_rel(got[r], ref[r]) <= 2e-3, r


def test_prologue_rotation_matches_oracle(qlin):
    m, k = 33, 1024
    g = torch.Generator().manual_seed(4)
    x = torch.randn(m, k, generator=g).to(torch.float16)
    for group in (128, 256):
        xr, f = qlin.prologue_f16(x.cuda(), group)
        got = xr[:, :k].float().cpu().numpy() * np.ldexp(1.0, f.cpu().numpy().astype(np.int64))[:, None]
        ref = O.rotate_rows(x.float().numpy(), group)
        assert np.abs(got - ref).max() <= 2e-3 * np.abs(ref).max()
        amax = np.abs(xr.float().cpu().numpy()).max(axis=1)
        assert np.all((amax >= 2 ** 14) & (amax <= 2 ** 15))


@pytest.mark.parametrize("x_dtype", [torch.float16, torch.bfloat16])
def test_prologue_rows_with_zero_tiny_and_mixed_scale_groups(qlin, x_dtype):
    """Rows whose rotation groups differ wildly in scale: zero groups, all-tiny rows, one group
    2^27 below the row maximum, an all-zero row.  The row exponent is that of the row maximum and
    every group keeps fp16 precision relative to its own magnitude."""
    m, k, group = 20, 1024, 128
    g = torch.Generator().manual_seed(21)
    x = torch.randn(m, k, generator=g)
    x[1, :256] = 0
    x[1] *= 1e-4
    x[2, :128] *= 1e3
    x[2, 640:768] *= 1e-5
    x[3] = 0
    x[4, 128:] = 0
    x = x.to(x_dtype)
    xr, f = qlin.prologue_f16(x.cuda(), group)
    xr = xr[:, :k].float().cpu().numpy().astype(np.float64)
    f = f.cpu().numpy().astype(np.int64)
    ref = O.rotate_rows(x.float().numpy(), group)
    got = xr * np.ldexp(1.0, f)[:, None]
    for r in range(m):
        amax = np.abs(ref[r]).max()
        if amax == 0:
            assert f[r] == 0 and np.all(xr[r] == 0)
            continue
        assert 2 ** 14 <= np.abs(xr[r]).max() <= 2 ** 15, r  # the row maximum sets the exponent
        for c in range(0, k, group):  # each group against its own scale
            gmax = np.abs(ref[r, c:c + group]).max()
            if gmax > 0:
                assert np.abs(got[r, c:c + group] - ref[r, c:c + group]).max() <= 2e-3 * gmax, (r, c)


@pytest.mark.parametrize("x_dtype", [torch.float16, torch.bfloat16])
def test_quantize_rows_int8_bit_exact(qlin, x_dtype):
    m, k = 64, 1536
    g = torch.Generator().manual_seed(12)
    x = (torch.randn(m, k, generator=g) * torch.linspace(0.01, 50, m)[:, None]).to(x_dtype)
    x[3] = 0
    q_ref, s_ref = O.quantize_int8_rowwise(x)
    q, s = qlin.quantize_int8_rowwise(x.cuda())
    assert torch.equal(q.cpu(), q_ref)
    assert torch.equal(s.cpu(), s_ref)
    qp, _ = qlin.quantize_int8_rowwise(x.cuda(), perm=True)
    perm = np.array([0, 2, 4, 6, 1, 3, 5, 7])
    want = q_ref.numpy().reshape(m, -1, 8)[:, :, perm].reshape(m, -1)
    assert np.array_equal(qp.cpu().numpy()[:, :k], want)


def _quant_edge_rows(x_dtype, k, seed):
    """Rows that probe the quantizer's rounding: exact ties and their neighbours, scales in the
    subnormal range and below it (the divisor replaced by the smallest normal), the dtype's
    extremes, zeros, and random rows over eleven decades; plus one row with +inf and one with a NaN."""
    g = torch.Generator().manual_seed(seed)
    m = 24
    x = torch.randn(m, k, generator=g) * torch.logspace(-5, 5, m)[:, None]
    x[0] = 0
    # quotients exactly n + 0.5: s = 0.125 (row maximum 127 / 8), values (2n + 1) / 16
    ties = (torch.arange(-127, 127).float() + 0.5) * 0.125
    x[1] = ties[torch.arange(k) % ties.numel()]
    x[1, k // 2] = 15.875
    xt = x[1].to(x_dtype)
    nxt = (xt.view(torch.int16) + 1).view(x_dtype)  # the neighbour one unit further from zero
    x[2] = torch.where(torch.arange(k) % 2 == 0, nxt.float(), xt.float())
    x[2, k // 2] = 15.875
    tiny = 1e-5 if x_dtype == torch.float16 else 1e-34
    x[3] = torch.randn(k, generator=g) * tiny  # divisor in the fp16 subnormal range / near bf16's floor
    x[4] = torch.randn(k, generator=g) * tiny * 0.01  # fp16: divisor rounds to zero -> smallest normal
    big = 65504.0 if x_dtype == torch.float16 else 3.3e38
    x[5] = torch.randn(k, generator=g).clamp(-1, 1) * big
    x[5, 3] = big
    x = x.to(x_dtype)
    x[6, 5] = float("inf")
    x[7, 9 % k] = float("nan")
    return x


@pytest.mark.parametrize("x_dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("k", [8, 1004, 1536, 5120, 12288, 13824, 32768, 40000])
def test_quantize_rows_int8_edge_rows(qlin, x_dtype, k):
    """Packed quantizer (K a multiple of 8 up to 32768) and the general one (other K), both perms,
    contiguous and strided rows: codes and scales equal to the oracle's.  Rows holding inf or NaN
    follow fmaxf: the row maximum ignores a NaN, an element that is NaN or inf / inf gets -128."""
    x = _quant_edge_rows(x_dtype, k, seed=k)
    m = x.shape[0]
    # the row maximum ignores a NaN; a NaN element, and inf / inf in a row whose maximum is inf
    # (fp16 rows scaled past 65504 hold several), get -128
    q_ref, s_ref = O.quantize_int8_rowwise(torch.nan_to_num(x, nan=0.0, posinf=float("inf"), neginf=float("-inf")))
    q_ref = q_ref.numpy().copy()
    s_ref = s_ref.numpy().copy()
    q_ref[~torch.isfinite(x).numpy()] = -128
    wide = torch.zeros(m, k + 16, dtype=x_dtype)
    wide[:, 8:8 + k] = x
    for xd in (x.cuda(), wide.cuda()[:, 8:8 + k]):  # contiguous; rows 16-byte aligned with ldx = k + 16
        q, s = qlin.quantize_int8_rowwise(xd)
        assert np.array_equal(q.cpu().numpy(), q_ref)
        assert np.array_equal(s.cpu().numpy(), s_ref)
        qp, _ = qlin.quantize_int8_rowwise(xd, perm=True)
        if k % 8 == 0:
            perm = np.array([0, 2, 4, 6, 1, 3, 5, 7])
            want = q_ref.reshape(m, -1, 8)[:, :, perm].reshape(m, -1)
            assert np.array_equal(qp.cpu().numpy()[:, :k], want)
    _check_status(qlin)


def test_int8_linear_streamed_from_host_memory(qlin):
    """Host activations in, host outputs out, copies overlapped in chunks: the same rows as the
    device path (per-row prologue, no K split at this shape)."""
    m, n, k = 1000, 512, 1024
    x, q, s, b = O.cfg_int8_convrot(m, k, n, seed=3)
    want = qlin.int8_linear(x.cuda(), q.cuda(), s.cuda(), b.cuda(), torch.float16, convrot=True,
                            convrot_groupsize=128).cpu()
    xh = x.pin_memory()
    for chunks in (1, 3, 8):
        got = qlin.int8_linear_streamed(xh, q.cuda(), s.cuda(), b.cuda(), convrot=True, convrot_groupsize=128,
                                        chunks=chunks)
        torch.cuda.current_stream().synchronize()
        assert got.device.type == "cpu" and got.shape == (m, n)
        assert O.max_abs_rel(got.float().numpy(), want.float().numpy()) <= 1e-3
    with pytest.raises(NotImplementedError):
        qlin.int8_linear_streamed(x.cuda(), q.cuda(), s.cuda())


def _small_m_k(qtype, i):
    qk = O.GGUF_TYPES[qtype][1]
    return (800, 96, 576, 1024, 2080)[i] if qk == 32 else (768, 256, 1280, 2048, 512)[i]


@pytest.mark.parametrize("qtype", ALL_TYPES)
@pytest.mark.parametrize("m,n,ki", [(1, 200, 0), (2, 384, 1), (9, 130, 2), (31, 256, 3), (64, 384, 4)])
def test_small_m_kernel_matches_fp64(qlin, qtype, m, n, ki):
    """Small M (text tokens, adapter side paths: the weight-streaming kernel for M = 1, the
    tensor-core GEMM with its K split above): odd stage counts, ragged N, K not a multiple of 64,
    and calls repeated bit for bit (the K-split partials are reduced in a fixed order)."""
    k = _small_m_k(qtype, ki)
    x, raw, b, ref = _gguf_case(qtype, m, n, k, seed=m * 13 + qtype + ki)
    raw_d = torch.from_numpy(raw).cuda()
    y = qlin.gguf_linear(x.cuda(), raw_d, qtype, (n, k), bias=b.cuda())
    got = y.float().cpu().numpy()
    assert np.isfinite(got).all()
    assert O.max_abs_rel(got, ref) <= 2e-3, O.max_abs_rel(got, ref)
    y2 = qlin.gguf_linear(x.cuda(), raw_d, qtype, (n, k), bias=b.cuda())
    assert torch.equal(y, y2)
    _check_status(qlin)


@pytest.mark.parametrize("m", [1, 3, 16, 40, 64])
@pytest.mark.parametrize("out_dtype", [torch.float16, torch.bfloat16, torch.float32])
def test_small_m_int8_matches_fp64(qlin, m, out_dtype):
    n, k = 300, 1088  # 17 stages of 64, a ragged last weight tile
    x, q, s, b = O.cfg_int8_convrot(m, k, n, seed=m)
    ref = O.int8_convrot_linear_ref(x.float().numpy(), q.numpy(), s.float().numpy(), b.float().numpy(), convrot=False)
    y = qlin.int8_linear(x.cuda(), q.cuda(), s.cuda(), b.cuda(), out_dtype)
    got = y.float().cpu().numpy()
    assert np.isfinite(got).all()
    assert O.max_abs_rel(got, ref) <= TOL[out_dtype], O.max_abs_rel(got, ref)


STRADDLE = [(8, 128, 1040), (2, 70, 1104), (12, 64, 1152), (14, 130, 640), (11, 40, 1600), (23, 96, 1920),
            (20, 200, 336)]


@pytest.mark.parametrize("qtype,n,k", STRADDLE)
@pytest.mark.parametrize("m", [1, 45, 300])
def test_gguf_linear_rows_straddling_blocks(qlin, qtype, n, k, m):
    """Weights whose rows are not whole blocks (ComfyUI-GGUF's orig_shape layers: the blocks run
    over the flattened [N, K] tensor) run the linear too: decoded once by flat element to fp16
    w * 2^-e per row, then the same tensor-core GEMM.  Against gguf-py's decode in float64."""
    qk = O.GGUF_TYPES[qtype][1]
    assert k % qk != 0 and (n * k) % qk == 0
    raw = O.random_gguf_blocks(qtype, 1, n * k, seed=qtype + m)  # one flat run of blocks
    w = O.gguf_dequantize(raw, qtype, 1, n * k).reshape(n, k)
    g = torch.Generator().manual_seed(m + k)
    x = torch.randn(m, k, generator=g).to(torch.float16)
    b = (torch.randn(n, generator=g) * 0.1).to(torch.float16)
    ref = O.linear_f64(x.float().numpy(), w, b.float().numpy())
    y = qlin.gguf_linear(x.cuda(), torch.from_numpy(raw).cuda(), qtype, (n, k), bias=b.cuda())
    got = y.float().cpu().numpy()
    assert np.isfinite(got).all()
    assert O.max_abs_rel(got, ref) <= 2e-3, O.max_abs_rel(got, ref)
    _check_status(qlin)


@pytest.mark.parametrize("qtype,n,k", STRADDLE[:3])
def test_straddling_rows_decoded_exactly_once_rounded(qlin, qtype, n, k):
    """One-hot activation rows pull single weights through the straddle path: each equals the
    exact decode rounded once to fp16 at its row's power of two, RN16(w * 2^-e) * 2^e."""
    raw = O.random_gguf_blocks(qtype, 1, n * k, seed=3)
    w = O.gguf_dequantize(raw, qtype, 1, n * k).reshape(n, k).astype(np.float64)
    amax = np.abs(w).max(axis=1)
    e = np.where(amax > 0, np.frexp(amax)[1] - 15, 0)
    exact = (np.ldexp(w, -e[:, None]).astype(np.float16).astype(np.float64) * np.ldexp(1.0, e)[:, None]).T
    eye = torch.eye(k, dtype=torch.float16).cuda()
    y = qlin.gguf_linear(eye, torch.from_numpy(raw).cuda(), qtype, (n, k), out_dtype=torch.float32).cpu().numpy()
    assert np.array_equal(y.astype(np.float64), exact)
