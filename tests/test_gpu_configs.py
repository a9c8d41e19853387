"""GPU parity at the benchmark configurations' own shapes (the shapes the bench times), so the
planner's large-shape choices -- 192 / 256-token tiles, CTA pairs, K splits, 96 exact int32 group
sums along K = 12288, ragged token tiles at M = 3240 -- are the code paths that are checked.

The CPU reference covers a strided sample of token rows that hits every token tile (rows 61 apart,
the last row of every 192-row span and the last row), across all output channels, in float64 (or
exact integer arithmetic); outputs come from freshly poisoned allocations (conftest), and every
sampled value must be finite.  Each test prints its max-abs-rel.

  1  GGUF Q8_0 / Q4_0, X [256, 3072] x W [3072, 3072], the configuration's scale distributions
  2  INT8 ConvRot H-128, X [4096, 3072] (1% outlier channels x20) x W int8 [12288, 3072], fp16 out
  3  W4A8 g128, X [4096, 12288] x W [3072, 12288]
  4  W6A8 g64 ("four values per three bytes"), X [3240, 5120] x W [13824, 5120] and the reverse
     projection X [3240, 13824] x W [5120, 13824]
  5  MMDiT-stack layers: Q4_K QKV X [4608, 3072] x W [9216, 3072] and Q6_K MLP-down
     X [4608, 12288] x W [3072, 12288]

Configuration 1 is also checked integer-exact (Q8_0 blocks of scale 1, integer activations and
bias, every output equal to the exact integer).  Configurations 3 and 4 are checked twice:
int32-exact (integer activations whose row maximum is 127 quantize with scale exactly 1;
power-of-two group scales; an integer bias; fp32 output must equal the exact integer sum bit for
bit) and on the configuration's random data, where the GPU's own per-token
int8 activations (bit-identical to the oracle's quantizer on the sampled rows) feed an exact
integer reference and the fp16 output must be within 2e-3 of it.
"""
import numpy as np
import pytest
import torch

import checks as C
from checks import finite_and_close as _finite_and_close, group_sums_f64 as _group_sums_f64, sample_rows
from oracle import qlin_oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def qlin():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    import qlin as q
    return q


def _status(qlin):
    code, where = qlin.device_status(reset=True)
    assert code == 0, f"a kernel timed out waiting (where={where:#x})"


# ------------------------------------------------------------------------------ configuration 1
@pytest.mark.parametrize("qtype", [8, 2])
def test_cfg1_gguf_256x3072x3072(qlin, qtype):
    m, k, n = 256, 3072, 3072
    x, raw = O.cfg_gguf(m, k, n, qtype=qtype, seed=0)
    w = O.gguf_dequantize(raw, qtype, n, k)
    ref = O.linear_f64(x.float().numpy(), w)
    y = qlin.gguf_linear(x.cuda(), torch.from_numpy(raw).cuda(), qtype, (n, k))
    assert y.dtype == torch.float16 and y.shape == (m, n)
    _finite_and_close(f"cfg1 {O.GGUF_TYPES[qtype][0]}", y.float().cpu().numpy(), ref)
    # M = 1 and 16 (text tokens / adapter side paths) of the same weight: the small-M path
    for mm in (1, 16):
        ys = qlin.gguf_linear(x[:mm].cuda(), torch.from_numpy(raw).cuda(), qtype, (n, k))
        _finite_and_close(f"cfg1 {O.GGUF_TYPES[qtype][0]} M={mm}", ys.float().cpu().numpy(), ref[:mm])
    _status(qlin)


@pytest.mark.parametrize("m", [256, 16, 1])
def test_cfg1_q8_0_integer_exact(qlin, m):
    """Q8_0 blocks of scale 1 with integer codes, integer activations and an integer bias: the fp32
    output must equal the exact integer answer in every row and channel, whatever the tile shape,
    K split or accumulation order (an fp16 accumulator, a dropped K stage or split, a misplaced
    tile or a doubled bias all change it)."""
    k, n = 3072, 3072
    x, raw, bias, want = C.q8_0_integer_case(m, k, n)
    y = qlin.gguf_linear(torch.from_numpy(x).cuda(), torch.from_numpy(raw).cuda(), 8, (n, k),
                         bias=torch.from_numpy(bias).cuda(), out_dtype=torch.float32)
    C.integer_exact(f"cfg1 Q8_0 integer M={m}", y.cpu().numpy(), want)
    _status(qlin)


# ------------------------------------------------------------------------------ configuration 2
def test_cfg2_int8_convrot_full_shape(qlin):
    m, k, n = 4096, 3072, 12288
    x, q, s, b = O.cfg_int8_convrot(m, k, n, seed=0)
    y = qlin.int8_linear(x.cuda(), q.cuda(), s.cuda(), b.cuda(), torch.float16, convrot=True, convrot_groupsize=128)
    rows = sample_rows(m)
    ref = O.int8_convrot_linear_ref(x[rows].float().numpy(), q.numpy(), s.float().numpy(), b.float().numpy(),
                                    group=128)
    got = y.float().cpu().numpy()
    assert np.isfinite(got).all()
    _finite_and_close("cfg2 int8 convrot H-128", got[rows], ref)
    _status(qlin)


# ------------------------------------------------------------------------------ configurations 3 and 4
A8_CASES = {
    "cfg3_w4a8": (4096, 12288, 3072, 4, 128),
    "cfg4_w6a8_fwd": (3240, 5120, 13824, 6, 64),
    "cfg4_w6a8_rev": (3240, 13824, 5120, 6, 64),
}


def _pack(wq, bits):
    return O.pack_w4_uniform(wq).view(np.uint8) if bits == 4 else O.pack_w6_interleaved(wq)


@pytest.mark.parametrize("case", sorted(A8_CASES))
def test_a8_int32_exact_full_shape(qlin, case):
    m, k, n, bits, group = A8_CASES[case]
    x, wq, s, bias = C.a8_integer_case(m, k, n, bits, group)
    y = qlin.w4a8_linear(torch.from_numpy(x).to(torch.float16).cuda(), torch.from_numpy(_pack(wq, bits).copy()).cuda(),
                         torch.from_numpy(s).cuda(), bits=bits, group_size=group, bias=torch.from_numpy(bias).cuda(),
                         out_dtype=torch.float32)
    rows = sample_rows(m)
    C.a8_exact(case, y.cpu().numpy(), x, wq, s, group, bias, rows)
    print(f"{case} int32-exact: {len(rows)} sampled rows x {n} channels bit-identical, {k // group} groups along K={k}")
    _status(qlin)


@pytest.mark.parametrize("case", sorted(A8_CASES))
def test_a8_random_full_shape(qlin, case):
    m, k, n, bits, group = A8_CASES[case]
    if bits == 4:
        x, wq, s = O.cfg_w4a8(m, k, n, seed=0, group=group)
    else:
        x, wq, s = O.cfg_w6a8(m, k, n, seed=0, group=group)
    g = torch.Generator().manual_seed(3)
    b = (torch.randn(n, generator=g) * 0.01).to(torch.float16)
    xd = x.cuda()
    y = qlin.w4a8_linear(xd, torch.from_numpy(_pack(wq, bits).copy()).cuda(), s.cuda(), bits=bits, group_size=group,
                         bias=b.cuda())
    assert y.dtype == torch.float16
    rows = sample_rows(m)
    # the GPU's own activation codes and scales, bit-identical to the oracle's quantizer
    xq, sx = qlin.quantize_int8_rowwise(xd)
    xq, sx = xq.cpu().numpy()[rows], sx.cpu().numpy()[rows]
    q_ref, s_ref = O.quantize_int8_rowwise(x[rows])
    assert np.array_equal(xq, q_ref.numpy()) and np.array_equal(sx, s_ref.numpy())
    ref = _group_sums_f64(xq, wq, s.numpy(), group) * sx.astype(np.float64) + b.double().numpy()[None, :]
    got = y.float().cpu().numpy()
    assert np.isfinite(got).all()
    _finite_and_close(f"{case} random", got[rows], ref)
    _status(qlin)


# ------------------------------------------------------------------------------ configuration 5
@pytest.mark.parametrize("name,qtype,n,k", [("qkv", 12, 9216, 3072), ("down", 14, 3072, 12288)])
def test_cfg5_mmdit_layers_full_shape(qlin, name, qtype, n, k):
    m = 4608
    g = torch.Generator().manual_seed(5)
    x = torch.randn(m, k, generator=g).to(torch.float16)
    raw = O.random_gguf_blocks(qtype, n, k, seed=50 + qtype)
    y = qlin.gguf_linear(x.cuda(), torch.from_numpy(raw).cuda(), qtype, (n, k))
    got = y.float().cpu().numpy()
    assert np.isfinite(got).all()
    rows = sample_rows(m)
    ref = O.linear_f64(x[rows].float().numpy(), O.gguf_dequantize(raw, qtype, n, k))
    _finite_and_close(f"cfg5 {name} {O.GGUF_TYPES[qtype][0]}", got[rows], ref)
    _status(qlin)
