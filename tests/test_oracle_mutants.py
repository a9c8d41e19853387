"""Mutation tests of the parity checkers (CPU only).

A parity test is only as good as its checker.  These tests plant realistic mistakes -- the ones a
decoder, a GEMM epilogue or a tile scheduler makes -- in CPU restatements (the oracle, patched for
the length of one test, or a CPU stand-in for a kernel's output) and show that the checker the
parity tests use rejects every one.  Each checker is first shown to pass on the unmutated code, so
a checker that rejects everything cannot pass for a strong one.

Nothing here runs on a GPU: the mistakes live in the oracle and in numpy stand-ins, never in a
kernel.  Mutants that a checker cannot see by design are listed with the check that does see them.
"""
import numpy as np
import pytest
import torch

import checks as C
from oracle import qlin_oracle as O

ORIG_BLOCKS = O.gguf_dequantize_blocks
ORIG_F16 = O._f16


def _rejects(check):
    with pytest.raises(AssertionError):
        check()


def _blocks(b, qtype):
    return np.ascontiguousarray(b, dtype=np.uint8).reshape(-1, O.GGUF_TYPES[qtype][2])


def _only(qtype, fn):
    """gguf_dequantize_blocks with type `qtype` decoded by `fn(blocks)` and the rest unchanged."""
    def patched(blocks, qt):
        if qt != qtype:
            return ORIG_BLOCKS(blocks, qt)
        return fn(_blocks(blocks, qt)).astype(np.float32)
    return patched


# ---------------------------------------------------------------------------------- GGUF decode
# Checker: bit-identical float32 against gguf-py 0.19.0's own decode of the committed blocks
# (tests/golden/gguf_types.npz: random blocks plus edge scales 0, -0, +-65504, subnormal, +-min).

def _check_gguf(qtype):
    raw, want = C.gguf_golden(qtype)
    C.bit_identical(O.gguf_dequantize(raw, qtype, *want.shape), want)


def _q4_0_high_nibble_first(b):
    d, qs = O._f16(b[:, 0:2]), b[:, 2:18]
    return d * (np.concatenate([qs >> 4, qs & 0xF], axis=1).astype(np.float32) - 8)


def _q8_0_unsigned_codes(b):
    return b[:, 2:34].astype(np.float32) * O._f16(b[:, 0:2])


def _q5_0_offset_15(b):
    d = O._f16(b[:, 0:2])
    q = O._nibbles32(b[:, 6:22]) | (O._bits32(b[:, 2:6]) << 4)
    return d * (q.astype(np.float32) - 15)


def _q4_k_min_added(b):
    """(d * sc) * q + dmin * m: the block minimum added instead of subtracted."""
    nb = b.shape[0]
    d, dmin = O._f16(b[:, 0:2]), O._f16(b[:, 2:4])
    sc, mn = O.q4k_scale_min(b[:, 4:16])
    qs = b[:, 16:144].reshape(nb, 4, 1, 32)
    q = np.concatenate([qs & 0xF, qs >> 4], axis=2).reshape(nb, 8, 32).astype(np.float32)
    return ((d * sc).reshape(nb, 8, 1) * q + (dmin * mn).reshape(nb, 8, 1)).reshape(nb, 256)


def _q6_k_offset_31(b):
    nb = b.shape[0]
    d = O._f16(b[:, 208:210])
    ds = (d * b[:, 192:208].view(np.int8).astype(np.float32)).reshape(nb, 16, 1)
    w = ORIG_BLOCKS(b, 14).reshape(nb, 16, 16)
    return (w + ds).reshape(nb, 256)  # (q - 31) * ds, formed as w + ds


def _q3_k_hmask_inverted(b):
    nb = b.shape[0]
    d = O._f16(b[:, 108:110])
    dl = (d * O.q3k_scales(b[:, 96:108])).reshape(nb, 16, 1)
    lo = O._crumbs256(b[:, 32:96])
    hm = b[:, 0:32].reshape(nb, 1, 32)
    hbit = np.concatenate([(hm >> i) & 1 for i in range(8)], axis=1).reshape(nb, 256)
    q = (lo.astype(np.int8) - (hbit << 2).astype(np.int8)).reshape(nb, 16, 16).astype(np.float32)
    return (dl * q).reshape(nb, 256)


def _q2_k_min_from_low_nibble(b):
    nb = b.shape[0]
    sc = b[:, 0:16]
    d, dmin = O._f16(b[:, 80:82]), O._f16(b[:, 82:84])
    dl = (d * (sc & 0xF).astype(np.float32)).reshape(nb, 16, 1)
    ml = (dmin * (sc & 0xF).astype(np.float32)).reshape(nb, 16, 1)
    q = O._crumbs256(b[:, 16:80]).reshape(nb, 16, 16).astype(np.float32)
    return (dl * q - ml).reshape(nb, 256)


def _q5_k_fifth_bit_reversed(b):
    nb = b.shape[0]
    d, dmin = O._f16(b[:, 0:2]), O._f16(b[:, 2:4])
    sc, mn = O.q4k_scale_min(b[:, 4:16])
    qs = b[:, 48:176].reshape(nb, 4, 1, 32)
    lo = np.concatenate([qs & 0xF, qs >> 4], axis=2).reshape(nb, 8, 32)
    qh = b[:, 16:48].reshape(nb, 1, 32)
    hi = np.concatenate([(qh >> (7 - s)) & 1 for s in range(8)], axis=1)
    q = (lo | (hi << 4)).astype(np.float32)
    return ((d * sc).reshape(nb, 8, 1) * q - (dmin * mn).reshape(nb, 8, 1)).reshape(nb, 256)


def _iq4_nl_table_off_by_one(b):
    d, qs = O._f16(b[:, 0:2]), b[:, 2:18]
    nib = np.concatenate([qs & 0xF, qs >> 4], axis=1)
    return d * O.IQ4_NL_VALUES[np.minimum(nib + 1, 15)]


def _q4k_pairs_4_7_high_nibble(scales12):
    s = scales12.astype(np.uint8).reshape(-1, 3, 4)
    d, m, md = s[:, 0], s[:, 1], s[:, 2]
    sc = np.concatenate([d & 0x3F, (md >> 4) | ((d >> 2) & 0x30)], axis=-1)
    mn = np.concatenate([m & 0x3F, (md & 0x0F) | ((m >> 2) & 0x30)], axis=-1)
    return sc.astype(np.float32), mn.astype(np.float32)


def _nibbles_interleaved(qs16):
    """byte i -> values 2i, 2i+1 (the other common nibble order) instead of i, i + 16."""
    return np.stack([qs16 & 0xF, qs16 >> 4], axis=2).reshape(qs16.shape[0], 32)


def _f16_read_as_bf16(raw2):
    u = np.ascontiguousarray(raw2).view(np.uint16).astype(np.uint32) << 16
    return u.view(np.float32)


def _f16_subnormals_flushed(raw2):
    v = ORIG_F16(raw2)
    return np.where(np.abs(v) < np.float32(2.0 ** -14), np.float32(0.0) * np.sign(v), v).astype(np.float32)


GGUF_MUTANTS = {
    # name: (type the checker runs on, attribute of the oracle patched, replacement)
    "Q4_0 high nibble first": (2, "gguf_dequantize_blocks", _only(2, _q4_0_high_nibble_first)),
    "Q8_0 codes read unsigned": (8, "gguf_dequantize_blocks", _only(8, _q8_0_unsigned_codes)),
    "Q5_0 offset 15 not 16": (6, "gguf_dequantize_blocks", _only(6, _q5_0_offset_15)),
    "Q4_K minimum added": (12, "gguf_dequantize_blocks", _only(12, _q4_k_min_added)),
    "Q6_K offset 31 not 32": (14, "gguf_dequantize_blocks", _only(14, _q6_k_offset_31)),
    "Q3_K hmask polarity inverted": (11, "gguf_dequantize_blocks", _only(11, _q3_k_hmask_inverted)),
    "Q2_K min from the low nibble": (10, "gguf_dequantize_blocks", _only(10, _q2_k_min_from_low_nibble)),
    "Q5_K fifth bit order reversed": (13, "gguf_dequantize_blocks", _only(13, _q5_k_fifth_bit_reversed)),
    "IQ4_NL table index off by one": (20, "gguf_dequantize_blocks", _only(20, _iq4_nl_table_off_by_one)),
    "Q4_K pairs 4-7 nibbles swapped": (12, "q4k_scale_min", _q4k_pairs_4_7_high_nibble),
    "Q5_K pairs 4-7 nibbles swapped": (13, "q4k_scale_min", _q4k_pairs_4_7_high_nibble),
    "Q4_1 nibbles interleaved": (3, "_nibbles32", _nibbles_interleaved),
    "IQ4_XS nibbles interleaved": (23, "_nibbles32", _nibbles_interleaved),
    "IQ4_XS scales without -32": (23, "iq4xs_scales", lambda blk: ORIG_IQ4XS(blk) + 32),
    "Q3_K scales without -32": (11, "q3k_scales", lambda s: ORIG_Q3K(s) + 32),
    "fp16 scale read as bf16 (Q8_0)": (8, "_f16", _f16_read_as_bf16),
    "fp16 scale read as bf16 (Q6_K)": (14, "_f16", _f16_read_as_bf16),
}
ORIG_IQ4XS = O.iq4xs_scales
ORIG_Q3K = O.q3k_scales
# Subnormal fp16 scales flushed to zero (a decoder built with flush-to-zero): the golden rows
# carry the smallest subnormal as an edge scale in every type's first scale field.
FTZ_TYPES = sorted(O.GGUF_TYPES)


@pytest.mark.parametrize("qtype", sorted(O.GGUF_TYPES))
def test_gguf_checker_passes_the_oracle(qtype):
    _check_gguf(qtype)


@pytest.mark.parametrize("name", sorted(GGUF_MUTANTS))
def test_gguf_checker_rejects(monkeypatch, name):
    qtype, attr, repl = GGUF_MUTANTS[name]
    monkeypatch.setattr(O, attr, repl)
    _rejects(lambda: _check_gguf(qtype))


@pytest.mark.parametrize("qtype", FTZ_TYPES)
def test_gguf_checker_rejects_flushed_subnormal_scales(monkeypatch, qtype):
    monkeypatch.setattr(O, "_f16", _f16_subnormals_flushed)
    _rejects(lambda: _check_gguf(qtype))


# ---------------------------------------------------------------------------------- row exponent
# Checker: the decoded fp16 weight w * 2^-e uses the top of fp16's range without overflowing
# (bound * 2^-e in (2^14, 2^15]) and the scale-only bound covers every decoded |w|.

def _check_row_exponent(qtype):
    C.row_exponent_check(qtype)


ORIG_EXPONENT = O.gguf_row_exponent
ORIG_BOUND = O.gguf_row_bound


def _bound_without_min(raw, qtype, n, k):
    """Q4_K bound d * sc * 15 alone (the block-minimum term forgotten)."""
    b = np.asarray(raw, dtype=np.uint8).reshape(n, k // 256, 144)
    d = np.abs(O._f16(b[..., 0:2])[..., 0].astype(np.float64))
    sc, _ = O.q4k_scale_min(b[..., 4:16].reshape(-1, 12))
    return (d[..., None] * sc.reshape(n, k // 256, 8) * 15).max(axis=-1).max(axis=1)


EXPONENT_MUTANTS = {
    "exponent one too small (precision lost)": ("gguf_row_exponent", lambda bd: ORIG_EXPONENT(bd) + 1),
    "exponent one too large (fp16 overflow)": ("gguf_row_exponent", lambda bd: ORIG_EXPONENT(bd) - 1),
    "Q4_K bound without the minimum term": ("gguf_row_bound", _bound_without_min),
}


@pytest.mark.parametrize("qtype", sorted(O.GGUF_TYPES))
def test_row_exponent_checker_passes_the_oracle(qtype):
    _check_row_exponent(qtype)


@pytest.mark.parametrize("name", sorted(EXPONENT_MUTANTS))
def test_row_exponent_checker_rejects(monkeypatch, name):
    attr, repl = EXPONENT_MUTANTS[name]
    monkeypatch.setattr(O, attr, repl)
    _rejects(lambda: _check_row_exponent(12))


# ---------------------------------------------------------------------------------- kitchen grid
# Checker: the int8 grid equals the reference port's grid (tests/golden/kitchen_w4a8.npz).

def _check_kitchen(fmt, bits):
    import os
    z = np.load(os.path.join(C.GOLD, "kitchen_w4a8.npz"))
    cb = z[f"{fmt}_codebook"] if f"{fmt}_codebook" in z else None
    grid = O.kitchen_int8_grid(z[f"{fmt}_q"], z[f"{fmt}_s_rel"], 1024, bits, 16, cb)
    assert np.array_equal(grid, z[f"{fmt}_grid"]), "int8 grid differs"


ORIG_UNPACK = O.unpack_codes_kitchen
ORIG_E4M3 = O.e4m3_to_float


def _unpack_odd_column_low(qdata, k, bits):
    c = ORIG_UNPACK(qdata, k, bits)
    lo, hi = c[:, 0::2] & 0xF, c[:, 1::2] & 0xF
    out = c.copy()
    out[:, 0::2] = (c[:, 0::2] & ~0xF) | hi
    out[:, 1::2] = (c[:, 1::2] & ~0xF) | lo
    return out


def _unpack_high_planes_reversed(qdata, k, bits):
    packed = np.asarray(qdata).view(np.uint8).astype(np.int32)
    c = ORIG_UNPACK(qdata, k, 4) if bits == 6 else ORIG_UNPACK(qdata, k, bits)
    if bits == 6:
        hi = packed[:, k // 2:]
        for j in range(4):
            c[:, j::4] |= ((hi >> (2 * (3 - j))) & 0x3) << 4
    return c


def _e4m3_no_subnormals(raw):
    v = ORIG_E4M3(raw)
    b = np.asarray(raw).view(np.uint8)
    return np.where((b & 0x78) == 0, np.float32(0.0), v).astype(np.float32)


def _e4m3_bias_8(raw):
    return (ORIG_E4M3(raw) * np.float32(0.5)).astype(np.float32)


KITCHEN_MUTANTS = {
    "W4A8 nibble pair swapped": ("w4a8", 4, "unpack_codes_kitchen", _unpack_odd_column_low),
    "W6A8 nibble pair swapped": ("w6a8", 6, "unpack_codes_kitchen", _unpack_odd_column_low),
    "W6A8 high 2-bit planes reversed": ("w6a8", 6, "unpack_codes_kitchen", _unpack_high_planes_reversed),
    "e4m3 group scale with exponent bias 8": ("w4a8", 4, "e4m3_to_float", _e4m3_bias_8),
}


@pytest.mark.parametrize("fmt,bits", [("w4a8", 4), ("w6a8", 6)])
def test_kitchen_checker_passes_the_oracle(fmt, bits):
    _check_kitchen(fmt, bits)


@pytest.mark.parametrize("name", sorted(KITCHEN_MUTANTS))
def test_kitchen_checker_rejects(monkeypatch, name):
    fmt, bits, attr, repl = KITCHEN_MUTANTS[name]
    monkeypatch.setattr(O, attr, repl)
    _rejects(lambda: _check_kitchen(fmt, bits))


def test_e4m3_subnormal_flush_is_seen_by_the_code_table_check(monkeypatch):
    """The golden group scales hold no e4m3 subnormal (the smallest is 0.75), so the grid check
    cannot see a decoder that flushes them; the all-256-codes check against torch's
    float8_e4m3fn does."""
    monkeypatch.setattr(O, "e4m3_to_float", _e4m3_no_subnormals)
    _check_kitchen("w6a8", 6)  # survives the grid check
    _rejects(C.e4m3_code_table)
    monkeypatch.undo()
    C.e4m3_code_table()


# ---------------------------------------------------------------------------------- INT8 quantizer
# Checker: codes and scales hash-identical to the reference's self-test records
# (tests/golden/selftest_hashes.json), for the row-wise and the ConvRot (H-256) quantizer.

def _check_quantizers():
    import json
    import os
    hashes = json.load(open(os.path.join(C.GOLD, "selftest_hashes.json")))
    inputs = O.selftest_inputs()
    for case in ("gauss_96x1024", "chunked_4200x1024"):
        f = hashes["cases"][case]["formats"]
        q, s = O.quantize_int8_rowwise(inputs[case].clone())
        assert C.sha(q) == f["int8_rowwise"]["q"] and C.sha(s) == f["int8_rowwise"]["scale"], "row-wise"
        q, s = O.quantize_int8_convrot(inputs[case], 256, "h4")
        assert C.sha(q) == f["int8_convrot"]["q"], "convrot codes"


def _quantize_truncating(x):
    abs_max = x.abs().amax(dim=-1, keepdim=True)
    scale = (abs_max.float() / 127.0).clamp(min=1e-30)
    q = (x / scale.to(x.dtype)).trunc().clamp(-128, 127).to(torch.int8)
    return q, scale


def _quantize_by_128(x):
    abs_max = x.abs().amax(dim=-1, keepdim=True)
    scale = (abs_max.float() / 128.0).clamp(min=1e-30)
    q = (x / scale.to(x.dtype)).round().clamp(-128, 127).to(torch.int8)
    return q, scale


def _quantize_times_reciprocal(x):
    """x * (1/s) instead of x / s: one extra rounding flips codes that sit near a half."""
    abs_max = x.abs().amax(dim=-1, keepdim=True)
    scale = (abs_max.float() / 127.0).clamp(min=1e-30)
    q = (x * (1.0 / scale.to(x.dtype))).round().clamp(-128, 127).to(torch.int8)
    return q, scale


ORIG_HADAMARD = O.hadamard


def _hadamard_one_row_negated(size, kind="auto"):
    h = ORIG_HADAMARD(size, kind).copy()
    h[size - 1] *= -1
    return h


QUANT_MUTANTS = {
    "codes truncated, not rounded": ("quantize_int8_rowwise", _quantize_truncating),
    "scale absmax / 128": ("quantize_int8_rowwise", _quantize_by_128),
    "x times the reciprocal scale": ("quantize_int8_rowwise", _quantize_times_reciprocal),
    "H-256 rotation built as Sylvester": ("hadamard", lambda size, kind="auto": O.hadamard_sylvester(size)),
    "H-256 last row negated": ("hadamard", _hadamard_one_row_negated),
}


def test_quantizer_checker_passes_the_oracle():
    _check_quantizers()


@pytest.mark.parametrize("name", sorted(QUANT_MUTANTS))
def test_quantizer_checker_rejects(monkeypatch, name):
    attr, repl = QUANT_MUTANTS[name]
    monkeypatch.setattr(O, attr, repl)
    _rejects(_check_quantizers)


# ---------------------------------------------------------------------------------- GEMM outputs
# CPU stand-ins for a kernel's output, each with one mistake a tiled quantized GEMM can make,
# judged by the checkers of the GPU parity tests: A8 integer-exact on sampled rows (configurations
# 3 and 4), Q8_0 integer-exact (configuration 1), one-hot decoded weights, and the 2e-3
# tolerance on random data.

A8_M, A8_K, A8_N, A8_GROUP = 400, 1024, 256, 128  # two full 192-token tiles and a ragged one


def _a8_standin(x, wq, s, bias, group, mutate=None):
    """fp32 output of a W4A8 linear computed from exact group partials, with `mutate` applied."""
    parts = O.int_group_partials(x.astype(np.int64), wq, group).astype(np.float64)  # [G, M, N]
    scale = np.asarray(s, dtype=np.float64).T[:, None, :]  # [G, 1, N]
    b = np.asarray(bias, dtype=np.float64)
    if mutate is None:
        return (np.sum(parts * scale, axis=0) + b).astype(np.float32)
    return mutate(parts, scale, b, x, wq, s, group).astype(np.float32)


def _tile_rows_unwritten(y, lo, hi):
    y = y.copy()
    y[lo:hi] = np.nan
    return y


def _channels_unwritten(y, lo, hi):
    y = y.copy()
    y[:, lo:hi] = np.nan
    return y


A8_MUTANTS = {
    "group scales one group late": lambda p, sc, b, *a: np.sum(p * np.roll(sc, 1, axis=0), axis=0) + b,
    "scale index from the K step (group read twice as long)":
        lambda p, sc, b, *a: np.sum(p * sc[np.arange(len(sc)) // 2], axis=0) + b,
    "accumulator not cleared at a group start":
        lambda p, sc, b, *a: np.sum(np.cumsum(p, axis=0) * sc, axis=0) + b,
    "last 64-column K stage skipped":
        lambda p, sc, b, x, wq, s, g: np.sum(O.int_group_partials(
            x.astype(np.int64), np.concatenate([wq[:, :-64], 0 * wq[:, -64:]], axis=1), g) * sc, axis=0) + b,
    "weight nibble pair swapped in the decoder":
        lambda p, sc, b, x, wq, s, g: np.sum(O.int_group_partials(
            x.astype(np.int64), wq.reshape(wq.shape[0], -1, 2)[:, :, ::-1].reshape(wq.shape), g) * sc, axis=0) + b,
    "ragged last token tile not written":
        lambda p, sc, b, *a: _tile_rows_unwritten(np.sum(p * sc, axis=0) + b, 384, 400),
    "one 128-channel tile not written":
        lambda p, sc, b, *a: _channels_unwritten(np.sum(p * sc, axis=0) + b, 128, 256),
    "second token tile holds the first tile's rows":
        lambda p, sc, b, *a: np.concatenate([(np.sum(p * sc, axis=0) + b)[:192]] * 2
                                            + [(np.sum(p * sc, axis=0) + b)[384:]], axis=0),
    "epilogue reads the next token's accumulator":
        lambda p, sc, b, *a: np.roll(np.sum(p * sc, axis=0), -1, axis=0) + b,
    "bias dropped": lambda p, sc, b, *a: np.sum(p * sc, axis=0),
    "bias added twice": lambda p, sc, b, *a: np.sum(p * sc, axis=0) + 2 * b,
}


def _a8_check(mutate=None):
    x, wq, s, bias = C.a8_integer_case(A8_M, A8_K, A8_N, 4, A8_GROUP)
    y = _a8_standin(x, wq, s, bias, A8_GROUP, mutate)
    C.a8_exact("stand-in", y, x, wq, s, A8_GROUP, bias, C.sample_rows(A8_M))


def test_a8_exact_checker_passes_the_exact_output():
    _a8_check()


@pytest.mark.parametrize("name", sorted(A8_MUTANTS))
def test_a8_exact_checker_rejects(name):
    _rejects(lambda: _a8_check(A8_MUTANTS[name]))


def test_a8_single_unsampled_row_is_seen_by_the_all_rows_tests():
    """The full-shape tests compare a sample of rows (every token tile, not every row), so one
    wrong row outside the sample passes them; the smaller-shape GPU tests compare every row."""
    x, wq, s, bias = C.a8_integer_case(A8_M, A8_K, A8_N, 4, A8_GROUP)
    y = _a8_standin(x, wq, s, bias, A8_GROUP)
    rows = C.sample_rows(A8_M)
    off = next(r for r in range(A8_M) if r not in set(rows))
    y[off] += 1.0
    C.a8_exact("sampled rows", y, x, wq, s, A8_GROUP, bias, rows)  # survives the sample
    _rejects(lambda: C.a8_exact("all rows", y, x, wq, s, A8_GROUP, bias, np.arange(A8_M)))


# Q8_0 integer-exact (configuration 1's checker): scale-1 blocks, integer activations and bias.
Q8_M, Q8_K, Q8_N = 48, 1024, 96


def _q8_standin(mutate=None):
    x, raw, bias, want = C.q8_0_integer_case(Q8_M, Q8_K, Q8_N)
    wn, e = O.gguf_normalized_fp16(raw, 8, Q8_N, Q8_K)  # the fp16 operand the tensor cores read
    wf = wn.astype(np.float64)
    xf = x.astype(np.float64)
    if mutate is None:
        acc = xf @ wf.T
    else:
        acc = mutate(xf, wf)
    y = np.ldexp(acc, e[None, :]) + bias.astype(np.float64)[None, :]
    return y.astype(np.float32), want


def _fp16_accumulate(xf, wf, step=16):
    """Partial sums of each 16-wide K step added into an fp16 accumulator."""
    acc = np.zeros((xf.shape[0], wf.shape[0]), dtype=np.float16)
    with np.errstate(over="ignore"):
        for k0 in range(0, xf.shape[1], step):
            acc = (acc.astype(np.float32) + (xf[:, k0:k0 + step] @ wf[:, k0:k0 + step].T).astype(np.float32)
                   ).astype(np.float16)
    return acc.astype(np.float64)


Q8_MUTANTS = {
    "fp16 accumulator": _fp16_accumulate,
    "second K split's partial dropped": lambda xf, wf: xf[:, :Q8_K // 2] @ wf[:, :Q8_K // 2].T,
    "K split partials added twice": lambda xf, wf: xf @ wf.T + xf[:, Q8_K // 2:] @ wf[:, Q8_K // 2:].T,
    "row exponent applied twice": lambda xf, wf: np.ldexp(xf @ wf.T, 7),
    "channel tiles swapped": lambda xf, wf: np.roll(xf @ wf.T, Q8_N // 2, axis=1),
    "activations read as the previous row": lambda xf, wf: np.roll(xf, 1, axis=0) @ wf.T,
}


def test_q8_integer_checker_passes_the_exact_output():
    y, want = _q8_standin()
    C.integer_exact("stand-in", y, want)


@pytest.mark.parametrize("name", sorted(Q8_MUTANTS))
def test_q8_integer_checker_rejects(name):
    y, want = _q8_standin(Q8_MUTANTS[name])
    _rejects(lambda: C.integer_exact("stand-in", y, want))


# 2e-3 tolerance on random data, and the one-hot decoded-weight check.
def _random_case(qtype, m=64, k=3072, n=256):
    g = torch.Generator().manual_seed(5)
    x = torch.randn(m, k, generator=g).to(torch.float16).float().numpy().astype(np.float64)
    raw = O.random_gguf_blocks(qtype, n, k, seed=3)
    ref = O.linear_f64(x, O.gguf_dequantize(raw, qtype, n, k))
    wn, e = O.gguf_normalized_fp16(raw, qtype, n, k)
    return x, raw, ref, wn.astype(np.float64), e


TOL_MUTANTS = {
    "row exponent not re-applied": lambda x, wn, e: x @ wn.T,
    "one 256-value superblock of K skipped":
        lambda x, wn, e: np.ldexp(x[:, 256:] @ wn[:, 256:].T, e[None, :]),
    "row exponents of the next channel": lambda x, wn, e: np.ldexp(x @ wn.T, np.roll(e, -1)[None, :]) * 2.0,
    "activations read one token row late": lambda x, wn, e: np.ldexp(np.roll(x, 1, axis=0) @ wn.T, e[None, :]),
}


def _tolerance_check(qtype, mutate=None):
    x, raw, ref, wn, e = _random_case(qtype)
    y = np.ldexp(x @ wn.T, e[None, :]) if mutate is None else mutate(x, wn, e)
    with np.errstate(over="ignore"):
        y16 = y.astype(np.float16)  # an fp16 output overflows to inf, as the kernel's would
    C.finite_and_close("stand-in", y16, ref)


@pytest.mark.parametrize("qtype", [2, 12])
def test_tolerance_checker_passes_the_exact_output(qtype):
    _tolerance_check(qtype)


@pytest.mark.parametrize("name", sorted(TOL_MUTANTS))
def test_tolerance_checker_rejects(name):
    _rejects(lambda: _tolerance_check(12, TOL_MUTANTS[name]))


@pytest.mark.parametrize("qtype", [2, 6, 8, 20])
def test_bf16_weights_pass_the_tolerance_but_not_the_onehot_check(qtype):
    """Decoded weights rounded to bf16 instead of fp16 land at the edge of the 2e-3 tolerance on
    random data (1.7e-3 to 2.2e-3 here, by type), so the tolerance alone does not reliably see
    them; one-hot activation rows read single weights, which must be RN16(w 2^-e) 2^e exactly for
    the types decoded with one rounding."""
    n, k = 64, 512
    x, raw, ref, wn, e = _random_case(qtype, m=64, k=3072, n=256)
    w = O.gguf_dequantize(raw, qtype, 256, 3072)
    wb = torch.from_numpy(np.ldexp(w, -e[:, None]).astype(np.float32)).to(torch.bfloat16).double().numpy()
    err = O.max_abs_rel(np.ldexp(x @ wb.T, e[None, :]).astype(np.float16), ref)
    assert 1e-3 < err < 3e-3, err  # the size of a bf16 rounding, next to the 2e-3 bound

    raw = O.random_gguf_blocks(qtype, n, k, seed=70 + qtype)
    w = O.gguf_dequantize(raw, qtype, n, k)
    e = O.gguf_row_exponent(O.gguf_row_bound(raw, qtype, n, k))
    wb = torch.from_numpy(np.ldexp(w, -e[:, None]).astype(np.float32)).to(torch.bfloat16).float().numpy()
    y_onehot = np.ldexp(wb, e[:, None]).T.astype(np.float32)  # identity rows through the linear
    rows = slice(0, k)
    _rejects(lambda: C.onehot_exact("bf16 weights", y_onehot[rows], raw, qtype, n, k, rows))
    wn, e = O.gguf_normalized_fp16(raw, qtype, n, k)
    C.onehot_exact("fp16 weights", np.ldexp(wn.astype(np.float32), e[:, None]).T[rows], raw, qtype, n, k, rows)
