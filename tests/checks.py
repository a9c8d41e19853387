"""The checkers the parity tests judge a result with, in one place so the CPU mutation tests
(test_oracle_mutants.py) exercise exactly the code the GPU tests use.

Each checker raises AssertionError on a mismatch and returns quietly otherwise."""
import hashlib
import os

import numpy as np
import torch

from oracle import qlin_oracle as O

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
TOL_F16 = 2e-3


def sha(t):
    if isinstance(t, torch.Tensor):
        t = t.contiguous()
        if t.dtype == torch.float8_e4m3fn:
            t = t.view(torch.uint8)
        t = t.numpy()
    return hashlib.sha256(np.ascontiguousarray(t).tobytes()).hexdigest()


def sample_rows(m):
    """Rows 61 apart, the last row of every 192-row span and the last row: every token tile of
    every size the planner picks (16 .. 256) holds at least one sampled row."""
    return np.array(sorted(set(range(0, m, 61)) | set(range(191, m, 192)) | {m - 1}))


def finite_and_close(name, got, ref, tol=TOL_F16):
    """All values finite and max-abs-rel within `tol` (2e-3 for fp16 outputs)."""
    got = np.asarray(got, dtype=np.float64)
    assert np.isfinite(got).all(), f"{name}: non-finite outputs (a tile was not written)"
    err = O.max_abs_rel(got, ref)
    print(f"{name}: max-abs-rel {err:.3e} over {got.shape[0]} sampled rows x {got.shape[1]} channels")
    assert err <= tol, (name, err)
    return err


def group_sums_f64(xq, wq, scales, group):
    """sum_g s[n, g] * P_g[m, n] with every P_g formed exactly (float64 holds these integer dot
    products exactly: |P_g| < 2^22) and the scaled sum accumulated in float64."""
    xq = np.asarray(xq, dtype=np.float64)
    wq = np.asarray(wq, dtype=np.float64)
    s = np.asarray(scales, dtype=np.float64)
    y = np.zeros((xq.shape[0], wq.shape[0]))
    for g in range(wq.shape[1] // group):
        sl = slice(g * group, (g + 1) * group)
        y += (xq[:, sl] @ wq[:, sl].T) * s[:, g][None, :]
    return y


def bit_identical(got, want):
    """Same float32 bit patterns (NaN payloads and signed zeros included)."""
    got = np.ascontiguousarray(got, dtype=np.float32)
    want = np.ascontiguousarray(want, dtype=np.float32)
    assert got.shape == want.shape
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), "decode differs bit-wise"


def gguf_golden(qtype):
    """(raw blocks, gguf-py's own float32 decode) from tests/golden/gguf_types.npz."""
    name = O.GGUF_TYPES[qtype][0]
    z = np.load(os.path.join(GOLD, "gguf_types.npz"))
    return z[f"{name}__raw"], z[f"{name}__f32"]


def row_exponent_rule(bound, e):
    """The per-row power of two keeps bound * 2^-e in (2^14, 2^15] (at most 2^15 for any bound)."""
    scaled = np.ldexp(np.asarray(bound, dtype=np.float64), -np.asarray(e))
    assert np.all(scaled <= 2.0 ** 15), "a decoded fp16 weight could overflow"
    assert np.all(scaled[np.asarray(bound) > 0] > 2.0 ** 14), "precision left unused"


def row_exponent_check(qtype):
    """On random blocks and on the golden edge-scale rows (zero, +-65504 and subnormal scales,
    where a block's minimum term alone sets |w|): the scale-only row bound covers every decoded
    |w| and the row exponent follows `row_exponent_rule`."""
    raw = O.random_gguf_blocks(qtype, 8, 512, seed=qtype + 10)
    gold, _ = gguf_golden(qtype)
    for r, n in ((raw, 8), (gold, gold.shape[0])):
        w = O.gguf_dequantize(r, qtype, n, 512)
        bound = O.gguf_row_bound(r, qtype, n, 512)
        assert np.all(np.abs(w).max(axis=1) <= bound), "the row bound misses a decoded weight"
        row_exponent_rule(bound, O.gguf_row_exponent(bound))


def e4m3_code_table():
    """All 256 float8_e4m3fn codes decode as torch decodes them (NaN where torch has NaN)."""
    raw = np.arange(256, dtype=np.uint8)
    want = torch.from_numpy(raw.copy()).view(torch.float8_e4m3fn).float().numpy()
    got = O.e4m3_to_float(raw)
    assert np.array_equal(np.isnan(want), np.isnan(got)), "NaN codes differ"
    ok = ~np.isnan(want)
    assert np.array_equal(got[ok], want[ok]), "e4m3 values differ"


def a8_integer_case(m, k, n, bits, group, seed=17):
    """An A8 problem whose answer is exact in fp32: integer activations whose row maximum is 127
    (the per-token scale is exactly 1), integer weights, power-of-two group scales (1, 1/2, 1/4 by
    row and group) and an integer bias.  Returns (x fp32 [m, k], wq int8 [n, k], s fp16
    [n, k/group], bias fp16 [n])."""
    rng = np.random.default_rng(seed)
    x = rng.integers(-127, 128, (m, k), dtype=np.int16).astype(np.float32)
    x[:, 5] = 127.0
    lo, hi = (-8, 8) if bits == 4 else (-32, 32)
    wq = rng.integers(lo, hi, (n, k), dtype=np.int8)
    expo = (np.arange(n)[:, None] + np.arange(k // group)[None, :]) % 3
    s = np.ldexp(1.0, -expo).astype(np.float16)
    bias = rng.integers(-64, 65, n).astype(np.float16)
    return x, wq, s, bias


def a8_exact(name, got, x, wq, s, group, bias, rows):
    """fp32 output finite everywhere and, on the sampled rows, equal bit for bit to the exact
    group sums plus bias."""
    got = np.asarray(got)
    assert np.isfinite(got).all(), f"{name}: non-finite outputs (a tile was not written)"
    want = group_sums_f64(x[rows], wq, s, group) + np.asarray(bias, dtype=np.float64)[None, :]
    diff = np.abs(got[rows].astype(np.float64) - want)
    assert np.array_equal(got[rows].astype(np.float64), want), f"{name}: max |diff| {diff.max()}"


def q8_0_integer_case(m, k, n, seed=23):
    """A GGUF Q8_0 problem whose answer is exact in fp32: every block scale 1.0, integer codes,
    integer activations in [-8, 8] and an integer bias.  The decoded fp16 weight code * 2^7 is
    exact, every product and partial sum is a multiple of 2^7 below 2^31, so any fp32 accumulation
    order gives the exact integer.  Returns (x fp16 [m, k], raw uint8 [n, k/32*34], bias fp16
    [n], want int64 [m, n])."""
    rng = np.random.default_rng(seed)
    codes = rng.integers(-127, 128, (n, k), dtype=np.int8)
    blocks = np.empty((n, k // 32, 34), dtype=np.uint8)
    blocks[..., 0:2] = np.array([1.0], dtype=np.float16).view(np.uint8)
    blocks[..., 2:] = codes.reshape(n, k // 32, 32).view(np.uint8)
    x = rng.integers(-8, 9, (m, k)).astype(np.float16)
    bias = rng.integers(-64, 65, n).astype(np.float16)
    want = x.astype(np.int64) @ codes.astype(np.int64).T + bias.astype(np.int64)[None, :]
    return x, blocks.reshape(n, -1), bias, want


def integer_exact(name, got, want):
    """fp32 output finite and equal to the exact integer answer."""
    got = np.asarray(got, dtype=np.float64)
    assert np.isfinite(got).all(), f"{name}: non-finite outputs"
    assert np.array_equal(got, np.asarray(want, dtype=np.float64)), \
        f"{name}: max |diff| {np.abs(got - want).max()}"


def onehot_exact(name, y, raw, qtype, n, k, rows):
    """One-hot activation rows (rows `rows` of the K x K identity) through the linear with fp32
    output: each output is a single decoded weight, which must equal the exact decode rounded once
    to fp16 at its row's power of two, RN16(w * 2^-e) * 2^e (types decoded with one rounding)."""
    wn, e = O.gguf_normalized_fp16(raw, qtype, n, k)
    exact = np.ldexp(wn.astype(np.float32), e.reshape(-1, 1)).T[rows]
    assert np.array_equal(np.asarray(y), exact), f"{name}: a decoded weight differs from RN16(w 2^-e) 2^e"
