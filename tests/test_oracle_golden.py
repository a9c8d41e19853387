"""The CPU oracle pinned against the reference's golden vectors and gguf 0.19.0.

Fixtures in tests/golden/ come from the reference's in-container self-test
(`modal/results/2026-11-09-weight-error-selftest-container.json`) and from the reference's CPU
port run once at fixture time (tests/golden/make_golden.py)."""
import base64
import hashlib
import json
import os

import numpy as np
import pytest
import torch

import checks as C
from oracle import qlin_oracle as O

GOLD = os.path.join(os.path.dirname(__file__), "golden")
HASHES = json.load(open(os.path.join(GOLD, "selftest_hashes.json")))


def sha(t):
    if isinstance(t, torch.Tensor):
        t = t.contiguous()
        if t.dtype == torch.float8_e4m3fn:
            t = t.view(torch.uint8)
        t = t.numpy()
    return hashlib.sha256(np.ascontiguousarray(t).tobytes()).hexdigest()


@pytest.fixture(scope="module")
def inputs():
    return O.selftest_inputs()


@pytest.mark.parametrize("case", ["gauss_96x1024", "heavy_96x1024", "chunked_4200x1024"])
def test_selftest_inputs_bit_identical(inputs, case):
    assert sha(inputs[case]) == HASHES["cases"][case]["input_sha256"]


@pytest.mark.parametrize("case", ["gauss_96x1024", "heavy_96x1024", "chunked_4200x1024"])
def test_int8_rowwise_codes_and_scales(inputs, case):
    q, s = O.quantize_int8_rowwise(inputs[case].clone())
    f = HASHES["cases"][case]["formats"]["int8_rowwise"]
    assert sha(q) == f["q"]
    assert sha(s) == f["scale"]


@pytest.mark.parametrize("case", ["gauss_96x1024", "heavy_96x1024", "chunked_4200x1024"])
def test_int8_convrot_codes(inputs, case):
    # Codes are bit-identical; float scales of the heavy-tailed case depend on the BLAS summation
    # order of the rotation (the reference records the same, docs/findings.md:1009).
    q, s = O.quantize_int8_convrot(inputs[case], 256, "h4")
    f = HASHES["cases"][case]["formats"]["int8_convrot"]
    assert sha(q) == f["q"]
    if case != "heavy_96x1024":
        assert sha(s) == f["scale"]


@pytest.mark.parametrize("case", ["gauss_96x1024", "heavy_96x1024"])
@pytest.mark.parametrize("fmt,qtype", [("gguf_q8_0", 8), ("gguf_q4_k", 12)])
def test_gguf_decode_matches_golden_ggml_vectors(case, fmt, qtype):
    raw = np.load(os.path.join(GOLD, "gguf_golden.npz"))[f"{case}__{fmt}"]
    f = HASHES["cases"][case]["formats"][fmt]
    assert hashlib.sha256(raw.tobytes()).hexdigest() == f["q"]
    w = O.gguf_dequantize(raw, qtype, 96, 1024)
    assert sha(w) == f["deq"]


ALL_TYPES = sorted(O.GGUF_TYPES)


@pytest.mark.parametrize("qtype", ALL_TYPES)
def test_gguf_decode_matches_committed_gguf_py_vectors(qtype):
    """Bit-exact against gguf-py's own decode of the same blocks (tests/golden/gguf_types.npz,
    made by tests/golden/make_gguf_types.py), edge scales included."""
    name, qk, ts = O.GGUF_TYPES[qtype]
    z = np.load(os.path.join(GOLD, "gguf_types.npz"))
    raw, want = z[f"{name}__raw"], z[f"{name}__f32"]
    got = O.gguf_dequantize(raw, qtype, *want.shape)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("qtype", ALL_TYPES)
def test_gguf_decode_matches_gguf_py(qtype):
    gguf = pytest.importorskip("gguf")
    from gguf import quants
    raw = O.random_gguf_blocks(qtype, 24, 512, seed=qtype)
    # Extreme scales: zero, +-65504, subnormal, in the first blocks.
    name, qk, ts = O.GGUF_TYPES[qtype]
    flat = raw.reshape(-1, ts)
    offs = O.GGUF_SCALE_FIELDS[name][0]
    for i, v in enumerate([0.0, 65504.0, -65504.0, 2.0 ** -24, -(2.0 ** -20)]):
        for off in offs:
            flat[i, off:off + 2] = np.array([v], dtype=np.float16).view(np.uint8)
    want = quants.dequantize(raw.reshape(-1), gguf.GGMLQuantizationType(qtype)).reshape(24, 512)
    got = O.gguf_dequantize(raw, qtype, 24, 512)
    assert got.dtype == np.float32
    assert np.array_equal(got.view(np.uint32), want.astype(np.float32).view(np.uint32))


@pytest.mark.parametrize("qtype", [12, 11, 23])
def test_gguf_rows_straddling_blocks(qtype):
    gguf = pytest.importorskip("gguf")
    from gguf import quants
    raw = O.random_gguf_blocks(qtype, 4, 768, seed=3)  # 12 superblocks
    want = quants.dequantize(raw.reshape(-1), gguf.GGMLQuantizationType(qtype)).reshape(-1)
    got = O.gguf_dequantize(raw, qtype, 6, 512)  # 6 rows of 512: rows start mid-block
    assert np.array_equal(got.reshape(-1), want)


def test_kitchen_pack_roundtrip_and_int8_grid():
    z = np.load(os.path.join(GOLD, "kitchen_w4a8.npz"))
    for fmt, bits in (("w4a8", 4), ("w6a8", 6)):
        q = z[f"{fmt}_q"]
        codes = O.unpack_codes_kitchen(q, 1024, bits)
        assert np.array_equal(O.pack_codes_kitchen(codes, bits).view(np.uint8), q.view(np.uint8))
        cb = z[f"{fmt}_codebook"] if f"{fmt}_codebook" in z else None
        grid = O.kitchen_int8_grid(q, z[f"{fmt}_s_rel"], 1024, bits, 16, cb)
        assert np.array_equal(grid, z[f"{fmt}_grid"])  # bit-exact with the reference port
        deq = O.dequantize_kitchen_w4a8(q, z[f"{fmt}_s_rel"], z[f"{fmt}_s_channel"], 1024, bits, 16, cb, 256)
        ref = z[f"{fmt}_deq16"].astype(np.float64)
        assert np.abs(deq[:16] - ref).max() <= 1e-6 * np.abs(ref).max()


def test_e4m3_decode_matches_torch():
    C.e4m3_code_table()


def test_hadamards_orthonormal_and_h4_matches_reference_construction():
    for size in (4, 16, 64, 256):
        h = O.hadamard_h4(size)
        assert np.allclose(h @ h.T, np.eye(size), atol=1e-12)
    for size in (2, 8, 32, 128):
        h = O.hadamard_sylvester(size)
        assert np.allclose(h @ h.T, np.eye(size), atol=1e-12)
    assert O.hadamard(128).shape == (128, 128)
    assert np.array_equal(O.hadamard(256), O.hadamard_h4(256))


def test_w4_w6_pack_roundtrip():
    rng = np.random.default_rng(0)
    q4 = rng.integers(-8, 8, (7, 256))
    assert np.array_equal(O.unpack_w4_uniform(O.pack_w4_uniform(q4), 256), q4)
    q6 = rng.integers(-32, 32, (5, 128))
    p6 = O.pack_w6_interleaved(q6)
    assert p6.shape == (5, 96)
    assert np.array_equal(O.unpack_w6_interleaved(p6, 128), q6)


def test_grouped_a8_reference_is_exact_on_integer_inputs():
    rng = np.random.default_rng(1)
    x = rng.integers(-127, 128, (9, 256)).astype(np.float16)
    x[:, 0] = 127  # absmax 127 -> activation scale exactly 1
    wq = rng.integers(-8, 8, (5, 256)).astype(np.int8)
    s = np.ones((5, 2), dtype=np.float16)
    y, xq, sx = O.grouped_linear_a8(x, wq, s, 128)
    assert np.all(sx == 1.0)
    assert np.array_equal(xq.astype(np.int64), x.astype(np.int64))
    assert np.array_equal(y, (x.astype(np.int64) @ wq.astype(np.int64).T).astype(np.float64))


@pytest.mark.parametrize("qtype", ALL_TYPES)
def test_row_exponent_bounds_decoded_rows(qtype):
    C.row_exponent_check(qtype)
