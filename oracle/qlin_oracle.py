"""CPU oracle for the quantized-linear hot path.  TEST INFRASTRUCTURE ONLY.

This module restates, on the CPU, the arithmetic the reference (roblennon/mac-kernels-public) and
its pinned third-party decoder (`gguf` 0.19.0, `gguf/quants.py`) define for:

  * ConvRot block-Hadamard rotation and the per-row INT8 quantizer
    (reference `modal/weight_error_app.py:90-127`, a port of comfy-kitchen's eager quantizers);
  * the comfy-kitchen W4A8/W6A8 ("AsymW4A8Int8Layout") pack/unpack and int8-grid decode
    (`modal/weight_error_app.py:145-166, 326-339`);
  * GGUF block decode for the twelve types the reference's kernel covers: Q4_0, Q4_1, Q5_0, Q5_1,
    Q8_0, Q2_K, Q3_K, Q4_K, Q5_K, Q6_K, IQ4_NL, IQ4_XS (formula table
    `docs/research/2026-10-03-gguf-on-metal.md:18-37`, type list `:59`; third-party algorithm
    `gguf` 0.19.0 `gguf/quants.py` Q4_0 :220, Q4_1 :275, Q5_0 :313, Q5_1 :356, Q8_0 :378,
    Q2_K :405, Q3_K :432, Q4_K :475, Q5_K :526, Q6_K :552, IQ4_NL :1330, IQ4_XS :1352);
  * the simplified synthetic layouts the benchmark configurations use (uniform 4-bit group-128
    and 6-bit "four values per three bytes" group-64 weights with fp16 group scales, and the
    Sylvester Hadamard of size 128).  These have no counterpart in the reference; their
    definitions here are this project's own and are documented next to each function.

Only tests, the `smoke()` self-check and `bench.py`'s CPU-baseline leg may import this module.
The product path (the CUDA library and its Python shim) never calls it.

Floating-point conventions: byte and integer work (codes, packing, int32 accumulators, GGUF fp32
decode) is bit-exact; float linears are computed in float64 and compared by tolerance.
"""
from __future__ import annotations

import numpy as np
import torch

# ----------------------------------------------------------------------------------------------
# Hadamard rotation
# ----------------------------------------------------------------------------------------------

_H4 = np.array([[1, 1, 1, -1], [1, 1, -1, 1], [1, -1, 1, 1], [-1, 1, 1, 1]], dtype=np.float64)


def hadamard_h4(size: int) -> np.ndarray:
    """Orthonormal Kronecker power of the regular 4x4 Hadamard (size a power of 4).

    Follows `modal/weight_error_app.py:90-98` (`build_hadamard`): start from H4 and Kronecker it
    with H4 on the right until the size is reached, then divide by sqrt(size)."""
    h = _H4.copy()
    while h.shape[0] < size:
        h = np.kron(h, _H4)
    if h.shape[0] != size:
        raise ValueError(f"H4 Kronecker Hadamard needs a power of 4, got {size}")
    return h / np.sqrt(size)


def hadamard_sylvester(size: int) -> np.ndarray:
    """Orthonormal Sylvester Hadamard (size a power of 2): H_{2n} = [[H, H], [H, -H]] / sqrt(2).

    The reference's builder only reaches powers of 4; the 128-wide rotation of the benchmark
    configuration uses this matrix.  Entry (i, j) is (-1)^popcount(i & j) / sqrt(size)."""
    if size < 1 or size & (size - 1):
        raise ValueError(f"Sylvester Hadamard needs a power of 2, got {size}")
    i = np.arange(size)
    bits = np.bitwise_and.outer(i, i)
    parity = np.zeros_like(bits)
    while bits.any():
        parity ^= bits & 1
        bits >>= 1
    return (1.0 - 2.0 * parity) / np.sqrt(size)


def hadamard(size: int, kind: str = "auto") -> np.ndarray:
    """`kind`: "h4" (reference, powers of 4), "sylvester", or "auto" (h4 when size is a power of
    4, else Sylvester).  The library uses the same rule."""
    if kind == "h4" or (kind == "auto" and size & (size - 1) == 0 and (size.bit_length() - 1) % 2 == 0):
        return hadamard_h4(size)
    return hadamard_sylvester(size)


def rotate_rows(x, group: int, kind: str = "auto"):
    """x @ blockdiag(H^T) over consecutive groups of `group` columns.

    Follows `modal/weight_error_app.py:101-106` (`rotate_weight`).  Accepts numpy or torch; a
    torch float32 input is rotated with torch.matmul in float32 (the reference's own arithmetic,
    which the golden code vectors were produced with); numpy input is rotated in float64."""
    if isinstance(x, torch.Tensor):
        rows, cols = x.shape
        h = torch.from_numpy(hadamard(group, kind)).to(x.dtype)
        return torch.matmul(x.reshape(rows, cols // group, group), h.T).reshape(rows, cols)
    x = np.asarray(x, dtype=np.float64)
    rows, cols = x.shape
    if cols % group:
        raise ValueError("columns must be a multiple of the rotation group")
    h = hadamard(group, kind)
    return (x.reshape(rows, cols // group, group) @ h.T).reshape(rows, cols)


# ----------------------------------------------------------------------------------------------
# INT8 row-wise quantizer (weights, and the per-token activation quantizer of the A8 formats)
# ----------------------------------------------------------------------------------------------


def int8_grad_input(dy, q, s, group: int = 0) -> np.ndarray:
    """dx = dy . W (float64) for the frozen INT8 ConvRot weight: W = (q * s) un-rotated per block,
    W = W_rot . H, the weight in the original basis as the reference's backward bench builds its
    exact answer (`bench/bench_int8_backward.py:36-39,53`: `dequant`, then `dy @ W`)."""
    w = np.asarray(q, dtype=np.float64) * np.asarray(s, dtype=np.float64).reshape(-1, 1)
    if group:
        w = rotate_rows(w, group)
    return np.asarray(dy, dtype=np.float64) @ w

def quantize_int8_rowwise(x: torch.Tensor):
    """Per-row absmax/127 INT8 quantization in x's dtype.

    Follows `modal/weight_error_app.py:109-115`: scale = max(absmax/127 in fp32, 1e-30); the
    divisor is that scale cast to x.dtype (zero replaced by the dtype's smallest normal); the
    quotient x / s is formed in x.dtype, rounded half-to-even and clamped to [-128, 127].
    Returns (int8 codes, fp32 scale [rows, 1])."""
    abs_max = x.abs().amax(dim=-1, keepdim=True)
    scale = (abs_max.float() / 127.0).clamp(min=1e-30)
    s = scale.to(x.dtype)
    s = torch.where(s == 0, torch.full_like(s, torch.finfo(x.dtype).tiny), s)
    q = (x / s).round_().clamp_(-128.0, 127.0).to(torch.int8)
    return q, scale


def quantize_int8_convrot(w: torch.Tensor, group: int = 256, kind: str = "auto"):
    """`modal/weight_error_app.py:118-119`: rotate, then quantize each row."""
    return quantize_int8_rowwise(rotate_rows(w, group, kind))


def dequantize_int8_convrot(q, scale, group: int = 256, kind: str = "auto"):
    """`modal/weight_error_app.py:126-127`: q * scale, then rotate back (float64 here)."""
    w = np.asarray(q, dtype=np.float64) * np.asarray(scale, dtype=np.float64).reshape(-1, 1)
    return rotate_rows(w, group, kind)


# ----------------------------------------------------------------------------------------------
# comfy-kitchen W4A8 / W6A8 storage (AsymW4A8Int8Layout)
# ----------------------------------------------------------------------------------------------

def pack_codes_kitchen(unsigned: np.ndarray, bits: int) -> np.ndarray:
    """Planar packing of unsigned codes [N, K] -> int8 [N, K*bits/8].

    Follows `modal/weight_error_app.py:145-152`: K/2 bytes of nibble pairs (even column in the
    low nibble), then for 6 bits K/4 bytes holding the 2-bit high planes of four consecutive
    columns (column 4j+i at bits 2i..2i+1)."""
    u = np.asarray(unsigned, dtype=np.int32)
    low = ((u[:, 0::2] & 0xF) | ((u[:, 1::2] & 0xF) << 4)).astype(np.uint8)
    if bits == 4:
        return low.view(np.int8)
    hi = np.zeros((u.shape[0], u.shape[1] // 4), dtype=np.int32)
    for j in range(4):
        hi |= ((u[:, j::4] >> 4) & 0x3) << (2 * j)
    return np.concatenate([low, hi.astype(np.uint8)], axis=1).view(np.int8)


def unpack_codes_kitchen(qdata: np.ndarray, k: int, bits: int) -> np.ndarray:
    """Inverse of `pack_codes_kitchen`; follows `modal/weight_error_app.py:155-166`."""
    packed = np.asarray(qdata).view(np.uint8).astype(np.int32)
    n = packed.shape[0]
    low = packed[:, : k // 2]
    codes = np.empty((n, k), dtype=np.int32)
    codes[:, 0::2] = low & 0xF
    codes[:, 1::2] = (low >> 4) & 0xF
    if bits == 6:
        hi = packed[:, k // 2:]
        for j in range(4):
            codes[:, j::4] |= ((hi >> (2 * j)) & 0x3) << 4
    return codes


def e4m3_to_float(raw: np.ndarray) -> np.ndarray:
    """float8_e4m3fn bytes -> float32 (exact).  Bias 7, no infinities, 0x7F/0xFF are NaN."""
    b = np.asarray(raw).view(np.uint8).astype(np.int32)
    sign = np.where(b & 0x80, -1.0, 1.0)
    exp = (b >> 3) & 0xF
    man = b & 0x7
    val = np.where(exp == 0, man / 8.0 * 2.0 ** -6, (1.0 + man / 8.0) * 2.0 ** (exp - 7))
    val = np.where((b & 0x7F) == 0x7F, np.nan, val)
    return (sign * val).astype(np.float32)


def kitchen_levels(bits: int, codebook=None) -> np.ndarray:
    """Per-code level table: the 16-entry fp32 codebook, or uniform levels code - 2^(bits-1)
    (`modal/weight_error_app.py:331-334`)."""
    if codebook is not None:
        return np.asarray(codebook, dtype=np.float32)
    return (np.arange(1 << bits, dtype=np.float32) - float(1 << (bits - 1)))


def kitchen_int8_grid(qdata, s_rel_raw, k: int, bits: int, group: int = 16, codebook=None) -> np.ndarray:
    """The int8 weight grid the kernels multiply with: round(level[code] * s_rel) clamped to
    +-127, computed in fp32 (`modal/weight_error_app.py:328-336`).  `s_rel_raw` holds e4m3
    bytes [N, K/group].  Bit-exact: one fp32 product, then round-half-even."""
    codes = unpack_codes_kitchen(qdata, k, bits)
    levels = kitchen_levels(bits, codebook)[codes]
    n = codes.shape[0]
    s = e4m3_to_float(s_rel_raw).reshape(n, k // group, 1)
    v = (levels.reshape(n, k // group, group) * s).astype(np.float32)
    return np.clip(np.rint(v), -127, 127).astype(np.int8).reshape(n, k)


def dequantize_kitchen_w4a8(qdata, s_rel_raw, s_channel, k: int, bits: int, group: int = 16,
                            codebook=None, convrot_group: int = 256) -> np.ndarray:
    """Full decode to the original basis (float64 rotation):
    `modal/weight_error_app.py:326-339`."""
    grid = kitchen_int8_grid(qdata, s_rel_raw, k, bits, group, codebook).astype(np.float64)
    w = grid * np.asarray(s_channel, dtype=np.float64).reshape(-1, 1)
    return rotate_rows(w, convrot_group) if convrot_group else w


# ----------------------------------------------------------------------------------------------
# Benchmark-configuration layouts (this project's definitions; no reference counterpart)
# ----------------------------------------------------------------------------------------------

def pack_w4_uniform(q: np.ndarray) -> np.ndarray:
    """Symmetric 4-bit values in [-8, 7] [N, K] -> int8 [N, K/2].  Stored as unsigned codes
    u = q + 8 in the kitchen nibble order (even column in the low nibble), so one decoder serves
    both layouts."""
    q = np.asarray(q, dtype=np.int32)
    if q.min() < -8 or q.max() > 7:
        raise ValueError("4-bit values must lie in [-8, 7]")
    return pack_codes_kitchen(q + 8, 4)


def unpack_w4_uniform(packed: np.ndarray, k: int) -> np.ndarray:
    return unpack_codes_kitchen(packed, k, 4) - 8


def pack_w6_interleaved(q: np.ndarray) -> np.ndarray:
    """Symmetric 6-bit values in [-32, 31] [N, K] -> uint8 [N, 3K/4], "four values per three
    bytes": each run of four columns 4j..4j+3 becomes the little-endian 24-bit word
    u0 | u1<<6 | u2<<12 | u3<<18 with u = q + 32, written as bytes 3j, 3j+1, 3j+2."""
    q = np.asarray(q, dtype=np.int64)
    if q.min() < -32 or q.max() > 31:
        raise ValueError("6-bit values must lie in [-32, 31]")
    u = q + 32
    n, k = u.shape
    word = u[:, 0::4] | (u[:, 1::4] << 6) | (u[:, 2::4] << 12) | (u[:, 3::4] << 18)
    out = np.empty((n, k // 4, 3), dtype=np.uint8)
    out[..., 0] = word & 0xFF
    out[..., 1] = (word >> 8) & 0xFF
    out[..., 2] = (word >> 16) & 0xFF
    return out.reshape(n, 3 * k // 4)


def unpack_w6_interleaved(packed: np.ndarray, k: int) -> np.ndarray:
    b = np.asarray(packed).view(np.uint8).astype(np.int64)
    n = b.shape[0]
    b = b.reshape(n, k // 4, 3)
    word = b[..., 0] | (b[..., 1] << 8) | (b[..., 2] << 16)
    out = np.empty((n, k), dtype=np.int32)
    for i in range(4):
        out[:, i::4] = ((word >> (6 * i)) & 0x3F) - 32
    return out


def grouped_linear_a8(x, wq: np.ndarray, group_scale: np.ndarray, group: int, bias=None):
    """Reference for the W4A8 / W6A8 benchmark layouts.

    Activations are quantized per token with `quantize_int8_rowwise` in their own dtype (a numpy
    array is taken as fp16; a torch tensor keeps its dtype).  For every K-group g the int32
    partial P_g = xq[:, g] . wq[:, g]^T is formed exactly (int64 here), then
    Y = sx[m] * sum_g s[n, g] * P_g[m, n] (+ bias), in float64.
    Returns (Y float64, xq int8, sx float32)."""
    xt = x if isinstance(x, torch.Tensor) else torch.from_numpy(np.asarray(x, dtype=np.float16))
    xq, sx = quantize_int8_rowwise(xt)
    return grouped_linear_from_codes(xq.numpy(), sx.numpy(), wq, group_scale, group, bias), xq.numpy(), sx.numpy()


def grouped_linear_from_codes(xq, sx, wq, group_scale, group: int, bias=None) -> np.ndarray:
    """Y = sx[m] * sum_g s[n, g] * P_g[m, n] (+ bias) from already-quantized activations;
    group 0 means one group over all of K with per-channel scales s[n]."""
    xq = np.asarray(xq, dtype=np.int64)
    sx = np.asarray(sx, dtype=np.float64).reshape(-1, 1)
    wq = np.asarray(wq, dtype=np.int64)
    n, k = wq.shape
    group = group or k
    groups = k // group
    s = np.asarray(group_scale, dtype=np.float64).reshape(n, groups)
    y = np.zeros((xq.shape[0], n), dtype=np.float64)
    for g in range(groups):
        sl = slice(g * group, (g + 1) * group)
        p = xq[:, sl] @ wq[:, sl].T
        y += p.astype(np.float64) * s[:, g][None, :]
    y *= sx
    if bias is not None:
        y += np.asarray(bias, dtype=np.float64)[None, :]
    return y


def int_group_partials(xq: np.ndarray, wq: np.ndarray, group: int) -> np.ndarray:
    """Exact per-group int32 partial sums [groups, M, N] (int64 arithmetic)."""
    xq = np.asarray(xq, dtype=np.int64)
    wq = np.asarray(wq, dtype=np.int64)
    k = wq.shape[1]
    return np.stack([xq[:, g:g + group] @ wq[:, g:g + group].T for g in range(0, k, group)])


# ----------------------------------------------------------------------------------------------
# GGUF block decode (restates gguf 0.19.0 gguf/quants.py; fp32, same operation order)
# ----------------------------------------------------------------------------------------------

# type id -> (name, values per block, bytes per block); ids are enum ggml_type.
GGUF_TYPES = {
    2: ("Q4_0", 32, 18),
    3: ("Q4_1", 32, 20),
    6: ("Q5_0", 32, 22),
    7: ("Q5_1", 32, 24),
    8: ("Q8_0", 32, 34),
    10: ("Q2_K", 256, 84),
    11: ("Q3_K", 256, 110),
    12: ("Q4_K", 256, 144),
    13: ("Q5_K", 256, 176),
    14: ("Q6_K", 256, 210),
    20: ("IQ4_NL", 32, 18),
    23: ("IQ4_XS", 256, 136),
}
GGUF_IDS = {v[0]: k for k, v in GGUF_TYPES.items()}
IQ4_NL_VALUES = np.array([-127, -104, -83, -65, -49, -35, -22, -10, 1, 13, 25, 38, 53, 69, 89, 113],
                         dtype=np.float32)


def _f16(raw2: np.ndarray) -> np.ndarray:
    return np.ascontiguousarray(raw2).view(np.float16).astype(np.float32)


def q4k_scale_min(scales12: np.ndarray):
    """Eight 6-bit (scale, min) pairs from the 12 packed bytes of a Q4_K block
    (`gguf/quants.py:479-500`): pairs 0-3 are the low 6 bits of bytes 0-3 / 4-7; pairs 4-7 take
    a nibble of bytes 8-11 plus the top two bits of bytes 0-3 / 4-7."""
    s = scales12.astype(np.uint8).reshape(-1, 3, 4)
    d, m, md = s[:, 0], s[:, 1], s[:, 2]
    sc = np.concatenate([d & 0x3F, (md & 0x0F) | ((d >> 2) & 0x30)], axis=-1)
    mn = np.concatenate([m & 0x3F, (md >> 4) | ((m >> 2) & 0x30)], axis=-1)
    return sc.astype(np.float32), mn.astype(np.float32)


def _nibbles32(qs16: np.ndarray) -> np.ndarray:
    """[nb, 16] bytes -> [nb, 32] codes of a 32-value run: byte i holds value i in its low nibble
    and value i + 16 in its high nibble (`gguf/quants.py:285-286`)."""
    return np.concatenate([qs16 & 0xF, qs16 >> 4], axis=1)


def _bits32(qh4: np.ndarray) -> np.ndarray:
    """[nb, 4] bytes of a little-endian uint32 -> [nb, 32], element i = bit i (`gguf/quants.py:323-325`)."""
    w = np.ascontiguousarray(qh4).view("<u4").astype(np.uint32)
    return ((w >> np.arange(32, dtype=np.uint32)) & 1).astype(np.uint8)


def _crumbs256(qs64: np.ndarray) -> np.ndarray:
    """[nb, 64] bytes -> [nb, 256] 2-bit codes: value j of a 256-superblock sits in byte
    32*(j // 128) + j % 32 at bits 2*((j % 128) // 32) (`gguf/quants.py:422-424`)."""
    q = qs64.reshape(-1, 2, 1, 32)
    return np.concatenate([(q >> s) & 3 for s in (0, 2, 4, 6)], axis=2).reshape(-1, 256)


def q3k_scales(scales12: np.ndarray) -> np.ndarray:
    """Sixteen signed 6-bit Q3_K scales (`gguf/quants.py:456-463`): low nibble of byte i (i < 8) or
    high nibble of byte i - 8, plus bits 2*(i // 4) of byte 8 + i % 4 as bits 4-5, minus 32."""
    s = scales12.astype(np.uint8).reshape(-1, 12)
    lo = np.concatenate([s[:, 0:8] & 0xF, s[:, 0:8] >> 4], axis=1)
    hi = np.concatenate([(s[:, 8:12] >> (2 * t)) & 3 for t in range(4)], axis=1)
    return ((lo | (hi << 4)).astype(np.int16) - 32).astype(np.float32)


def iq4xs_scales(block: np.ndarray) -> np.ndarray:
    """Eight signed 6-bit IQ4_XS sub-block scales (`gguf/quants.py:1363-1369`): nibble i % 2 of
    scales_l[i // 2] plus bits 2i..2i+1 of the uint16 scales_h as bits 4-5, minus 32."""
    b = block.astype(np.uint8).reshape(-1, block.shape[-1])
    sh = b[:, 2].astype(np.uint32) | (b[:, 3].astype(np.uint32) << 8)
    sl = b[:, 4:8]
    lo = np.stack([sl & 0xF, sl >> 4], axis=2).reshape(-1, 8).astype(np.uint32)
    hi = (sh[:, None] >> (2 * np.arange(8, dtype=np.uint32))) & 3
    return ((lo | (hi << 4)).astype(np.int16) - 32).astype(np.float32)


def gguf_dequantize_blocks(blocks: np.ndarray, qtype: int) -> np.ndarray:
    """uint8 blocks [nb, type_size] -> float32 [nb, block_values], bit-exact with gguf 0.19.0.

    Every product and sum below is one numpy float32 operation in the order gguf-py evaluates it
    (no fused multiply-add), so the roundings are the same."""
    name, qk, ts = GGUF_TYPES[qtype]
    b = np.ascontiguousarray(blocks, dtype=np.uint8).reshape(-1, ts)
    nb = b.shape[0]
    if name in ("Q4_1", "Q5_0", "Q5_1"):
        # Q4_1 d, m, qs[16] (`gguf/quants.py:275-288`); Q5_0 d, qh u32, qs[16] (:313-330);
        # Q5_1 d, m, qh u32, qs[16] (:356-375).  w = d*q (+ m), Q5_0 with q - 16.
        d = _f16(b[:, 0:2])
        has_m = name != "Q5_0"
        m = _f16(b[:, 2:4]) if has_m else None
        qs_off = {"Q4_1": 4, "Q5_0": 6, "Q5_1": 8}[name]
        q = _nibbles32(b[:, qs_off:qs_off + 16])
        if name != "Q4_1":
            q = q | (_bits32(b[:, qs_off - 4:qs_off]) << 4)
        if name == "Q5_0":
            return d * (q.astype(np.int8) - np.int8(16)).astype(np.float32)
        return d * q.astype(np.float32) + m
    if name == "Q2_K":
        # scales[16], qs[64], d, dmin (`gguf/quants.py:405-428`): w = (d*(sc & 15))*q - dmin*(sc >> 4)
        sc = b[:, 0:16]
        d = _f16(b[:, 80:82])
        dmin = _f16(b[:, 82:84])
        dl = (d * (sc & 0xF).astype(np.float32)).reshape(nb, 16, 1)
        ml = (dmin * (sc >> 4).astype(np.float32)).reshape(nb, 16, 1)
        q = _crumbs256(b[:, 16:80]).reshape(nb, 16, 16).astype(np.float32)
        return (dl * q - ml).reshape(nb, 256)
    if name == "Q3_K":
        # hmask[32], qs[64], scales[12], d (`gguf/quants.py:432-472`): w = (d*sc)*q with
        # q = crumb - 4 where the hmask bit (bit j // 32 of hmask[j % 32]) is clear.
        d = _f16(b[:, 108:110])
        dl = (d * q3k_scales(b[:, 96:108])).reshape(nb, 16, 1)
        lo = _crumbs256(b[:, 32:96])
        hm = b[:, 0:32].reshape(nb, 1, 32)
        hbit = np.concatenate([(hm >> i) & 1 for i in range(8)], axis=1).reshape(nb, 256)
        q = (lo.astype(np.int8) - ((hbit ^ 1) << 2).astype(np.int8)).reshape(nb, 16, 16).astype(np.float32)
        return (dl * q).reshape(nb, 256)
    if name == "Q5_K":
        # d, dmin, scales[12], qh[32], qs[128] (`gguf/quants.py:526-549`): Q4_K plus a fifth bit,
        # bit s of qh[l] for value l of sub-block s.
        d = _f16(b[:, 0:2])
        dmin = _f16(b[:, 2:4])
        sc, mn = q4k_scale_min(b[:, 4:16])
        ds = (d * sc).reshape(nb, 8, 1)
        dm = (dmin * mn).reshape(nb, 8, 1)
        qs = b[:, 48:176].reshape(nb, 4, 1, 32)
        lo = np.concatenate([qs & 0xF, qs >> 4], axis=2).reshape(nb, 8, 32)
        qh = b[:, 16:48].reshape(nb, 1, 32)
        hi = np.concatenate([(qh >> s) & 1 for s in range(8)], axis=1)
        q = (lo | (hi << 4)).astype(np.float32)
        return (ds * q - dm).reshape(nb, 256)
    if name == "IQ4_XS":
        # d, scales_h u16, scales_l[4], qs[128] (`gguf/quants.py:1352-1377`): sub-block i is an
        # IQ4_NL run of 32 with scale d*sc_i.
        d = _f16(b[:, 0:2])
        dl = (d * iq4xs_scales(b)).reshape(nb, 8, 1)
        nib = _nibbles32(b[:, 8:136].reshape(nb * 8, 16)).reshape(nb, 8, 32)
        return (dl * IQ4_NL_VALUES[nib]).reshape(nb, 256)
    if name in ("Q4_0", "IQ4_NL"):
        d = _f16(b[:, 0:2])
        qs = b[:, 2:18]
        nib = np.concatenate([qs & 0xF, qs >> 4], axis=1)  # values 0..15: low nibbles first
        if name == "Q4_0":
            v = (nib.astype(np.int8) - np.int8(8)).astype(np.float32)
        else:
            v = IQ4_NL_VALUES[nib]
        return d * v
    if name == "Q8_0":
        d = _f16(b[:, 0:2])
        return b[:, 2:34].view(np.int8).astype(np.float32) * d
    if name == "Q4_K":
        d = _f16(b[:, 0:2])
        dmin = _f16(b[:, 2:4])
        sc, mn = q4k_scale_min(b[:, 4:16])
        ds = (d * sc).reshape(nb, 8, 1)
        dm = (dmin * mn).reshape(nb, 8, 1)
        qs = b[:, 16:144].reshape(nb, 4, 1, 32)
        q = np.concatenate([qs & 0xF, qs >> 4], axis=2).reshape(nb, 8, 32).astype(np.float32)
        return (ds * q - dm).reshape(nb, 256)
    if name == "Q6_K":
        ql = b[:, 0:128]
        qh = b[:, 128:192]
        sc = b[:, 192:208].view(np.int8).astype(np.float32)
        d = _f16(b[:, 208:210])
        ds = (d * sc).reshape(nb, 16, 1)
        lo = ql.reshape(nb, 2, 1, 64)
        lo = np.concatenate([lo & 0xF, lo >> 4], axis=2).reshape(nb, 2, 128)
        hi = qh.reshape(nb, 2, 1, 32)
        hi = np.concatenate([(hi >> s) & 0x3 for s in (0, 2, 4, 6)], axis=2).reshape(nb, 2, 128)
        q = ((lo | (hi << 4)).astype(np.int8) - np.int8(32)).reshape(nb, 16, 16).astype(np.float32)
        return (ds * q).reshape(nb, 256)
    raise ValueError(f"unsupported GGUF type {qtype}")


def gguf_dequantize(raw: np.ndarray, qtype: int, n: int, k: int) -> np.ndarray:
    """Rows of raw blocks -> float32 [n, k].  Blocks are indexed by flat element
    (block = (row*K + col) / QK), so rows may straddle blocks as ComfyUI-GGUF's reshaped tensors
    do (`docs/research/2026-10-03-gguf-on-metal.md:38`)."""
    return gguf_dequantize_blocks(np.asarray(raw, dtype=np.uint8).reshape(-1), qtype).reshape(n, k)


def gguf_row_bound(raw: np.ndarray, qtype: int, n: int, k: int) -> np.ndarray:
    """Upper bound on |w| per row read from block scales only (float64), as the reference's
    per-row exponent pass does (`docs/research/2026-10-03-gguf-on-metal.md:89`)."""
    name, qk, ts = GGUF_TYPES[qtype]
    if k % qk:
        raise ValueError("row bound needs whole blocks per row")
    b = np.asarray(raw, dtype=np.uint8).reshape(n, k // qk, ts)
    def f16abs(off):
        return np.abs(_f16(b[..., off:off + 2])[..., 0].astype(np.float64))

    if name == "Q4_0":
        bound = np.abs(_f16(b[..., 0:2])[..., 0].astype(np.float64)) * 8
    elif name == "Q4_1":
        bound = f16abs(0) * 15 + f16abs(2)
    elif name == "Q5_0":
        bound = f16abs(0) * 16
    elif name == "Q5_1":
        bound = f16abs(0) * 31 + f16abs(2)
    elif name == "Q2_K":
        sc = b[..., 0:16]
        bound = (f16abs(80)[..., None] * (sc & 0xF).astype(np.float64) * 3
                 + f16abs(82)[..., None] * (sc >> 4).astype(np.float64)).max(axis=-1)
    elif name == "Q3_K":
        sc = np.abs(q3k_scales(b[..., 96:108].reshape(-1, 12)).reshape(n, k // qk, 16).astype(np.float64))
        bound = (f16abs(108)[..., None] * sc * 4).max(axis=-1)
    elif name == "Q5_K":
        sc, mn = q4k_scale_min(b[..., 4:16].reshape(-1, 12))
        sc = sc.reshape(n, k // qk, 8).astype(np.float64)
        mn = mn.reshape(n, k // qk, 8).astype(np.float64)
        bound = (f16abs(0)[..., None] * sc * 31 + f16abs(2)[..., None] * mn).max(axis=-1)
    elif name == "IQ4_XS":
        sc = np.abs(iq4xs_scales(b.reshape(-1, ts)).reshape(n, k // qk, 8).astype(np.float64))
        bound = (f16abs(0)[..., None] * sc * 127).max(axis=-1)
    elif name == "Q8_0":
        bound = np.abs(_f16(b[..., 0:2])[..., 0].astype(np.float64)) * 128
    elif name == "IQ4_NL":
        bound = np.abs(_f16(b[..., 0:2])[..., 0].astype(np.float64)) * 127
    elif name == "Q4_K":
        d = np.abs(_f16(b[..., 0:2])[..., 0].astype(np.float64))
        dmin = np.abs(_f16(b[..., 2:4])[..., 0].astype(np.float64))
        sc, mn = q4k_scale_min(b[..., 4:16].reshape(-1, 12))
        sc = sc.reshape(n, k // qk, 8).astype(np.float64)
        mn = mn.reshape(n, k // qk, 8).astype(np.float64)
        bound = (d[..., None] * sc * 15 + dmin[..., None] * mn).max(axis=-1)
    elif name == "Q6_K":
        d = np.abs(_f16(b[..., 208:210])[..., 0].astype(np.float64))
        sc = np.abs(b[..., 192:208].view(np.int8).astype(np.float64))
        bound = (d[..., None] * sc * 32).max(axis=-1)
    else:
        raise ValueError(name)
    return bound.reshape(n, -1).max(axis=1)


def gguf_row_exponent(bound: np.ndarray) -> np.ndarray:
    """Power-of-two exponent e per row such that bound * 2^-e <= 2^15 and, for bounds above
    2^14, > 2^14: the decoded fp16 weight w * 2^-e keeps the most precision fp16 allows and
    cannot overflow.  Zero rows get e = 0.  Matches the library's rule."""
    bound = np.asarray(bound, dtype=np.float64)
    e = np.zeros(bound.shape, dtype=np.int32)
    nz = bound > 0
    # smallest e with bound * 2^-e <= 2^15
    m, ex = np.frexp(bound[nz])  # bound = m * 2^ex, m in [0.5, 1)
    e[nz] = ex - 15
    return e


def gguf_normalized_fp16(raw, qtype, n, k):
    """The weight the GEMM kernels feed the tensor cores: fp32 decode * 2^-e rounded once to
    fp16, plus the row exponents."""
    w = gguf_dequantize(raw, qtype, n, k)
    e = gguf_row_exponent(gguf_row_bound(raw, qtype, n, k))
    return np.ldexp(w, -e.reshape(-1, 1)).astype(np.float16), e


def random_gguf_blocks(qtype: int, n: int, k: int, seed: int = 0, scale: float | None = None) -> np.ndarray:
    """Random legal blocks: every byte uniform, fp16 scale fields overwritten with
    |N(0, scale)|-sized values, the way the reference's GGUF bench builds them
    (`bench/bench_gguf_linear.py:35-40,69-78`).  Returns uint8 [n, k/QK*type_size]."""
    name, qk, ts = GGUF_TYPES[qtype]
    offs, mag = GGUF_SCALE_FIELDS[name]
    if scale is not None:
        mag = scale
    rng = np.random.default_rng(seed)
    nb = n * k // qk
    raw = rng.integers(0, 256, size=(nb, ts), dtype=np.uint8)
    for off in offs:
        raw[:, off:off + 2] = np.abs(rng.standard_normal(nb) * mag + mag).astype(np.float16).view(np.uint8).reshape(nb, 2)
    if name in ("Q4_1", "Q5_1"):  # the block minimum m is signed (negative for most real blocks)
        m = -np.abs(rng.standard_normal(nb) * 8 * mag).astype(np.float16)
        raw[:, 2:4] = m.view(np.uint8).reshape(nb, 2)
    return raw.reshape(n, (k // qk) * ts)


# name -> (byte offsets of the fp16 block scales that `random_gguf_blocks` overwrites, magnitude)
GGUF_SCALE_FIELDS = {"Q4_0": ([0], 5e-3), "Q4_1": ([0], 1.5e-3), "Q5_0": ([0], 1.5e-3), "Q5_1": ([0], 7e-4),
                     "Q8_0": ([0], 3e-4), "Q2_K": ([80, 82], 4e-4), "Q3_K": ([108], 2e-4),
                     "Q4_K": ([0, 2], 5e-5), "Q5_K": ([0, 2], 3e-5), "Q6_K": ([208], 3e-5),
                     "IQ4_NL": ([0], 3e-4), "IQ4_XS": ([0], 1e-5)}


def baseline_gguf_blocks(qtype: int, n: int, k: int, seed: int = 0) -> np.ndarray:
    """Configuration-1 weights: Q8_0 blocks with d = fp16(|N(0, 0.02)| / 127) and int8 codes
    uniform in [-127, 127]; Q4_0 blocks with d = fp16(|N(0, 0.02)| / 7) and nibbles uniform in
    [0, 15]."""
    name, qk, ts = GGUF_TYPES[qtype]
    rng = np.random.default_rng(seed)
    nb = n * k // qk
    raw = np.empty((nb, ts), dtype=np.uint8)
    if name == "Q8_0":
        d = (np.abs(rng.standard_normal(nb) * 0.02) / 127).astype(np.float16)
        qs = rng.integers(-127, 128, size=(nb, 32), dtype=np.int64).astype(np.int8)
        raw[:, 0:2] = d.view(np.uint8).reshape(nb, 2)
        raw[:, 2:] = qs.view(np.uint8)
    elif name == "Q4_0":
        d = (np.abs(rng.standard_normal(nb) * 0.02) / 7).astype(np.float16)
        nib = rng.integers(0, 16, size=(nb, 32), dtype=np.int64)
        raw[:, 0:2] = d.view(np.uint8).reshape(nb, 2)
        raw[:, 2:] = (nib[:, :16] | (nib[:, 16:] << 4)).astype(np.uint8)
    else:
        return random_gguf_blocks(qtype, n, k, seed)
    return raw.reshape(n, (k // qk) * ts)


# ----------------------------------------------------------------------------------------------
# Float references for the linears
# ----------------------------------------------------------------------------------------------

def linear_f64(x, w, bias=None) -> np.ndarray:
    y = np.asarray(x, dtype=np.float64) @ np.asarray(w, dtype=np.float64).T
    if bias is not None:
        y = y + np.asarray(bias, dtype=np.float64)[None, :]
    return y


def int8_convrot_linear_ref(x, q, scale, bias=None, group: int = 128, kind: str = "auto", convrot=True):
    """Y = rot(X) . (q*s)^T + b in float64 (the weight is stored rotated)."""
    xr = rotate_rows(np.asarray(x, dtype=np.float64), group, kind) if convrot else np.asarray(x, np.float64)
    w = np.asarray(q, dtype=np.float64) * np.asarray(scale, dtype=np.float64).reshape(-1, 1)
    return linear_f64(xr, w, bias)


def max_abs_rel(got, ref) -> float:
    """max |got - ref| / max |ref| (the north-star gate, 2e-3 for fp16 outputs)."""
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    den = np.abs(ref).max()
    return float(np.abs(got - ref).max() / (den if den > 0 else 1.0))


def rel_l2(got, ref) -> float:
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    den = np.linalg.norm(ref)
    return float(np.linalg.norm(got - ref) / (den if den > 0 else 1.0))


# ----------------------------------------------------------------------------------------------
# Seeded inputs of the benchmark configurations
# ----------------------------------------------------------------------------------------------

def cfg_int8_convrot(m=4096, k=3072, n=12288, seed=0, outlier_frac=0.01):
    """Configuration 2: X fp16 N(0,1) with 1% of K-channels x20; W int8 U[-127,127] (stored
    rotated); per-output-channel fp16 scale |N(0,0.02)|/127; fp16 bias N(0,0.01)."""
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(m, k, generator=g)
    idx = torch.randperm(k, generator=g)[: max(1, int(k * outlier_frac))]
    x[:, idx] *= 20
    q = torch.randint(-127, 128, (n, k), generator=g, dtype=torch.int32).to(torch.int8)
    s = (torch.randn(n, generator=g).abs() * 0.02 / 127).to(torch.float16)
    b = (torch.randn(n, generator=g) * 0.01).to(torch.float16)
    return x.to(torch.float16), q, s, b


def cfg_w4a8(m=4096, k=12288, n=3072, seed=0, group=128):
    """Configuration 3: X fp16 N(0,1); W uniform [-8,7] two per byte; fp16 group scales
    |N(0,0.02)|/7 per 128 K-columns."""
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(m, k, generator=g).to(torch.float16)
    wq = torch.randint(-8, 8, (n, k), generator=g, dtype=torch.int32)
    s = (torch.randn(n, k // group, generator=g).abs() * 0.02 / 7).to(torch.float16)
    return x, wq.numpy().astype(np.int8), s


def cfg_w6a8(m=3240, k=5120, n=13824, seed=0, group=64):
    """Configuration 4: X fp16 N(0,1); W uniform [-32,31] four per three bytes; fp16 group
    scales |N(0,0.02)|/31 per 64 K-columns."""
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(m, k, generator=g).to(torch.float16)
    wq = torch.randint(-32, 32, (n, k), generator=g, dtype=torch.int32)
    s = (torch.randn(n, k // group, generator=g).abs() * 0.02 / 31).to(torch.float16)
    return x, wq.numpy().astype(np.int8), s


def cfg_gguf(m=256, k=3072, n=3072, qtype=8, seed=0):
    """Configuration 1: X fp16 N(0,1) [M, K]; W raw GGUF blocks [N, K/QK*type_size]."""
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(m, k, generator=g).to(torch.float16)
    return x, baseline_gguf_blocks(qtype, n, k, seed)


# ----------------------------------------------------------------------------------------------
# Reference self-test inputs (bit-reproducible integer-derived tensors)
# ----------------------------------------------------------------------------------------------

def selftest_inputs():
    """Restates `modal/weight_error_app.py:421-437` (`selftest_inputs`): seeded integer draws and
    exact arithmetic only, so the tensors are identical on every platform."""
    g = torch.Generator().manual_seed(1234)

    def gauss(n, k):
        u = torch.randint(0, 65536, (12, n, k), generator=g, dtype=torch.int64).sum(0) - 6 * 65535
        return (u.double() * 2.0 ** -22).float().to(torch.bfloat16).float()

    wa = gauss(96, 1024)
    u = torch.randint(0, 256, (4, 96, 1024), generator=g, dtype=torch.int64).sum(0) - 510
    cubes = u.double() ** 3
    h = torch.from_numpy(hadamard_h4(256))
    rot = torch.matmul((cubes * 16.0).reshape(96, 4, 256), h.T).reshape(96, 1024)
    wb = (rot / 256.0 * 2.0 ** -30).float().to(torch.bfloat16).float()
    wc = gauss(4200, 1024)
    return {"gauss_96x1024": wa, "heavy_96x1024": wb, "chunked_4200x1024": wc}
