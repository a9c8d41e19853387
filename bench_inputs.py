"""Seeded synthetic inputs of the benchmark configurations, for bench.py and bench_cases.py.

The configurations' shapes and value distributions drawn from fixed
seeds, and the host-side packing of the benchmark weight layouts.  This module is measurement
infrastructure written independently of the CPU oracle, so the bench never calls the oracle except
as the checker of its pre-timing parity test and as its CPU baseline; tests/test_bench_inputs.py
checks that the packings here equal the oracle's byte for byte.

GGUF block types (ggml ids): 2 Q4_0, 3 Q4_1, 6 Q5_0, 7 Q5_1, 8 Q8_0, 10 Q2_K, 11 Q3_K, 12 Q4_K,
13 Q5_K, 14 Q6_K, 20 IQ4_NL, 23 IQ4_XS.
"""
import numpy as np
import torch

# ggml type id -> (name, values per block, bytes per block)
GGUF_TYPES = {2: ("Q4_0", 32, 18), 3: ("Q4_1", 32, 20), 6: ("Q5_0", 32, 22), 7: ("Q5_1", 32, 24),
              8: ("Q8_0", 32, 34), 10: ("Q2_K", 256, 84), 11: ("Q3_K", 256, 110), 12: ("Q4_K", 256, 144),
              13: ("Q5_K", 256, 176), 14: ("Q6_K", 256, 210), 20: ("IQ4_NL", 32, 18), 23: ("IQ4_XS", 256, 136)}

# name -> (byte offsets of the fp16 block scales, their magnitude): realistic scale fields so decoded
# weights and linear outputs stay in a normal range
_SCALE_FIELDS = {"Q4_0": ([0], 5e-3), "Q4_1": ([0], 1.5e-3), "Q5_0": ([0], 1.5e-3), "Q5_1": ([0], 7e-4),
                 "Q8_0": ([0], 3e-4), "Q2_K": ([80, 82], 4e-4), "Q3_K": ([108], 2e-4),
                 "Q4_K": ([0, 2], 5e-5), "Q5_K": ([0, 2], 3e-5), "Q6_K": ([208], 3e-5),
                 "IQ4_NL": ([0], 3e-4), "IQ4_XS": ([0], 1e-5)}


def _f16_bytes(v):
    return np.asarray(v, dtype=np.float16).view(np.uint8).reshape(-1, 2)


def gguf_blocks(qtype, n, k, seed=0):
    """Random legal GGUF blocks uint8 [n, k/QK*type_size]: uniform bytes, the fp16 scale fields
    replaced by positive values of the type's magnitude (Q4_1 / Q5_1 block minimum negative)."""
    name, qk, ts = GGUF_TYPES[qtype]
    offs, mag = _SCALE_FIELDS[name]
    rng = np.random.default_rng(seed)
    nb = n * k // qk
    raw = rng.integers(0, 256, size=(nb, ts), dtype=np.uint8)
    for off in offs:
        raw[:, off:off + 2] = _f16_bytes(np.abs(rng.normal(mag, mag, nb)))
    if name in ("Q4_1", "Q5_1"):
        raw[:, 2:4] = _f16_bytes(-np.abs(rng.normal(0.0, 8 * mag, nb)))
    return raw.reshape(n, (k // qk) * ts)


def cfg1_gguf(m=256, k=3072, n=3072, qtype=8, seed=0):
    """Configuration 1: X fp16 N(0,1) [M, K]; W Q8_0 (d = |N(0,0.02)|/127, codes U[-127,127]) or
    Q4_0 (d = |N(0,0.02)|/7, nibbles U[0,15]) blocks [N, K/32 * type_size] (other types: random
    blocks of `gguf_blocks`)."""
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(m, k, generator=g).to(torch.float16)
    rng = np.random.default_rng(seed + 1)
    nb = n * k // 32
    if qtype == 8:
        blocks = np.empty((nb, 34), dtype=np.uint8)
        blocks[:, 0:2] = _f16_bytes(np.abs(rng.normal(0.0, 0.02, nb)) / 127)
        blocks[:, 2:] = rng.integers(-127, 128, size=(nb, 32)).astype(np.int8).view(np.uint8)
    elif qtype == 2:
        blocks = np.empty((nb, 18), dtype=np.uint8)
        blocks[:, 0:2] = _f16_bytes(np.abs(rng.normal(0.0, 0.02, nb)) / 7)
        blocks[:, 2:] = rng.integers(0, 256, size=(nb, 16), dtype=np.uint8)
    else:  # other types at configuration 1's shapes: the generic random blocks
        return x, gguf_blocks(qtype, n, k, seed)
    return x, blocks.reshape(n, -1)


def cfg2_int8_convrot(m=4096, k=3072, n=12288, seed=0, outlier_frac=0.01):
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


def pack_w4(q):
    """Symmetric 4-bit values [N, K] in [-8, 7] -> uint8 [N, K/2]: u = q + 8, even column in the
    low nibble."""
    u = torch.as_tensor(q).to(torch.int32) + 8
    return ((u[:, 0::2] & 0xF) | ((u[:, 1::2] & 0xF) << 4)).to(torch.uint8)


def pack_w6(q):
    """Symmetric 6-bit values [N, K] in [-32, 31] -> uint8 [N, 3K/4], four values per three bytes:
    u0 | u1<<6 | u2<<12 | u3<<18 (u = q + 32) little-endian."""
    u = torch.as_tensor(q).to(torch.int64) + 32
    word = u[:, 0::4] | (u[:, 1::4] << 6) | (u[:, 2::4] << 12) | (u[:, 3::4] << 18)
    return torch.stack([word & 0xFF, (word >> 8) & 0xFF, (word >> 16) & 0xFF], dim=-1).reshape(u.shape[0], -1) \
        .to(torch.uint8)


def pack_kitchen(codes, bits):
    """comfy-kitchen planar packing of unsigned codes [N, K] -> int8 [N, K*bits/8]: K/2 nibble bytes
    (even column low), then for 6 bits K/4 bytes of 2-bit high planes (column 4j+i at bits
    2i..2i+1 of byte j)."""
    u = torch.as_tensor(codes).to(torch.int32)
    planes = [(u[:, 0::2] & 0xF) | ((u[:, 1::2] & 0xF) << 4)]
    if bits == 6:
        planes.append(sum(((u[:, j::4] >> 4) & 3) << (2 * j) for j in range(4)))
    return torch.cat(planes, dim=1).to(torch.uint8).view(torch.int8)
