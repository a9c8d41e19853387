"""Named benchmark configurations, runnable on their own (for profiling and reproduction):

    python bench_cases.py cfg1_q8_0 --iters 3

Synthetic seeded inputs with the configurations' shapes and value distributions:
  cfg1_q8_0 / cfg1_q4_0   GGUF Q8_0 / Q4_0 linear, X fp16 [256, 3072], W [3072, 3072]
  cfg2                    INT8 ConvRot weight-only linear, X [4096, 3072], W [12288, 3072], H-128
  cfg2_grad               its input gradient: dY fp16 [4096, 12288] -> dX [4096, 3072], H-128
  cfg2_q4_0 / cfg2_iq4nl  GGUF Q4_0 / IQ4_NL linear at the configuration-2 shape
  cfg3                    W4A8, X [4096, 12288], W 4-bit [3072, 12288], group 128
  cfg4_fwd / cfg4_rev     W6A8, X [3240, 5120] / [3240, 13824], W 6-bit, group 64
  cfg5_q4k / cfg5_q6k     MMDiT-block GGUF linears, X [4608, 3072] / [4608, 12288]
  kitchen_w4a8 / _w6a8    kitchen layouts at the configuration-2 shape (grid decoded per call)
  small_q8_0_m1 / _m16 / _m64   the small-M path: Q8_0 [3072, 3072] with M = 1 / 16 / 64 tokens
  small_q4k_m1            the small-M path: Q4_K [12288, 3072], M = 1
"""
import argparse
import os
import sys

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "mac-kernels-public_b200")
for _p in (ROOT, PKG):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import torch  # noqa: E402

import qlin  # noqa: E402


def _gguf_blocks(qtype, n, k, gen, dev):
    name, qk, ts = qlin.GGUF_TYPES[qtype]
    nb = n * k // qk
    raw = torch.randint(0, 256, (nb, ts), generator=gen, dtype=torch.int32).to(torch.uint8)
    mag = {8: 0.02 / 127, 2: 0.02 / 7, 12: 5e-5, 14: 3e-5, 20: 3e-4}[qtype]
    offs = {8: [0], 2: [0], 12: [0, 2], 14: [208], 20: [0]}[qtype]
    for off in offs:
        d = (torch.randn(nb, generator=gen).abs() * mag).to(torch.float16)
        raw[:, off:off + 2] = d.view(torch.uint8).reshape(nb, 2)
    return raw.reshape(n, -1).to(dev)


def build(name, dev):
    """Returns (callable running the op once, flops per call)."""
    gen = torch.Generator().manual_seed(0)
    gguf_cases = {"cfg1_q8_0": (8, 256, 3072, 3072), "cfg1_q4_0": (2, 256, 3072, 3072),
                  "cfg2_q4_0": (2, 4096, 3072, 12288), "cfg2_iq4nl": (20, 4096, 3072, 12288),
                  "cfg5_q4k": (12, 4608, 3072, 9216), "cfg5_q6k": (14, 4608, 12288, 3072),
                  "small_q8_0_m1": (8, 1, 3072, 3072), "small_q8_0_m16": (8, 16, 3072, 3072),
                  "small_q8_0_m64": (8, 64, 3072, 3072), "small_q4k_m1": (12, 1, 3072, 12288)}
    if name in gguf_cases:
        qtype, m, k, n = gguf_cases[name]
        x = torch.randn(m, k, generator=gen).to(torch.float16).to(dev)
        raw = _gguf_blocks(qtype, n, k, gen, dev)
        qlin.repack_gguf(raw, qtype, (n, k))
        return (lambda: qlin.gguf_linear(x, raw, qtype, (n, k))), 2.0 * m * k * n
    if name == "cfg2":
        m, k, n = 4096, 3072, 12288
        x = torch.randn(m, k, generator=gen)
        x[:, torch.randperm(k, generator=gen)[: k // 100]] *= 20
        x = x.to(torch.float16).to(dev)
        q = torch.randint(-127, 128, (n, k), generator=gen, dtype=torch.int32).to(torch.int8).to(dev)
        s = (torch.randn(n, generator=gen).abs() * 0.02 / 127).to(torch.float16).to(dev)
        b = (torch.randn(n, generator=gen) * 0.01).to(torch.float16).to(dev)
        return (lambda: qlin.int8_linear(x, q, s, b, torch.float16, convrot=True, convrot_groupsize=128)), 2.0 * m * k * n
    if name == "cfg2_grad":
        m, k, n = 4096, 3072, 12288
        q = torch.randint(-127, 128, (n, k), generator=gen, dtype=torch.int32).to(torch.int8).to(dev)
        s = (torch.randn(n, generator=gen).abs() * 0.02 / 127).to(torch.float16).to(dev)
        dy = torch.randn(m, n, generator=gen).to(torch.float16).to(dev)
        qlin.int8_linear_grad_input(dy, q, s, True, 128)  # the one-time transposed weight copy
        return (lambda: qlin.int8_linear_grad_input(dy, q, s, True, 128)), 2.0 * m * k * n
    if name in ("kitchen_w4a8", "kitchen_w6a8"):
        # the kitchen layouts at the configuration-2 shape: codes decoded per call to the int8 grid
        m, k, n = 4096, 3072, 12288
        bits = 4 if name == "kitchen_w4a8" else 6
        x = torch.randn(m, k, generator=gen).to(torch.float16).to(dev)
        u = torch.randint(0, 1 << bits, (n, k), generator=gen, dtype=torch.int32)
        # planar kitchen packing: K/2 nibble bytes (even column low), then for 6 bits K/4 bytes of
        # 2-bit high planes (column 4j+i at bits 2i..2i+1 of byte j)
        planes = [(u[:, 0::2] & 0xF) | ((u[:, 1::2] & 0xF) << 4)]
        if bits == 6:
            planes.append(sum(((u[:, j::4] >> 4) & 3) << (2 * j) for j in range(4)))
        qdata = torch.cat(planes, dim=1).to(torch.uint8).view(torch.int8).to(dev)
        s_rel = (torch.rand(n, k // 16, generator=gen) * 12 + 2).to(torch.float8_e4m3fn).to(dev)
        s_ch = (torch.rand(n, generator=gen) * 1e-3 + 1e-4).to(dev)
        cb = (torch.sort(torch.randn(16, generator=gen)).values * 3).to(dev) if bits == 4 else None
        return (lambda: qlin.w4a8_int8_linear(x, qdata, s_rel, s_ch, cb, None, None, 16, 128, torch.float16)), \
            2.0 * m * k * n
    m, k, n, bits, grp = {"cfg3": (4096, 12288, 3072, 4, 128), "cfg4_fwd": (3240, 5120, 13824, 6, 64),
                          "cfg4_rev": (3240, 13824, 5120, 6, 64)}[name]
    x = torch.randn(m, k, generator=gen).to(torch.float16).to(dev)
    if bits == 4:
        u = torch.randint(0, 16, (n, k), generator=gen, dtype=torch.int32)
        w = (u[:, 0::2] | (u[:, 1::2] << 4)).to(torch.uint8)
    else:
        u = torch.randint(0, 64, (n, k), generator=gen, dtype=torch.int64)
        word = u[:, 0::4] | (u[:, 1::4] << 6) | (u[:, 2::4] << 12) | (u[:, 3::4] << 18)
        w = torch.stack([word & 0xFF, (word >> 8) & 0xFF, (word >> 16) & 0xFF], dim=-1).reshape(n, -1).to(torch.uint8)
    w = w.to(dev)
    s = (torch.randn(n, k // grp, generator=gen).abs() * 0.003).to(torch.float16).to(dev)
    return (lambda: qlin.w4a8_linear(x, w, s, bits=bits, group_size=grp)), 2.0 * m * k * n


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("case")
    ap.add_argument("--iters", type=int, default=3)
    a = ap.parse_args(argv)
    dev = torch.device("cuda", 0)
    fn, flops = build(a.case, dev)
    for _ in range(a.iters):
        fn()
    torch.cuda.synchronize()
    code, where = qlin.device_status()
    if code:
        print(f"device wait timed out at {where:#x}", file=sys.stderr)
        return 1
    print(f"{a.case}: ran {a.iters} calls ({flops / 1e9:.1f} GFLOP each)")
    return 0


if __name__ == "__main__":
    sys.exit(main())
