"""The bounds-checked build (libqlin_checked.so, compiled with -DQLIN_CHECKS) over every kernel
family at small and ragged shapes.

That build tests every plain global access and every computed shared-memory index against a limit
the host derives from the call's arguments, records the first failure and skips the access (it
never traps); TMA coordinates are also checked for 16-byte alignment.  The test runs the cases in a
child process that loads the checked library through QLIN_LIB, with fresh allocations poisoned, and
requires after every call: no failed check, no timed-out wait, and outputs that match the CPU
oracle.  Cases:

  GGUF linear     all twelve types at M = 1 (small-M kernel), 2, 37, 300 and a K-split shape;
                  fp32 / bf16 inputs (prologue), fp32 / bf16 outputs, bias; rows straddling blocks
  INT8 linear     ConvRot groups 128 (tensor-core prologue, rotated epilogue) and 256, plain
  W4A8 / W6A8     groups 64 / 128 / per channel, M = 33 (single-CTA kernel) and 100 / 300 (pairs)
  kitchen         W4A8 codebook and W6A8 grid decode + linear
  LoRA            fused low-rank path (down projection on the GEMM, up stages in the K loop)
  gradients       INT8 input gradient (transpose, gradient prologue, rotation)
  decode          dequantize_gguf, quantize_int8_rowwise, prologue_f16
"""
import os
import subprocess
import sys

import numpy as np
import pytest
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
PKG = os.path.join(ROOT, "mac-kernels-public_b200")
CHECKED = os.path.join(PKG, "qlin", "libqlin_checked.so")


@pytest.mark.gpu
def test_checked_build_finds_no_out_of_bounds_access():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    assert os.path.exists(CHECKED), "build it with: python mac-kernels-public_b200/build.py --checks"
    env = dict(os.environ, QLIN_LIB=CHECKED)
    r = subprocess.run([sys.executable, os.path.abspath(__file__)], env=env, capture_output=True, text=True,
                       timeout=900)
    print(r.stdout[-6000:])
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert "cases clean" in r.stdout


# ---------------------------------------------------------------------------------------- child
def _child():
    for p in (ROOT, PKG, HERE):
        if p not in sys.path:
            sys.path.insert(0, p)
    import qlin
    from qlin import _lib
    from oracle import qlin_oracle as O

    assert os.path.samefile(_lib.LIB_PATH, CHECKED), _lib.LIB_PATH
    assert qlin.bounds_check() is None  # the checked build answers (the ordinary one declines)
    torch.use_deterministic_algorithms(True, warn_only=True)
    torch.utils.deterministic.fill_uninitialized_memory = True
    dev = torch.device("cuda:0")
    done = []

    def clean(name, got=None, ref=None, tol=2e-3):
        torch.cuda.synchronize()
        rec = qlin.bounds_check()
        assert rec is None, f"{name}: {rec}"
        code, where = qlin.device_status(reset=True)
        assert code == 0, f"{name}: a wait timed out at {where:#x}"
        if got is not None:
            g = got.float().cpu().numpy() if isinstance(got, torch.Tensor) else got
            assert np.isfinite(g).all(), f"{name}: non-finite output"
            err = O.max_abs_rel(g, ref)
            assert err <= tol, (name, err)
        done.append(name)

    # GGUF linear: every type, small-M / GEMM / K-split shapes, input and output dtypes
    for qtype in sorted(O.GGUF_TYPES):
        name = O.GGUF_TYPES[qtype][0]
        for m, n, k in ((1, 200, 512), (2, 136, 768), (37, 130, 1024), (300, 256, 512), (24, 128, 8192)):
            raw = O.random_gguf_blocks(qtype, n, k, seed=qtype * 7 + m)
            g = torch.Generator().manual_seed(m + k)
            x = torch.randn(m, k, generator=g)
            b = (torch.randn(n, generator=g) * 0.1).to(torch.float16)
            w = O.gguf_dequantize(raw, qtype, n, k)
            for xdt, odt in ((torch.float16, torch.float16), (torch.bfloat16, torch.float32),
                             (torch.float32, torch.bfloat16)):
                xx = x.to(xdt)
                ref = O.linear_f64(xx.float().numpy(), w, b.float().numpy())
                y = qlin.gguf_linear(xx.to(dev), torch.from_numpy(raw).to(dev), qtype, (n, k), bias=b.to(dev),
                                     out_dtype=odt)
                clean(f"gguf {name} {m}x{n}x{k} {xdt} -> {odt}", y, ref, tol=2e-3 if odt != torch.bfloat16 else 8e-3)
    # rows straddling blocks (repacked to fp16 rows)
    for qtype, n, k in ((12, 12, 1152), (8, 70, 1104), (23, 96, 1920)):
        raw = O.random_gguf_blocks(qtype, 1, n * k, seed=5)
        x = torch.randn(40, k, generator=torch.Generator().manual_seed(1)).to(torch.float16)
        ref = O.linear_f64(x.float().numpy(), O.gguf_dequantize(raw, qtype, 1, n * k).reshape(n, k))
        y = qlin.gguf_linear(x.to(dev), torch.from_numpy(raw).to(dev), qtype, (n, k))
        clean(f"gguf straddle {O.GGUF_TYPES[qtype][0]} {n}x{k}", y, ref)

    # INT8 ConvRot / plain
    for m, n, k, rot in ((1, 256, 1024, 128), (70, 200, 1024, 128), (300, 384, 2048, 256), (33, 136, 512, 0)):
        x, q, s, b = O.cfg_int8_convrot(m, k, n, seed=m)
        y = qlin.int8_linear(x.to(dev), q.to(dev), s.to(dev), b.to(dev), torch.float16, convrot=rot > 0,
                             convrot_groupsize=rot or 256)
        ref = O.int8_convrot_linear_ref(x.float().numpy(), q.numpy(), s.float().numpy(), b.float().numpy(),
                                        group=rot or 128, convrot=rot > 0)
        clean(f"int8 {m}x{n}x{k} rot {rot}", y, ref)

    # W4A8 / W6A8 benchmark layouts
    for bits, group, m in ((4, 128, 33), (4, 128, 300), (4, 64, 100), (4, 0, 130), (6, 64, 300), (6, 128, 33),
                           (6, 256, 100), (6, 0, 300)):
        n, k = 320, 1024
        gen = torch.Generator().manual_seed(bits * 100 + m)
        x = torch.randn(m, k, generator=gen).to(torch.float16)
        lo, hi = (-8, 8) if bits == 4 else (-32, 32)
        wq = torch.randint(lo, hi, (n, k), generator=gen, dtype=torch.int32).numpy().astype(np.int8)
        gs = group or k
        s = (torch.rand(n, k // gs, generator=gen) * 0.01 + 0.001)
        s = s.to(torch.float16) if group else s.reshape(n).float()
        b = (torch.randn(n, generator=gen) * 0.01).to(torch.float16)
        packed = O.pack_w4_uniform(wq).view(np.uint8) if bits == 4 else O.pack_w6_interleaved(wq)
        ref, _, _ = O.grouped_linear_a8(x.numpy(), wq, s.float().numpy().reshape(n, -1), gs, b.float().numpy())
        y = qlin.w4a8_linear(x.to(dev), torch.from_numpy(np.ascontiguousarray(packed)).to(dev), s.to(dev), bits=bits,
                             group_size=group, bias=b.to(dev))
        clean(f"w{bits}a8 g{group} {m}x{n}x{k}", y, ref)

    # kitchen grid + linear
    z = np.load(os.path.join(HERE, "golden", "kitchen_w4a8.npz"))
    for fmt, bits in (("w4a8", 4), ("w6a8", 6)):
        q = torch.from_numpy(z[f"{fmt}_q"]).to(dev)
        s_rel = torch.from_numpy(z[f"{fmt}_s_rel"]).view(torch.float8_e4m3fn).to(dev)
        s_ch = torch.from_numpy(z[f"{fmt}_s_channel"]).to(dev)
        cb = torch.from_numpy(z["w4a8_codebook"]).to(dev) if fmt == "w4a8" else None
        x = torch.randn(40, 1024, generator=torch.Generator().manual_seed(bits)).to(torch.float16)
        w = O.dequantize_kitchen_w4a8(z[f"{fmt}_q"], z[f"{fmt}_s_rel"], z[f"{fmt}_s_channel"], 1024, bits, 16,
                                      z["w4a8_codebook"] if fmt == "w4a8" else None, 256)
        y = qlin.w4a8_int8_linear(x.to(dev), q, s_rel, s_ch, cb, None, None, 16, 256)
        clean(f"kitchen {fmt}", y, O.linear_f64(x.float().numpy(), w))

    # fused LoRA (bf16 activations, rank 16) on GGUF Q8_0
    n, k, rank = 256, 1024, 16
    raw = O.random_gguf_blocks(8, n, k, seed=9)
    gen = torch.Generator().manual_seed(9)
    x = torch.randn(50, k, generator=gen).to(torch.bfloat16)
    down = (torch.randn(rank, k, generator=gen) * 0.02).to(torch.bfloat16)
    up = (torch.randn(n, rank, generator=gen) * 0.02).to(torch.bfloat16)
    wf = O.gguf_dequantize(raw, 8, n, k).astype(np.float64)
    xf = x.double().numpy()
    ref = xf @ wf.T + 0.5 * (xf @ down.double().numpy().T) @ up.double().numpy().T
    y = qlin.gguf_linear(x.to(dev), torch.from_numpy(raw).to(dev), 8, (n, k), lora_down=down.to(dev),
                         lora_up=up.to(dev), lora_scale=0.5)
    clean("gguf Q8_0 fused LoRA rank 16", y, ref, tol=8e-3)

    # INT8 input gradient
    for group in (128, 0):
        _, q, s, _ = O.cfg_int8_convrot(8, 1024, 200, seed=3)
        dy = torch.randn(70, 200, generator=torch.Generator().manual_seed(4)).to(torch.float16)
        dx = qlin.int8_linear_grad_input(dy.to(dev), q.to(dev), s.to(dev), group > 0, group or 256)
        clean(f"int8 grad input group {group}", dx, O.int8_grad_input(dy.double().numpy(), q.numpy(),
                                                                       s.float().numpy(), group))

    # decode-only and prologue entry points
    raw = O.random_gguf_blocks(14, 64, 512, seed=2)
    wd = qlin.dequantize_gguf(torch.from_numpy(raw).to(dev), 14, (64, 512))
    clean("dequantize_gguf Q6_K", wd, O.gguf_dequantize(raw, 14, 64, 512), tol=0.0)
    x = torch.randn(45, 1000, generator=torch.Generator().manual_seed(6)).to(torch.float16)
    xq, sx = qlin.quantize_int8_rowwise(x.to(dev))
    q_ref, s_ref = O.quantize_int8_rowwise(x)
    clean("quantize_int8_rowwise")
    assert torch.equal(xq.cpu(), q_ref) and torch.equal(sx.cpu().reshape(s_ref.shape), s_ref)
    x = torch.randn(45, 1024, generator=torch.Generator().manual_seed(7)).to(torch.bfloat16)
    qlin.prologue_f16(x.to(dev), rotate_group=128)
    clean("prologue_f16 rot 128")
    print(f"{len(done)} cases clean under the bounds-checked build")


if __name__ == "__main__":
    _child()
