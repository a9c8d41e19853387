"""W4A8 / W6A8 linears on the integer tensor cores (kind::i8) behind the kitchen surface.

`w4a8_linear` serves the symmetric uniform packed layouts (4-bit nibbles; 6-bit "four values per
three bytes" or the kitchen's planar 6-bit packing) with fp16 group scales or fp32 per-channel
scales.  Activations are quantized per token with the reference's `quantize_int8_rowwise`
rounding; every group's int32 partial is exact.
"""
from __future__ import annotations

import ctypes
import weakref

import torch

from ._lib import QlinDecline, check, lib

_DT = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}
_CACHE: dict = {}


def repack_w(qweight, bits, layout, n, k):
    """One-time conversion of packed weights into the kernel's stage layout (cached per tensor).
    4-bit weights are used as stored."""
    if bits == 4:
        return qweight.contiguous()
    key = (qweight.data_ptr(), qweight.device.index, bits, layout, n, k, qweight._version)
    hit = _CACHE.get(key)
    if hit is not None:
        return hit
    nbytes = ctypes.c_size_t(0)
    check(lib.qlin_w4a8_repacked_bytes(bits, layout, n, k, ctypes.byref(nbytes)), "qlin_w4a8_repacked_bytes")
    src = qweight.contiguous()
    out = torch.empty(nbytes.value, dtype=torch.uint8, device=qweight.device)
    check(lib.qlin_w4a8_repack(src.data_ptr(), bits, layout, n, k, out.data_ptr(), nbytes.value,
                               torch.cuda.current_stream(qweight.device).cuda_stream), "qlin_w4a8_repack")
    _CACHE[key] = out
    try:
        weakref.finalize(qweight, _CACHE.pop, key, None)
    except TypeError:
        pass
    return out


def w4a8_linear(x, qweight, scales, bits=4, group_size=128, layout=0, bias=None, out_dtype=None, rotate_group=0):
    """y = sx * sum_g s[:, g] * (xq . wq_g^T) + bias.

    qweight: uint8/int8 packed weights of logical shape [N, K] (4-bit: [N, K/2]; 6-bit: [N, 3K/4]).
    scales:  fp16 [N, K/group_size], or fp32 [N] with group_size=0 (per-channel)."""
    if not x.is_cuda or not qweight.is_cuda:
        raise NotImplementedError("qlin runs on CUDA tensors only (there is no CPU path)")
    n = qweight.shape[0]
    k = x.shape[-1]
    y = torch.empty(*x.shape[:-1], n, dtype=out_dtype or x.dtype, device=x.device)
    if x.numel() == 0 or n == 0:
        return y
    if x.dtype not in _DT or y.dtype not in _DT:
        raise QlinDecline(1, "w4a8_linear: unsupported dtype")
    x2 = x.reshape(-1, k)
    if x2.stride(-1) != 1:
        x2 = x2.contiguous()
    m = x2.shape[0]
    w = repack_w(qweight, bits, layout, n, k)
    if group_size:
        sc = scales.to(torch.float16).contiguous()
        sdt = 1
    else:
        sc = scales.reshape(-1).float().contiguous()
        sdt = 0
    b = None if bias is None else bias.contiguous()
    if b is not None and b.dtype not in _DT:
        b = b.float()
    ws_bytes = lib.qlin_w4a8_linear_workspace(m, n, k, rotate_group)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=x.device)
    y2 = y.view(m, n)
    check(lib.qlin_w4a8_linear(x2.data_ptr(), _DT[x2.dtype], m, k, x2.stride(0), w.data_ptr(), bits, group_size, n,
                               sc.data_ptr(), sdt, rotate_group, None if b is None else b.data_ptr(),
                               0 if b is None else _DT[b.dtype], y2.data_ptr(), _DT[y2.dtype], n, ws.data_ptr(),
                               ws_bytes, torch.cuda.current_stream(x.device).cuda_stream), "qlin_w4a8_linear")
    return y


def w4a8_int8_linear(x, qdata, s_rel, s_channel, codebook=None, correction=None, bias=None, group_size=16,
                     convrot_groupsize=256, out_dtype=None, lora_down=None, lora_up=None, lora_scale=None):
    """comfy-kitchen AsymW4A8Int8Layout linear (bench/bench_lora_fused_rank.py:42-44)."""
    raise QlinDecline(1, "w4a8_int8_linear: the kitchen AsymW4A8Int8Layout path is not built yet")
