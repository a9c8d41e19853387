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


def _hadamard(g, device):
    """The rotation's block matrix: H4 (x) ... (x) H4 for powers of four (the reference's
    build_hadamard, modal/weight_error_app.py:90-98), else Sylvester; orthonormal."""
    import math
    h = torch.ones(1, 1, dtype=torch.float64)
    if 4 ** round(math.log(g, 4)) == g:
        h4 = torch.ones(4, 4, dtype=torch.float64) - 2 * torch.eye(4, dtype=torch.float64).flip(0)
        while h.shape[0] < g:
            h = torch.kron(h, h4)
    else:
        h2 = torch.tensor([[1.0, 1.0], [1.0, -1.0]], dtype=torch.float64)
        while h.shape[0] < g:
            h = torch.kron(h, h2)
    return (h / math.sqrt(g)).to(device=device, dtype=torch.float32)


def kitchen_grid(qdata, s_rel, codebook=None, group_size=16):
    """The int8 weight grid [N, K] of a kitchen W4A8 / W6A8 weight, decoded on the GPU (bit-exact).

    The grid is transient: every linear decodes it from the packed codes into a fresh tensor that
    the caching allocator takes back after the call, so what stays resident per weight is only the
    caller's packed codes and scales (N*K*bits/8 + N*K/group bytes), as the format intends.  The
    decode costs one pass writing N*K bytes per call (most of which the following GEMM then reads
    back from L2)."""
    if not qdata.is_cuda or not s_rel.is_cuda:
        raise NotImplementedError("qlin runs on CUDA tensors only (there is no CPU path)")
    n = qdata.shape[0]
    k = s_rel.shape[1] * group_size
    bits = qdata.shape[1] * 8 // k
    if bits not in (4, 6) or qdata.shape[1] * 8 != bits * k:
        raise QlinDecline(1, "w4a8_int8_linear: qdata width matches neither 4 nor 6 bits")
    cb = None
    if codebook is not None:
        cb = codebook.to(device=qdata.device, dtype=torch.float32).contiguous()
        if cb.numel() != 1 << bits:
            raise QlinDecline(1, f"w4a8_int8_linear: a {bits}-bit codebook has {1 << bits} levels")
    q = qdata.contiguous()
    sr = s_rel.contiguous().view(torch.uint8)
    out = torch.empty(n, k, dtype=torch.int8, device=qdata.device)
    check(lib.qlin_kitchen_w4a8_grid(q.data_ptr(), bits, sr.data_ptr(), None if cb is None else cb.data_ptr(),
                                     group_size, n, k, out.data_ptr(),
                                     torch.cuda.current_stream(qdata.device).cuda_stream), "qlin_kitchen_w4a8_grid")
    return out


def w4a8_int8_linear(x, qdata, s_rel, s_channel, codebook=None, correction=None, bias=None, group_size=16,
                     convrot_groupsize=256, out_dtype=None, lora_down=None, lora_up=None, lora_scale=None):
    """comfy-kitchen AsymW4A8Int8Layout linear (bench/bench_lora_fused_rank.py:42-44;
    bench/bench_w4a8_linear.py:83), symmetric form.  Like the reference backend it is weight-only
    (docs/upstream/comfy-kitchen-mps-backend.md:42): the stored codes decode per call to the exact
    int8 grid (a transient tensor), and the linear is the INT8 ConvRot linear with s_channel per
    output channel.  An
    asymmetric `correction` declines (QlinDecline), as an unsupported layout does in the kitchen."""
    if correction is not None:
        raise QlinDecline(1, "w4a8_int8_linear: the asymmetric correction term is not supported")
    from . import int8_linear
    grid = kitchen_grid(qdata, s_rel, codebook, group_size)  # transient: freed when the call returns
    return int8_linear(x, grid, s_channel.float().reshape(-1), bias, out_dtype=out_dtype,
                       convrot=convrot_groupsize > 0, convrot_groupsize=convrot_groupsize,
                       lora_down=lora_down, lora_up=lora_up, lora_scale=lora_scale)


def dequantize_w4a8_int8_weight(qdata, s_rel, s_channel, codebook=None, correction=None, group_size=16,
                                convrot_groupsize=256, output_dtype=torch.float32):
    """Decode-only entry point (docs/upstream/comfy-kitchen-mps-backend.md:30): the weight in the
    original basis, grid * s_channel un-rotated per block (modal/weight_error_app.py:326-339)."""
    if correction is not None:
        raise QlinDecline(1, "dequantize_w4a8_int8_weight: the asymmetric correction term is not supported")
    grid = kitchen_grid(qdata, s_rel, codebook, group_size)
    w = grid.float() * s_channel.float().reshape(-1, 1)
    if convrot_groupsize:
        g = convrot_groupsize
        n, k = w.shape
        w = (w.view(n, k // g, g) @ _hadamard(g, w.device)).view(n, k)
    return w.to(output_dtype)
