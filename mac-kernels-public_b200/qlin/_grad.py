"""Input gradients of the packed linears for frozen weights (LoRA training on a packed base).

Names and argument order follow comfy-kitchen's MPS autograd entry points as the reference calls
them:
  int8_linear_grad_input(dy, q, s, convrot, convrot_groupsize, out_dtype=)
      bench/bench_int8_backward.py:52, bench/probe_packed_backward_real_k.py:151
  w4a8_linear_grad_input(dy, q, s_rel, s_channel, codebook, correction, group_size,
                         convrot_groupsize, out_dtype)
      bench/probe_packed_backward_real_k.py:152
  int8_linear_trainable(x, q, s, bias, convrot, convrot_groupsize)
      bench/bench_int8_backward.py:70, bench/probe_packed_backward_real_k.py:157
  w4a8_linear_trainable(x, q, s_rel, s_channel, codebook, correction, bias, group_size,
                        convrot_groupsize)
      bench/probe_packed_backward_real_k.py:158

dx = dy . W with W the weight in the original basis, (q * s) un-rotated per block.  The library
reads a transposed copy of q (int8 [K, roundup(N, 64)], made once per weight tensor version and
cached like the GGUF repack), scales dy's columns by s, runs the same tensor-core GEMM as the
forward over N, and rotates dx's rows.  The W4A8 / W6A8 kitchen layout goes through its int8 grid,
as its forward does.
"""
from __future__ import annotations

import weakref

import torch

from ._lib import QlinDecline, check, lib

_GRAD_WEIGHT_CACHE: dict = {}
_DT = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}


def grad_weight(qdata, cache=True):
    """The transposed int8 copy of `qdata` [N, K] the gradient GEMM reads (cached per tensor version
    unless cache=False, for a transient weight such as a decoded kitchen grid)."""
    n, k = qdata.shape
    key = (qdata.data_ptr(), qdata.device.index, n, k, qdata._version)
    hit = _GRAD_WEIGHT_CACHE.get(key) if cache else None
    if hit is not None:
        return hit
    nbytes = lib.qlin_int8_grad_weight_bytes(n, k)
    qt = torch.empty(nbytes, dtype=torch.int8, device=qdata.device)
    q = qdata.contiguous()
    check(lib.qlin_int8_grad_weight(q.data_ptr(), n, k, qt.data_ptr(), nbytes,
                                    torch.cuda.current_stream(qdata.device).cuda_stream), "qlin_int8_grad_weight")
    if not cache:
        return qt
    _GRAD_WEIGHT_CACHE[key] = qt
    try:
        weakref.finalize(qdata, _GRAD_WEIGHT_CACHE.pop, key, None)
    except TypeError:
        pass
    return qt


def int8_linear_grad_input(dy, qdata, scale, convrot=False, convrot_groupsize=256, out_dtype=None, *,
                           _transient_weight=False):
    """dx = dy . W for the frozen INT8 (ConvRot) weight W = (qdata * scale) un-rotated per block;
    dy [..., N] float, returns [..., K] in out_dtype (default dy's dtype).  The transposed weight
    copy is cached per weight tensor, except for a weight decoded for this call only
    (_transient_weight, the kitchen grid)."""
    for t in (dy, qdata):
        if not t.is_cuda:
            raise NotImplementedError("qlin runs on CUDA tensors only (there is no CPU path)")
    if qdata.dtype != torch.int8 or qdata.dim() != 2:
        raise QlinDecline(1, "int8_linear_grad_input: qdata must be a 2-D int8 tensor")
    n, k = qdata.shape
    if dy.shape[-1] != n:
        raise ValueError(f"int8_linear_grad_input: dy has {dy.shape[-1]} features, weight has {n} rows")
    out_dtype = out_dtype or dy.dtype
    if dy.dtype not in _DT or out_dtype not in _DT:
        raise QlinDecline(1, "int8_linear_grad_input: dy and dx must be f32, f16 or bf16")
    dx = torch.empty(*dy.shape[:-1], k, dtype=out_dtype, device=dy.device)
    if dx.numel() == 0:
        return dx
    m = dx.numel() // k
    dy2 = dy.reshape(m, n)
    if n > 0 and dy2.stride(-1) != 1:
        dy2 = dy2.contiguous()
    sc = scale.reshape(-1)
    if sc.numel() == 1:
        sc = sc.expand(n)
    if sc.dtype not in (torch.float32, torch.float16):
        sc = sc.float()
    sc = sc.contiguous()
    group = convrot_groupsize if convrot else 0
    qt = grad_weight(qdata, cache=not _transient_weight) if n > 0 else None
    nws = lib.qlin_int8_linear_grad_input_workspace(m, n, k, group)
    ws = torch.empty(nws, dtype=torch.uint8, device=dy.device) if nws else None
    check(lib.qlin_int8_linear_grad_input(dy2.data_ptr() if n > 0 else None, _DT[dy2.dtype], m, n,
                                          dy2.stride(0) if n > 0 else 0, None if qt is None else qt.data_ptr(), k,
                                          sc.data_ptr() if n > 0 else None, _DT[sc.dtype], group, dx.data_ptr(),
                                          _DT[out_dtype], k, None if ws is None else ws.data_ptr(), nws,
                                          torch.cuda.current_stream(dy.device).cuda_stream),
          "qlin_int8_linear_grad_input")
    return dx


def w4a8_linear_grad_input(dy, qdata, s_rel, s_channel, codebook=None, correction=None, group_size=16,
                           convrot_groupsize=256, out_dtype=None):
    """dx = dy . W for the frozen kitchen AsymW4A8Int8Layout weight (symmetric form): the int8
    grid times s_channel, un-rotated per block.  An asymmetric `correction` declines."""
    if correction is not None:
        raise QlinDecline(1, "w4a8_linear_grad_input: the asymmetric correction term is not supported")
    from ._w4a8 import kitchen_grid
    grid = kitchen_grid(qdata, s_rel, codebook, group_size)  # transient, like the forward's
    return int8_linear_grad_input(dy, grid, s_channel.float().reshape(-1), convrot_groupsize > 0,
                                  convrot_groupsize, out_dtype, _transient_weight=True)


class _Int8Trainable(torch.autograd.Function):
    """y = int8_linear(x, ...); backward gives x (and a bias that requires grad) their gradients,
    the packed weight stays frozen."""

    @staticmethod
    def forward(ctx, x, qdata, scale, bias, convrot, convrot_groupsize, transient=False):
        from . import int8_linear
        ctx.save_for_backward(qdata, scale)
        ctx.rot = (convrot, convrot_groupsize)
        ctx.transient = transient
        ctx.x_dtype = x.dtype
        ctx.bias_dtype = None if bias is None else bias.dtype
        return int8_linear(x, qdata, scale, bias, out_dtype=x.dtype, convrot=convrot,
                           convrot_groupsize=convrot_groupsize)

    @staticmethod
    def backward(ctx, gy):
        qdata, scale = ctx.saved_tensors
        gx = gb = None
        if ctx.needs_input_grad[0]:
            gx = int8_linear_grad_input(gy, qdata, scale, ctx.rot[0], ctx.rot[1], out_dtype=ctx.x_dtype,
                                        _transient_weight=ctx.transient)
        if ctx.bias_dtype is not None and ctx.needs_input_grad[3]:
            gb = gy.reshape(-1, gy.shape[-1]).float().sum(0).to(ctx.bias_dtype)
        return gx, None, None, gb, None, None, None


def int8_linear_trainable(x, qdata, scale, bias=None, convrot=False, convrot_groupsize=256):
    """int8_linear with autograd: gradients for x (and bias), none for the frozen packed weight."""
    return _Int8Trainable.apply(x, qdata, scale, bias, convrot, convrot_groupsize)


def w4a8_linear_trainable(x, qdata, s_rel, s_channel, codebook=None, correction=None, bias=None, group_size=16,
                          convrot_groupsize=256):
    """w4a8_int8_linear with autograd, through the kitchen layout's int8 grid (decoded for this call
    and kept by autograd until the backward pass, like an activation)."""
    if correction is not None:
        raise QlinDecline(1, "w4a8_linear_trainable: the asymmetric correction term is not supported")
    from ._w4a8 import kitchen_grid
    grid = kitchen_grid(qdata, s_rel, codebook, group_size)
    return _Int8Trainable.apply(x, grid, s_channel.float().reshape(-1), bias, convrot_groupsize > 0,
                                convrot_groupsize, True)
