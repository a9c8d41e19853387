"""qlin: B200-native quantized linears behind the comfy-kitchen operator surface.

Python signatures follow the reference's callers (roblennon/mac-kernels-public):
  int8_linear          bench/bench_ck01_int8.py:57, bench/bench_lora_fused_rank.py:39
  gguf_linear          bench/bench_gguf_linear.py:120
  dequantize_gguf      docs/upstream/comfy-kitchen-mps-followups.md:43
  w4a8_int8_linear     bench/bench_lora_fused_rank.py:42-44, bench/bench_lora_sidepath_kernel.py:78
  quantize_int8_rowwise  modal/weight_error_app.py:109-115 (activation quantizer of the A8 formats)
  int8_linear_grad_input, w4a8_linear_grad_input, int8_linear_trainable, w4a8_linear_trainable
                       bench/bench_int8_backward.py:52,70, bench/probe_packed_backward_real_k.py:151-158

Every op runs the CUDA library (libqlin.so, sm_100a) on the tensors' device and the current
stream.  There is no CPU or eager fallback: unsupported inputs raise `QlinDecline`
(a NotImplementedError), the way the kitchen registry reports an unsupported backend.
Leading dimensions of x are flattened; empty contractions return before any launch.
"""
from __future__ import annotations

import weakref

import torch

from . import _lib
from ._lib import QlinDecline, QlinError, check, lib

__all__ = ["int8_linear", "int8_linear_streamed", "gguf_linear", "gguf_linear_slabs", "gguf_linear_allgather", "peer_wait", "dequantize_gguf", "w4a8_linear", "w4a8_int8_linear", "dequantize_w4a8_int8_weight",
           "quantize_int8_rowwise", "prologue_f16", "repack_gguf", "GGUF_TYPES", "QlinDecline", "QlinError",
           "device_status", "bounds_check", "int8_linear_grad_input", "w4a8_linear_grad_input", "int8_linear_trainable",
           "w4a8_linear_trainable"]

# ggml type id -> (name, values per block, bytes per block)
GGUF_TYPES = {2: ("Q4_0", 32, 18), 3: ("Q4_1", 32, 20), 6: ("Q5_0", 32, 22), 7: ("Q5_1", 32, 24),
              8: ("Q8_0", 32, 34), 10: ("Q2_K", 256, 84), 11: ("Q3_K", 256, 110), 12: ("Q4_K", 256, 144),
              13: ("Q5_K", 256, 176), 14: ("Q6_K", 256, 210), 20: ("IQ4_NL", 32, 18), 23: ("IQ4_XS", 256, 136)}
GGUF_IDS = {v[0]: k for k, v in GGUF_TYPES.items()}
_DT = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2, torch.int8: 3, torch.uint8: 4, torch.int32: 5,
       torch.float8_e4m3fn: 6}


def _stream(device):
    return torch.cuda.current_stream(device).cuda_stream


def _require_cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise NotImplementedError("qlin runs on CUDA tensors only (there is no CPU path)")


def _workspace(nbytes, device):
    if nbytes == 0:
        return None, 0
    return torch.empty(nbytes, dtype=torch.uint8, device=device), nbytes


def _flatten_x(x):
    k = x.shape[-1]
    x2 = x.reshape(-1, k)
    if x2.stride(-1) != 1:
        x2 = x2.contiguous()
    return x2


def _out(x, n, out_dtype):
    lead = x.shape[:-1]
    return torch.empty(*lead, n, dtype=out_dtype or x.dtype, device=x.device)


def device_status(reset=True):
    import ctypes
    where = ctypes.c_uint32(0)
    code = lib.qlin_device_status(1 if reset else 0, ctypes.byref(where))
    return code, where.value


# Site numbers of the bounds-checked build (enum BoundsSite in csrc/qlin_checks.cuh).
SITE_NAMES = {
    1: "gemm output", 2: "gemm bias/scale/exponent", 3: "gemm token exponent", 4: "gemm split-K partial",
    5: "gemm weight bulk copy", 6: "gemm LoRA up row", 7: "gemm staged/peer store", 8: "gemm shared memory",
    9: "TMA coordinate alignment", 10: "int8 gemm output", 11: "int8 gemm scale/bias", 12: "int8 gemm weight bulk copy",
    13: "int8 gemm shared memory", 14: "small-M weights", 15: "small-M activations", 16: "small-M output/bias/scale",
    17: "prologue input", 18: "prologue output", 19: "repack/decode source", 20: "repack/decode destination",
    21: "split-K finalize", 22: "LoRA packing", 23: "gradient kernels", 24: "kitchen grid", 25: "peer flags",
}


def bounds_check(reset=True):
    """Bounds record of the library built with QLIN_CHECKS (libqlin_checked.so, selected with the
    QLIN_LIB environment variable): None when no check failed since the last reset, else a dict
    with the number of failures and the first one's site, index, limit and block.  Raises
    QlinDecline on the ordinary build, which has no checks."""
    import ctypes
    count, site, block = ctypes.c_uint32(0), ctypes.c_uint32(0), ctypes.c_uint32(0)
    index, limit = ctypes.c_int64(0), ctypes.c_int64(0)
    rc = lib.qlin_bounds_check(1 if reset else 0, ctypes.byref(count), ctypes.byref(site), ctypes.byref(index),
                               ctypes.byref(limit), ctypes.byref(block))
    if rc != 0:
        raise QlinDecline(rc, lib.qlin_last_error().decode())
    if count.value == 0:
        return None
    return {"count": count.value, "site": SITE_NAMES.get(site.value, site.value), "index": index.value,
            "limit": limit.value, "block": block.value}


# ---------------------------------------------------------------------------------------------- INT8
def int8_linear(x, qdata, scale, bias=None, out_dtype=None, convrot=False, convrot_groupsize=256,
                lora_down=None, lora_up=None, lora_scale=None):
    """y = rot(x) . (qdata * scale)^T + bias, weight-only INT8 (qdata int8 [N, K], stored rotated when
    convrot).  `scale` is per output channel, [N] or [N, 1], fp32 or fp16; a scalar scale is broadcast.
    The unmerged LoRA arguments run beside the layer: y += lora_scale * (x . down^T) . up^T."""
    _require_cuda(x, qdata)
    if qdata.dtype != torch.int8 or qdata.dim() != 2:
        raise QlinDecline(1, "int8_linear: qdata must be a 2-D int8 tensor")
    n, k = qdata.shape
    if x.shape[-1] != k:
        raise ValueError(f"int8_linear: x has {x.shape[-1]} features, weight has {k}")
    y = _out(x, n, out_dtype)
    if x.numel() == 0 or n == 0:
        return y
    if k == 0:
        y.zero_()
        if bias is not None:
            y += bias.to(y.dtype)
        return y
    x2 = _flatten_x(x)
    m = x2.shape[0]
    sc = scale.reshape(-1)
    if sc.numel() == 1:
        sc = sc.expand(n)
    if sc.dtype not in (torch.float32, torch.float16):
        sc = sc.float()
    sc = sc.contiguous()
    q = qdata.contiguous()
    b = None if bias is None else bias.contiguous()
    if b is not None and b.dtype not in (torch.float16, torch.float32, torch.bfloat16):
        b = b.float()
    group = convrot_groupsize if convrot else 0
    y2 = y.view(m, n)
    lora = _lora_fused_args(x2, lora_down, lora_up, lora_scale) if lora_down is not None else None
    if lora is not None:
        d, u, rank, ls = lora
        ws, wsb = _workspace(lib.qlin_int8_linear_lora_down_workspace(m, n, k, rank), x.device)
        check(lib.qlin_int8_linear_lora_down(x2.data_ptr(), _DT[x2.dtype], m, k, x2.stride(0), q.data_ptr(), n,
                                             sc.data_ptr(), _DT[sc.dtype], None if b is None else b.data_ptr(),
                                             0 if b is None else _DT[b.dtype], group, d.data_ptr(), _DT[d.dtype],
                                             d.stride(0), u.data_ptr(), _DT[u.dtype], u.stride(0), rank, ls,
                                             y2.data_ptr(), _DT[y2.dtype], n, None if ws is None else ws.data_ptr(),
                                             wsb, _stream(x.device)), "qlin_int8_linear_lora_down")
        return y
    ws, wsb = _workspace(lib.qlin_int8_linear_workspace(m, n, k), x.device)
    check(lib.qlin_int8_linear(x2.data_ptr(), _DT[x2.dtype], m, k, x2.stride(0), q.data_ptr(), n, sc.data_ptr(),
                               _DT[sc.dtype], None if b is None else b.data_ptr(), 0 if b is None else _DT[b.dtype],
                               group, y2.data_ptr(), _DT[y2.dtype], n, None if ws is None else ws.data_ptr(), wsb,
                               _stream(x.device)), "qlin_int8_linear")
    if lora_down is not None:
        _lora_beside(y, x, lora_down, lora_up, lora_scale)
    return y


_STREAMS: dict = {}


def int8_linear_streamed(x, qdata, scale, bias=None, out=None, out_dtype=torch.float16, convrot=False,
                         convrot_groupsize=256, chunks=8):
    """int8_linear for activations and outputs in host memory: x is a (pinned) CPU tensor [M, K], the
    weights live on the GPU, and the result lands in `out` (a pinned CPU tensor [M, N], allocated if
    None).  Rows are processed in `chunks` pieces so the host-to-device copy of one piece, the op on
    the previous one and the device-to-host copy of the one before run at the same time (two copy
    streams besides the current stream).  Stream-ordered: the copies start after the work already on
    the current stream, and the current stream waits for the last copy back, so synchronize it (or
    record an event on it) before reading `out`."""
    if x.is_cuda or not qdata.is_cuda:
        raise NotImplementedError("int8_linear_streamed takes host activations and device weights")
    dev = qdata.device
    n, k = qdata.shape
    x2 = x.reshape(-1, k)
    m = x2.shape[0]
    if out is None:
        out = torch.empty(m, n, dtype=out_dtype, pin_memory=True)
    y2 = out.view(m, n)
    if m == 0:
        return out
    cur = torch.cuda.current_stream(dev)
    if dev not in _STREAMS:
        _STREAMS[dev] = (torch.cuda.Stream(dev), torch.cuda.Stream(dev))
    h2d, d2h = _STREAMS[dev]
    h2d.wait_stream(cur)
    d2h.wait_stream(cur)
    rows = -(-m // max(1, chunks))
    for r0 in range(0, m, rows):
        r1 = min(m, r0 + rows)
        with torch.cuda.stream(h2d):
            xb = torch.empty(r1 - r0, k, dtype=x2.dtype, device=dev)
            xb.copy_(x2[r0:r1], non_blocking=True)
        cur.wait_stream(h2d)
        xb.record_stream(cur)
        yb = int8_linear(xb, qdata, scale, bias, out_dtype=y2.dtype, convrot=convrot, convrot_groupsize=convrot_groupsize)
        d2h.wait_stream(cur)
        with torch.cuda.stream(d2h):
            y2[r0:r1].copy_(yb, non_blocking=True)
        yb.record_stream(d2h)
    cur.wait_stream(d2h)
    return out


def _lora_beside(y, x, down, up, scale):
    """Unmerged LoRA beside the layer in fp32: y += scale * (x . down^T) . up^T."""
    s = 1.0 if scale is None else float(scale)
    side = torch.nn.functional.linear(torch.nn.functional.linear(x.float(), down.float()), up.float())
    y.add_((side * s).to(y.dtype))


def _lora_fused_args(x2, down, up, scale):
    """Operands of the fused LoRA: the down factor [rank, K] and up [N, rank] as stored (float, unit
    inner stride), the rank and the scale; the library computes t = x . down^T with its own GEMM and
    runs the up-projection as extra K stages of the linear's GEMM.  None when the LoRA must run
    beside the layer (rank above 256, shapes that do not match)."""
    if up is None or down.dim() != 2 or up.dim() != 2 or down.shape[0] != up.shape[1] or down.shape[0] > 256:
        return None
    if down.shape[1] != x2.shape[1] or not down.is_cuda or not up.is_cuda:
        return None
    fl = (torch.float16, torch.bfloat16, torch.float32)
    d = down if (down.dtype in fl and down.stride(-1) == 1) else down.float().contiguous()
    u = up if (up.dtype in fl and up.stride(-1) == 1) else up.float().contiguous()
    return d, u, int(down.shape[0]), 1.0 if scale is None else float(scale)


# ---------------------------------------------------------------------------------------------- GGUF
_REPACK_CACHE: dict = {}


def _repack_key(weight, qtype, shape):
    return (weight.data_ptr(), weight.device.index, int(qtype), tuple(shape), weight._version)


def repack_gguf(weight, qtype, shape):
    """One-time repack of raw ggml blocks into the resident stage layout; cached per weight
    tensor (dropped when the tensor is freed or modified in place)."""
    import ctypes
    n, k = int(shape[0]), int(shape[1])
    key = _repack_key(weight, qtype, (n, k))
    hit = _REPACK_CACHE.get(key)
    if hit is not None:
        return hit
    nbytes = ctypes.c_size_t(0)
    npad = ctypes.c_int64(0)
    check(lib.qlin_gguf_repacked_bytes(int(qtype), n, k, ctypes.byref(nbytes), ctypes.byref(npad)),
          "qlin_gguf_repacked_bytes")
    raw = weight.contiguous()
    packed = torch.empty(nbytes.value, dtype=torch.uint8, device=weight.device)
    row_exp = torch.empty(npad.value, dtype=torch.int32, device=weight.device)
    check(lib.qlin_gguf_repack(raw.data_ptr(), int(qtype), n, k, packed.data_ptr(), nbytes.value,
                               row_exp.data_ptr(), npad.value, _stream(weight.device)), "qlin_gguf_repack")
    entry = (packed, row_exp)
    _REPACK_CACHE[key] = entry
    try:
        weakref.finalize(weight, _REPACK_CACHE.pop, key, None)
    except TypeError:
        pass
    return entry


def gguf_linear(x, weight, qtype, shape, bias=None, out_dtype=None, lora_down=None, lora_up=None, lora_scale=None):
    """y = x . dequant_gguf(weight)^T + bias for raw ggml blocks `weight` (uint8, rows of whole
    blocks) of logical `shape` (N, K); bias joins the fp32 sum before the one rounding."""
    _require_cuda(x, weight)
    qtype = int(qtype)
    if qtype not in GGUF_TYPES:
        raise QlinDecline(1, f"gguf_linear: type {qtype} is not supported")
    n, k = int(shape[0]), int(shape[1])
    if x.shape[-1] != k:
        raise ValueError(f"gguf_linear: x has {x.shape[-1]} features, weight has {k}")
    y = _out(x, n, out_dtype)
    if x.numel() == 0 or n == 0:
        return y
    x2 = _flatten_x(x)
    m = x2.shape[0]
    packed, row_exp = repack_gguf(weight, qtype, (n, k))
    b = None if bias is None else bias.contiguous()
    if b is not None and b.dtype not in (torch.float16, torch.float32, torch.bfloat16):
        b = b.float()
    y2 = y.view(m, n)
    lora = _lora_fused_args(x2, lora_down, lora_up, lora_scale) if lora_down is not None else None
    if lora is not None:
        d, u, rank, ls = lora
        ws, wsb = _workspace(lib.qlin_gguf_linear_lora_down_workspace(m, n, k, _DT[x2.dtype], x2.stride(0), rank),
                             x.device)
        check(lib.qlin_gguf_linear_lora_down(x2.data_ptr(), _DT[x2.dtype], m, k, x2.stride(0), packed.data_ptr(),
                                             row_exp.data_ptr(), qtype, n, None if b is None else b.data_ptr(),
                                             0 if b is None else _DT[b.dtype], d.data_ptr(), _DT[d.dtype], d.stride(0),
                                             u.data_ptr(), _DT[u.dtype], u.stride(0), rank, ls, y2.data_ptr(),
                                             _DT[y2.dtype], n, None if ws is None else ws.data_ptr(), wsb,
                                             _stream(x.device)), "qlin_gguf_linear_lora_down")
        return y
    ws, wsb = _workspace(lib.qlin_gguf_linear_workspace(m, n, k, _DT[x2.dtype], x2.stride(0)), x.device)
    check(lib.qlin_gguf_linear(x2.data_ptr(), _DT[x2.dtype], m, k, x2.stride(0), packed.data_ptr(),
                               row_exp.data_ptr(), qtype, n, None if b is None else b.data_ptr(),
                               0 if b is None else _DT[b.dtype], y2.data_ptr(), _DT[y2.dtype], n,
                               None if ws is None else ws.data_ptr(), wsb, _stream(x.device)), "qlin_gguf_linear")
    if lora_down is not None:
        _lora_beside(y, x, lora_down, lora_up, lora_scale)
    return y


def gguf_linear_slabs(x_slabs, packed, row_exp, qtype, n, bias=None, out=None):
    """GGUF linear on an fp16 activation stored as column slabs, x_slabs [S, M, K/S] (the layout
    an all-gather of column shards produces).  `packed`, `row_exp` come from repack_gguf.
    Returns (or fills) out [M, n] fp16."""
    s_, m, ks = x_slabs.shape
    k = s_ * ks
    if x_slabs.dtype != torch.float16 or x_slabs.stride(2) != 1:
        raise QlinDecline(1, "gguf_linear_slabs needs fp16 slabs with contiguous rows")
    y = out if out is not None else torch.empty(m, n, dtype=torch.float16, device=x_slabs.device)
    b = None if bias is None else bias.contiguous()
    ws_bytes = lib.qlin_gguf_linear_workspace(m, n, k, 1, x_slabs.stride(1))
    ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=x_slabs.device)
    check(lib.qlin_gguf_linear_slabs(x_slabs.data_ptr(), m, k, x_slabs.stride(1), s_, x_slabs.stride(0),
                                     packed.data_ptr(), row_exp.data_ptr(), int(qtype), n,
                                     None if b is None else b.data_ptr(), 0 if b is None else _DT[b.dtype],
                                     y.data_ptr(), 1, y.stride(0), ws.data_ptr(), ws_bytes,
                                     _stream(x_slabs.device)), "qlin_gguf_linear_slabs")
    return y


def gguf_linear_allgather(x_slabs, packed, row_exp, qtype, n, y_ranks, sync_ranks, rank, bias=None,
                          timeout_ms=0):
    """gguf_linear_slabs whose [M, n] fp16 output shard is stored by the GEMM's epilogue into every
    rank's gathered buffer: y_ranks[r] = device address of this rank's slab inside rank r's buffer
    (row pitch n), sync_ranks[r] = address of rank r's flag pad (see qlin.peer.PeerBuffer).  Every
    rank of the group must make the same sequence of these calls."""
    import ctypes
    s_, m, ks = x_slabs.shape
    k = s_ * ks
    if x_slabs.dtype != torch.float16 or x_slabs.stride(2) != 1:
        raise QlinDecline(1, "gguf_linear_allgather needs fp16 slabs with contiguous rows")
    world = len(y_ranks)
    if len(sync_ranks) != world:
        raise ValueError("one output slab and one flag pad per rank")
    b = None if bias is None else bias.contiguous()
    ws_bytes = lib.qlin_gguf_linear_workspace(m, n, k, 1, x_slabs.stride(1))
    ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=x_slabs.device)
    ys = (ctypes.c_void_p * world)(*y_ranks)
    syncs = (ctypes.c_void_p * world)(*sync_ranks)
    check(lib.qlin_gguf_linear_allgather(x_slabs.data_ptr(), m, k, x_slabs.stride(1), s_, x_slabs.stride(0),
                                         packed.data_ptr(), row_exp.data_ptr(), int(qtype), n,
                                         None if b is None else b.data_ptr(), 0 if b is None else _DT[b.dtype],
                                         world, rank, ys, 1, n, syncs, int(timeout_ms), ws.data_ptr(), ws_bytes,
                                         _stream(x_slabs.device)), "qlin_gguf_linear_allgather")


def peer_wait(sync_ranks, rank, timeout_ms=0, device=None):
    """Stream-ordered wait until every rank has finished as many gguf_linear_allgather calls as this
    one: afterwards this rank's gathered buffers hold every rank's output of those calls."""
    import ctypes
    world = len(sync_ranks)
    syncs = (ctypes.c_void_p * world)(*sync_ranks)
    check(lib.qlin_peer_wait(world, rank, syncs, int(timeout_ms), _stream(device or torch.cuda.current_device())),
          "qlin_peer_wait")


def dequantize_gguf(weight, qtype, shape, out_dtype=torch.float32):
    """Decode-only, bit-exact with gguf-py 0.19.0 (fp16 / bf16 outputs round that value once)."""
    _require_cuda(weight)
    n, k = int(shape[0]), int(shape[1])
    out = torch.empty(n, k, dtype=out_dtype, device=weight.device)
    raw = weight.contiguous()
    check(lib.qlin_gguf_dequantize(raw.data_ptr(), int(qtype), n, k, out.data_ptr(), _DT[out_dtype],
                                   _stream(weight.device)), "qlin_gguf_dequantize")
    return out


# ---------------------------------------------------------------------------------------------- prologues
def prologue_f16(x, rotate_group=0):
    """(fp16 [M, Kp] operand, int32 row exponents): rotation + power-of-two row scaling."""
    x2 = _flatten_x(x)
    m, k = x2.shape
    kp = (k + 63) // 64 * 64
    out = torch.empty(m, kp, dtype=torch.float16, device=x.device)
    rexp = torch.empty(m, dtype=torch.int32, device=x.device)
    check(lib.qlin_prologue_f16(x2.data_ptr(), _DT[x2.dtype], m, k, x2.stride(0), rotate_group, out.data_ptr(), kp,
                                rexp.data_ptr(), _stream(x.device)), "qlin_prologue_f16")
    return out, rexp


def quantize_int8_rowwise(x, rotate_group=0, perm=False):
    """Per-token INT8 quantization with the reference's rounding; returns (q int8 [M, K], scale fp32 [M, 1])."""
    x2 = _flatten_x(x)
    m, k = x2.shape
    kp = (k + 127) // 128 * 128 if perm else k
    q = torch.empty(m, kp, dtype=torch.int8, device=x.device)
    s = torch.empty(m, 1, dtype=torch.float32, device=x.device)
    check(lib.qlin_quantize_rows_int8(x2.data_ptr(), _DT[x2.dtype], m, k, x2.stride(0), rotate_group, 1 if perm else 0,
                                      q.data_ptr(), kp, s.data_ptr(), _stream(x.device)), "qlin_quantize_rows_int8")
    return (q if kp == k else q[:, :k]), s


# ---------------------------------------------------------------------------------------------- W4A8 / W6A8
def w4a8_linear(*args, **kwargs):
    """Benchmark-configuration W4A8 / W6A8 (per-token int8 activations, kind::i8); see _w4a8."""
    from ._w4a8 import w4a8_linear as impl
    return impl(*args, **kwargs)


def w4a8_int8_linear(*args, **kwargs):
    """Kitchen AsymW4A8Int8Layout linear (weight-only, like the reference backend); see _w4a8."""
    from ._w4a8 import w4a8_int8_linear as impl
    return impl(*args, **kwargs)


def dequantize_w4a8_int8_weight(*args, **kwargs):
    """Kitchen W4A8 / W6A8 decode-only entry point; see _w4a8."""
    from ._w4a8 import dequantize_w4a8_int8_weight as impl
    return impl(*args, **kwargs)


# ---------------------------------------------------------------------------------------------- gradients
from ._grad import (int8_linear_grad_input, int8_linear_trainable, w4a8_linear_grad_input,  # noqa: E402
                    w4a8_linear_trainable)
