"""ComfyUI-GGUF fast-path hook: `linear(layer, x) -> Tensor | None`.

Mirrors the reference fork's `mps.linear` contract (roblennon/mac-kernels-public
`bench/gguf_node.py:50-92`, `docs/research/2026-10-03-gguf-on-metal.md:114-122`,
`tests/test_gguf_node.py`): `GGMLOps.Linear.forward_ggml_cast_weights` calls `linear(layer, x)`
first and takes its stock dequantize-per-call path when this returns None.

It returns None (stock path) for: weights that are not GGML-quantized with a supported type
(F16 / F32 tensors), an explicit `dequant_dtype` on the layer, a `patch_dtype` on a layer that has
patches, any patch that is not a plain LoRA (DoRA, other adapters), and inputs that are not on a
CUDA device.  Plain LoRAs stay unmerged: call-local fp32 factors are built from the patches on
every call (`_lora_for_call`; nothing is cached, so factors follow patch changes and never outlive
the call).  Whole-layer LoRAs are stacked along the rank; for bf16 activations and a stacked rank of
at most FUSED_MAX_RANK they run inside the GEMM as extra K stages (the fork's fused case), otherwise
beside it in fp32.  Row-slice LoRAs are applied to their output slice beside a base output produced
in fp32.  Either way the LoRA terms join the sum before the single rounding to the input dtype.

`FUSED_MAX_RANK` and `_kernel()` are the module contract the fork's callers read: the ComfyUI glue
classifies a call as fused when `rank > 0 and x.dtype == torch.bfloat16 and rank <= FUSED_MAX_RANK`
(`bench/gguf_node.py:55-70`), and tests wrap `_kernel().gguf_linear` to count kernel calls
(`tests/test_gguf_node.py:80-92`).  `linear` looks `gguf_linear` up on `_kernel()` at every call, so
such a wrapper sees every call, with `lora_down` among the keyword arguments exactly when fused.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import torch

import qlin

# Largest stacked LoRA rank that runs inside the GEMM (for bf16 activations), as in the fork.
FUSED_MAX_RANK = 128


def _kernel():
    """The kernel module whose `gguf_linear` this hook calls (the fork's comfy_kitchen handle), or
    None when no CUDA device is present."""
    return qlin if torch.cuda.is_available() else None


@dataclass
class LoraFactors:
    stacked: tuple | None = None            # (down [R, K], up [N, R]) fp32, scales folded into down
    sliced: list = field(default_factory=list)  # [(down [R, K], up [S, R], start)] for row slices


def _adapter_lora(adapter):
    """(up, down, alpha) for a plain LoRA adapter, else None.  Accepts ComfyUI's LoRAAdapter (weights
    = (up, down, alpha, mid, dora_scale, reshape)) or a bare tuple in that order."""
    weights = getattr(adapter, "weights", adapter)
    if not isinstance(weights, (tuple, list)) or len(weights) < 2:
        return None
    up, down = weights[0], weights[1]
    alpha = weights[2] if len(weights) > 2 else None
    mid = weights[3] if len(weights) > 3 else None
    dora = weights[4] if len(weights) > 4 else None
    reshape = weights[5] if len(weights) > 5 else None
    if mid is not None or dora is not None or reshape is not None:
        return None
    if not (isinstance(up, torch.Tensor) and isinstance(down, torch.Tensor)) or up.dim() != 2 or down.dim() != 2:
        return None
    return up, down, alpha


def _lora_for_call(weight, x):
    """Call-local fp32 LoRA factors for the weight's patches, or None when a patch is not a plain
    LoRA (the caller then takes the stock path).  Returns an empty LoraFactors without patches."""
    factors = LoraFactors()
    downs, ups = [], []
    n, k = int(weight.tensor_shape[0]), int(weight.tensor_shape[1])
    for entry in getattr(weight, "patches", None) or []:
        patch_list = entry[0] if isinstance(entry, tuple) and len(entry) == 2 and isinstance(entry[0], list) else [entry]
        for patch in patch_list:
            strength, adapter = float(patch[0]), patch[1]
            offset = patch[3] if len(patch) > 3 else None
            function = patch[4] if len(patch) > 4 else None
            if function is not None:
                return None
            lora = _adapter_lora(adapter)
            if lora is None:
                return None
            up, down, alpha = lora
            rank = down.shape[0]
            scale = strength * ((float(alpha) / rank) if alpha is not None else 1.0)
            d = down.to(x.device, torch.float32) * scale
            u = up.to(x.device, torch.float32)
            if offset is None:
                if u.shape[0] != n or d.shape[1] != k:
                    return None
                downs.append(d)
                ups.append(u)
            else:
                dim, start, size = offset
                if dim != 0 or d.shape[1] != k or u.shape[0] != size:
                    return None
                factors.sliced.append((d, u, int(start)))
    if downs:
        factors.stacked = (torch.cat(downs, 0), torch.cat(ups, 1))
    return factors


def linear(layer, x):
    """Fast GGUF linear for a ComfyUI-GGUF GGMLOps.Linear, or None for the stock path."""
    w = layer.weight
    qtype = getattr(w, "tensor_type", None)
    if qtype is None or int(qtype) not in qlin.GGUF_TYPES:
        return None
    if getattr(layer, "dequant_dtype", None) is not None:
        return None
    patches = getattr(w, "patches", None) or []
    if patches and getattr(layer, "patch_dtype", None) is not None:
        return None
    if not x.is_cuda or x.dtype not in (torch.float16, torch.bfloat16, torch.float32):
        return None
    ck = _kernel()
    if ck is None:
        return None
    factors = _lora_for_call(w, x)
    if factors is None:
        return None
    raw = w.as_subclass(torch.Tensor) if type(w) is not torch.Tensor else w
    bias = getattr(layer, "bias", None)
    if bias is not None:
        bias = bias.as_subclass(torch.Tensor) if type(bias) is not torch.Tensor else bias
        bias = bias.to(x.device)
    shape = (int(w.tensor_shape[0]), int(w.tensor_shape[1]))
    rank = 0 if factors.stacked is None else int(factors.stacked[0].shape[0])
    fused = rank > 0 and x.dtype == torch.bfloat16 and rank <= FUSED_MAX_RANK
    beside = (rank > 0 and not fused) or bool(factors.sliced)
    kwargs = dict(bias=bias, out_dtype=torch.float32 if beside else x.dtype)
    if fused:
        # whole-layer LoRAs inside the GEMM (extra K stages), added before the output's rounding
        down, up = factors.stacked
        kwargs.update(lora_down=down, lora_up=up, lora_scale=1.0)
    try:
        y = ck.gguf_linear(x, raw, int(qtype), shape, **kwargs)
    except NotImplementedError:
        return None
    if not beside:
        return y
    xf = x.float()
    if rank > 0 and not fused:
        down, up = factors.stacked
        y += torch.nn.functional.linear(torch.nn.functional.linear(xf, down), up)
    for down, up, start in factors.sliced:
        y[..., start:start + up.shape[0]] += torch.nn.functional.linear(torch.nn.functional.linear(xf, down), up)
    return y.to(x.dtype)
