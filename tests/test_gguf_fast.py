"""ComfyUI-GGUF fork hook (`qlin.gguf_fast.linear`): decline rules on the CPU, and on the GPU the
fast path against the stock path (dequantize + F.linear, with LoRA patches merged in fp32), like
the reference's tests/test_gguf_node.py (8e-3 bf16 / 3e-3 fp16 relative L2)."""
import types

import numpy as np
import pytest
import torch

from oracle import qlin_oracle as O


class FakeGGML(torch.Tensor):
    """Stand-in for ComfyUI-GGUF's GGMLTensor: uint8 blocks with tensor_type / tensor_shape."""

    @staticmethod
    def make(raw, qtype, shape):
        t = raw.as_subclass(FakeGGML)
        t.tensor_type = qtype
        t.tensor_shape = torch.Size(shape)
        t.patches = []
        return t


def make_layer(qtype=12, n=192, k=512, device="cpu", bias=True, seed=0):
    raw = torch.from_numpy(O.random_gguf_blocks(qtype, n, k, seed=seed)).to(device)
    layer = types.SimpleNamespace(weight=FakeGGML.make(raw, qtype, (n, k)), bias=None, dequant_dtype=None,
                                  patch_dtype=None)
    if bias:
        layer.bias = (torch.randn(n, generator=torch.Generator().manual_seed(seed)) * 0.1).to(device)
    return layer


def lora_patch(up, down, alpha=None, strength=1.0, offset=None, dora=None):
    adapter = types.SimpleNamespace(weights=(up, down, alpha, None, dora, None))
    return (strength, adapter, 1.0, offset, None)


def stock(layer, x):
    """Dequantize in fp32, merge plain LoRAs in fp32, F.linear in fp32."""
    w = torch.from_numpy(O.gguf_dequantize(layer.weight.as_subclass(torch.Tensor).cpu().numpy(), layer.weight.tensor_type,
                                           *layer.weight.tensor_shape)).clone()
    for entry in layer.weight.patches:
        for strength, adapter, _, offset, _ in entry[0]:
            up, down, alpha = adapter.weights[:3]
            scale = strength * ((alpha / down.shape[0]) if alpha is not None else 1.0)
            delta = scale * (up.float() @ down.float())
            if offset is None:
                w += delta
            else:
                w[offset[1]:offset[1] + offset[2]] += delta
    b = None if layer.bias is None else layer.bias.float().cpu()
    return torch.nn.functional.linear(x.float().cpu(), w, b)


def test_declines_on_cpu_inputs_and_unsupported_settings():
    from qlin import gguf_fast
    layer = make_layer()
    assert gguf_fast.linear(layer, torch.randn(2, 512)) is None  # not on a CUDA device
    f16 = types.SimpleNamespace(weight=FakeGGML.make(torch.zeros(4, 8, dtype=torch.uint8), 1, (4, 8)), bias=None)
    assert gguf_fast.linear(f16, torch.randn(2, 8)) is None  # F16 tensor type: stock path


def test_lora_factors_follow_patch_kinds():
    from qlin import gguf_fast
    layer = make_layer()
    x = torch.randn(3, 512)
    g = torch.Generator().manual_seed(1)
    up, down = torch.randn(192, 8, generator=g), torch.randn(8, 512, generator=g)
    layer.weight.patches = [([lora_patch(up, down, alpha=4.0, strength=0.5)], "k")]
    f = gguf_fast._lora_for_call(layer.weight, x)
    assert f.stacked[0].dtype == torch.float32 and f.stacked[0].shape == (8, 512)
    assert torch.allclose(f.stacked[0], down * 0.25)
    layer.weight.patches = [([lora_patch(up, down, dora=torch.ones(192))], "k")]
    assert gguf_fast._lora_for_call(layer.weight, x) is None  # DoRA takes the stock path
    layer.weight.patches = [([lora_patch(up[:64], down, offset=(0, 64, 64))], "k")]
    f = gguf_fast._lora_for_call(layer.weight, x)
    assert f.stacked is None and f.sliced[0][2] == 64


@pytest.mark.gpu
@pytest.mark.parametrize("qtype", sorted(O.GGUF_TYPES))
@pytest.mark.parametrize("dtype,tol", [(torch.bfloat16, 8e-3), (torch.float16, 3e-3)])
def test_fast_path_matches_stock(qtype, dtype, tol):
    from qlin import gguf_fast
    layer = make_layer(qtype, device="cuda")
    x = torch.randn(2, 40, 512, device="cuda", dtype=dtype)
    got = gguf_fast.linear(layer, x)
    assert got is not None and got.dtype == dtype and got.shape == (2, 40, 192)
    ref = stock(layer, x)
    assert ((got.float().cpu() - ref).norm() / ref.norm()).item() < tol


@pytest.mark.gpu
def test_whole_layer_and_slice_loras_stay_unmerged():
    from qlin import gguf_fast
    layer = make_layer(12, device="cuda")
    g = torch.Generator().manual_seed(1)
    p1 = lora_patch(torch.randn(192, 16, generator=g) * 0.05, torch.randn(16, 512, generator=g) * 0.05, alpha=8.0)
    p2 = lora_patch(torch.randn(192, 4, generator=g) * 0.05, torch.randn(4, 512, generator=g) * 0.05, strength=0.5)
    p3 = lora_patch(torch.randn(64, 4, generator=g) * 0.05, torch.randn(4, 512, generator=g) * 0.05,
                    offset=(0, 64, 64))
    layer.weight.patches = [([p1, p2, p3], "diffusion_model.x.weight")]
    raw_before = layer.weight.as_subclass(torch.Tensor).clone()
    x = torch.randn(64, 512, device="cuda", dtype=torch.bfloat16)
    got = gguf_fast.linear(layer, x)
    ref = stock(layer, x)
    assert ((got.float().cpu() - ref).norm() / ref.norm()).item() < 8e-3
    assert torch.equal(layer.weight.as_subclass(torch.Tensor), raw_before)  # nothing merged


@pytest.mark.gpu
def test_declines_explicit_precision_settings_on_gpu():
    from qlin import gguf_fast
    layer = make_layer(8, device="cuda")
    x = torch.randn(4, 512, device="cuda", dtype=torch.float16)
    layer.dequant_dtype = torch.float32
    assert gguf_fast.linear(layer, x) is None
    layer.dequant_dtype = None
    layer.patch_dtype = torch.float32
    assert gguf_fast.linear(layer, x) is not None  # patch_dtype without patches: fast path
    layer.weight.patches = [([lora_patch(torch.zeros(192, 2), torch.zeros(2, 512))], "k")]
    assert gguf_fast.linear(layer, x) is None


# ---------------------------------------------------------------------------------------------
# The fork's module contract, exercised the way the reference's ComfyUI glue and node tests do:
# a Spy wrapping `_kernel().gguf_linear` (tests/test_gguf_node.py:80-92) and the route audit that
# classifies fused / beside LoRA calls with FUSED_MAX_RANK (bench/gguf_node.py:50-70).
# ---------------------------------------------------------------------------------------------
class Spy:
    def __init__(self, fast, monkeypatch):
        self.calls = []
        ck = fast._kernel()
        assert ck is not None, "a kernel module with gguf_linear on CUDA is required"
        real = ck.gguf_linear

        def spy(*a, **kw):
            self.calls.append(kw)
            return real(*a, **kw)

        monkeypatch.setattr(ck, "gguf_linear", spy)


def install_audit(fast, monkeypatch):
    record = dict(kernel=False, kernel_fused=0, kernel_beside=0, kernel_slices=0)
    real_prepare, real_linear = fast._lora_for_call, fast.linear

    def prepare(weight, x):
        factors = real_prepare(weight, x)
        if factors is not None:
            rank = 0 if factors.stacked is None else factors.stacked[0].shape[0]
            fused = rank > 0 and x.dtype == torch.bfloat16 and rank <= fast.FUSED_MAX_RANK
            record.update(kernel_fused=int(fused), kernel_beside=int(rank > 0 and not fused),
                          kernel_slices=len(factors.sliced))
        return factors

    def linear(layer, x):
        result = real_linear(layer, x)
        record["kernel"] = result is not None
        return result

    monkeypatch.setattr(fast, "_lora_for_call", prepare)
    monkeypatch.setattr(fast, "linear", linear)
    return record


def test_module_contract_names():
    from qlin import gguf_fast
    assert gguf_fast.FUSED_MAX_RANK == 128
    assert callable(gguf_fast._kernel)
    ck = gguf_fast._kernel()
    assert ck is None or callable(ck.gguf_linear)


@pytest.mark.gpu
@pytest.mark.parametrize("qtype", [12, 14, 8, 6, 11])
@pytest.mark.parametrize("dtype,tol", [(torch.bfloat16, 8e-3), (torch.float16, 3e-3)])
def test_spy_sees_one_kernel_call_without_lora(qtype, dtype, tol, monkeypatch):
    from qlin import gguf_fast
    layer = make_layer(qtype, device="cuda")
    x = torch.randn(2, 40, 512, device="cuda", dtype=dtype)
    spy = Spy(gguf_fast, monkeypatch)
    got = gguf_fast.linear(layer, x)
    assert len(spy.calls) == 1 and "lora_down" not in spy.calls[0]
    assert got.dtype == dtype and got.shape == (2, 40, 192)
    ref = stock(layer, x)
    assert ((got.float().cpu() - ref).norm() / ref.norm()).item() < tol


@pytest.mark.gpu
@pytest.mark.parametrize("dtype,rank,fused", [(torch.bfloat16, 16, True), (torch.float16, 16, False),
                                              (torch.bfloat16, 200, False)])
@pytest.mark.parametrize("sliced", [False, True])
def test_fused_classification_matches_the_kernel_call(dtype, rank, fused, sliced, monkeypatch):
    from qlin import gguf_fast
    layer = make_layer(12, device="cuda")
    g = torch.Generator().manual_seed(1)
    patches = [lora_patch(torch.randn(192, rank, generator=g) * 0.05, torch.randn(rank, 512, generator=g) * 0.05,
                          alpha=rank / 2),
               lora_patch(torch.randn(192, 4, generator=g) * 0.05, torch.randn(4, 512, generator=g) * 0.05, strength=0.5)]
    if sliced:
        patches.append(lora_patch(torch.randn(64, 4, generator=g) * 0.05, torch.randn(4, 512, generator=g) * 0.05,
                                  offset=(0, 64, 64)))
    layer.weight.patches = [(patches, "diffusion_model.x.weight")]
    x = torch.randn(64, 512, device="cuda", dtype=dtype)
    audit = install_audit(gguf_fast, monkeypatch)
    spy = Spy(gguf_fast, monkeypatch)
    got = gguf_fast.linear(layer, x)
    assert audit["kernel"] and audit["kernel_slices"] == int(sliced)
    assert audit["kernel_fused"] == int(fused) and audit["kernel_beside"] == int(not fused)
    assert len(spy.calls) == 1 and ("lora_down" in spy.calls[0]) == fused
    ref = stock(layer, x)
    layer.weight.patches = []
    base = stock(layer, x)
    assert ((ref - base).norm() / base.norm()).item() > 0.05  # the LoRA is visible
    tol = 8e-3 if dtype == torch.bfloat16 else 3e-3
    assert got.dtype == dtype and ((got.float().cpu() - ref).norm() / ref.norm()).item() < tol


@pytest.mark.gpu
def test_dora_never_reaches_the_kernel(monkeypatch):
    from qlin import gguf_fast
    layer = make_layer(8, device="cuda")
    g = torch.Generator().manual_seed(3)
    layer.weight.patches = [([lora_patch(torch.randn(192, 8, generator=g) * 0.05, torch.randn(8, 512, generator=g) * 0.05,
                                         dora=torch.ones(192, 1))], "k")]
    spy = Spy(gguf_fast, monkeypatch)
    assert gguf_fast.linear(layer, torch.randn(16, 512, device="cuda", dtype=torch.bfloat16)) is None
    assert spy.calls == []
