"""CPU checks of the drop-in boundary: libqlin.so loads without a GPU and exports every entry
point include/qlin.h declares; host-side argument checks answer without launching anything."""
import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    src = open(os.path.join(ROOT, "include", "qlin.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(qlin_[a-z0-9_]+)\s*\(", src)))


def test_library_exports_every_declared_symbol():
    from qlin import _lib
    names = declared_symbols()
    assert len(names) >= 10
    missing = [n for n in names if not hasattr(_lib.lib, n)]
    assert not missing, missing
    assert set(names) <= set(_lib.SIGNATURES), set(names) - set(_lib.SIGNATURES)


def test_version_and_host_side_declines_without_gpu():
    from qlin import _lib
    lib = _lib.lib
    assert lib.qlin_version().startswith(b"qlin")
    size = ctypes.c_size_t(0)
    npad = ctypes.c_int64(0)
    # unsupported GGUF type and a K that is not whole blocks decline on the host
    for unsupported in (9, 15, 16, 21):  # Q8_1, Q8_K, IQ2_XXS, IQ3_S
        assert lib.qlin_gguf_repacked_bytes(unsupported, 10, 256, ctypes.byref(size), ctypes.byref(npad)) == 1
    assert lib.qlin_gguf_repacked_bytes(12, 10, 300, ctypes.byref(size), ctypes.byref(npad)) == 1
    # rows that straddle blocks (the flattened tensor is whole blocks): plain fp16 rows, pitch 64-aligned
    assert lib.qlin_gguf_repacked_bytes(12, 64, 1152, ctypes.byref(size), ctypes.byref(npad)) == 0
    assert npad.value == 128 and size.value == 128 * 1152 * 2
    assert lib.qlin_gguf_repacked_bytes(12, 130, 512, ctypes.byref(size), ctypes.byref(npad)) == 0
    assert npad.value == 256 and size.value == 2 * 8 * 128 * 40
    # every supported type: bytes per 64-value stage of a 128-row tile (16 B planes + side record)
    stage = {2: 36, 3: 40, 6: 44, 7: 48, 8: 68, 10: 24, 11: 32, 12: 40, 13: 48, 14: 72, 20: 36, 23: 36}
    for qtype, per_row in stage.items():
        qk = 256 if qtype in (10, 11, 12, 13, 14, 23) else 32
        assert lib.qlin_gguf_repacked_bytes(qtype, 10, 4 * qk, ctypes.byref(size), ctypes.byref(npad)) == 0
        assert size.value == (4 * qk // 64) * 128 * per_row, qtype
    assert lib.qlin_gguf_repacked_bytes(3, 10, 96, ctypes.byref(size), ctypes.byref(npad)) == 0  # 3 blocks
    assert size.value == 2 * 128 * 40
    assert b"block" in lib.qlin_last_error() or lib.qlin_last_error() == b""
    # workspace queries are pure host arithmetic
    assert lib.qlin_int8_linear_workspace(4096, 12288, 3072) >= 4096 * 3072 * 2
    # input gradient: transposed weight [k, roundup(n, 64)]; empty problems need no workspace
    assert lib.qlin_int8_grad_weight_bytes(130, 256) == 256 * 192
    assert lib.qlin_int8_grad_weight_bytes(0, 256) == 0
    assert lib.qlin_int8_linear_grad_input_workspace(5, 0, 256, 128) == 0
    assert lib.qlin_int8_linear_grad_input_workspace(0, 64, 256, 0) == 0
    assert lib.qlin_int8_linear_grad_input_workspace(64, 100, 256, 128) >= 64 * 128 * 2 + 64 * 256 * 4


def test_kitchen_signatures_match_reference_surface():
    import inspect
    import qlin
    assert list(inspect.signature(qlin.int8_linear).parameters) == [
        "x", "qdata", "scale", "bias", "out_dtype", "convrot", "convrot_groupsize", "lora_down", "lora_up",
        "lora_scale"]
    assert list(inspect.signature(qlin.gguf_linear).parameters) == [
        "x", "weight", "qtype", "shape", "bias", "out_dtype", "lora_down", "lora_up", "lora_scale"]
    assert list(inspect.signature(qlin.dequantize_gguf).parameters) == ["weight", "qtype", "shape", "out_dtype"]


def test_cpu_tensors_are_refused_loudly():
    import torch
    import qlin
    with pytest.raises(NotImplementedError):
        qlin.int8_linear(torch.zeros(2, 16), torch.zeros(4, 16, dtype=torch.int8), torch.ones(4))


def test_bounds_check_entry_point_in_both_builds():
    """The ordinary library declines qlin_bounds_check (it has no checks) without touching a
    device; the bounds-checked build (built by build() next to it) loads and exports the same
    entry points."""
    from qlin import _lib
    count, site, block = ctypes.c_uint32(7), ctypes.c_uint32(0), ctypes.c_uint32(0)
    index, limit = ctypes.c_int64(0), ctypes.c_int64(0)
    rc = _lib.lib.qlin_bounds_check(1, ctypes.byref(count), ctypes.byref(site), ctypes.byref(index),
                                    ctypes.byref(limit), ctypes.byref(block))
    assert rc == 1 and b"QLIN_CHECKS" in _lib.lib.qlin_last_error()
    checked = os.path.join(ROOT, "mac-kernels-public_b200", "qlin", "libqlin_checked.so")
    if not os.path.exists(checked):
        pytest.skip("the bounds-checked build is made by __graft_entry__.build()")
    lib = ctypes.CDLL(checked)
    missing = [n for n in declared_symbols() if not hasattr(lib, n)]
    assert not missing, missing
