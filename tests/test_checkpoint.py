"""Checkpoint readers (qlin.checkpoint) against files written by the third-party reference writers
(gguf-py 0.19.0 GGUFWriter, safetensors 0.7.0; tests/golden/make_checkpoint_files.py): header
fields, tensor placement and bytes on the CPU; the loaded linears against float64 on the GPU."""
import importlib.util
import os

import numpy as np
import pytest
import torch

from oracle import qlin_oracle as O

GOLD = os.path.join(os.path.dirname(__file__), "golden")
GGUF_PATH = os.path.join(GOLD, "tiny.gguf")
ST_PATH = os.path.join(GOLD, "tiny_int8.safetensors")


def _maker():
    spec = importlib.util.spec_from_file_location("make_checkpoint_files", os.path.join(GOLD, "make_checkpoint_files.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_gguf_header_and_tensor_bytes():
    from qlin.checkpoint import GGUFFile
    mk = _maker()
    with GGUFFile(GGUF_PATH) as f:
        assert f.version == 3
        assert f.kv["general.architecture"] == "qlin-test" and f.kv["general.name"] == "tiny"
        assert f.kv["qlin.test.u32"] == 7 and f.kv["qlin.test.i64"] == -3
        assert f.kv["qlin.test.f32"] == 0.5 and f.kv["qlin.test.bool"] is True
        assert f.kv["qlin.test.array"] == [1, 2, 3]
        for name, qt, n, k, seed in mk.GGUF_TENSORS:
            t = f.tensors[name]
            assert (t.shape, t.qtype) == ((n, k), qt)
            assert t.offset % 32 == 0
            want = O.random_gguf_blocks(qt, n, k, seed=seed)
            assert np.array_equal(f.raw(name).numpy().reshape(n, -1), want), name
        assert f.tensors["blk.0.proj.weight"].shape == (16, 64)
        assert np.array_equal(f.raw("blk.0.proj.weight").numpy().view(np.float16).reshape(16, 64),
                              np.arange(16 * 64, dtype=np.float16).reshape(16, 64))
        assert np.array_equal(f.raw("blk.0.norm.weight").numpy().view(np.float32),
                              np.linspace(-1, 1, 256, dtype=np.float32))
        assert f.orig_shape("blk.0.attn_qkv.weight") is None


def test_safetensors_header_and_tensors():
    from qlin.checkpoint import SafetensorsFile, load_int8_linears
    want = _maker().int8_tensors()
    with SafetensorsFile(ST_PATH) as f:
        assert f.metadata == {"format": "pt"}
        assert set(f.tensors) == set(want)
        for name, arr in want.items():
            assert np.array_equal(f.tensor(name).numpy(), arr), name
    lin = load_int8_linears(ST_PATH, "cpu")  # loading alone launches nothing
    assert set(lin) == {"blocks.0.attn.wq"}  # the unpaired int8 matrix has no scale
    assert np.array_equal(lin["blocks.0.attn.wq"].qdata.numpy(), want["blocks.0.attn.wq.weight"])


def test_readers_refuse_malformed_files(tmp_path):
    from qlin.checkpoint import GGUFFile, SafetensorsFile
    bad = tmp_path / "bad.gguf"
    bad.write_bytes(b"GGML" + bytes(60))
    with pytest.raises(ValueError):
        GGUFFile(bad)
    cut = tmp_path / "cut.gguf"
    cut.write_bytes(open(GGUF_PATH, "rb").read()[:200])  # header cut inside the key-value pairs
    with pytest.raises(ValueError):
        GGUFFile(cut)
    short = tmp_path / "short.gguf"
    short.write_bytes(open(GGUF_PATH, "rb").read()[:20000])  # tensor data cut
    with pytest.raises(ValueError):
        GGUFFile(short)
    st = tmp_path / "bad.safetensors"
    st.write_bytes((1000).to_bytes(8, "little") + b"{}")
    with pytest.raises(ValueError):
        SafetensorsFile(st)


@pytest.mark.gpu
def test_loaded_linears_match_fp64():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    from qlin.checkpoint import load_gguf_linears, load_int8_linears
    mk = _maker()
    lin = load_gguf_linears(GGUF_PATH, "cuda")
    assert set(lin) == {t[0] for t in mk.GGUF_TENSORS}  # the F16 matrix and the F32 vector stay out
    g = torch.Generator().manual_seed(0)
    for name, qt, n, k, seed in mk.GGUF_TENSORS:
        x = torch.randn(40, k, generator=g).to(torch.float16)
        ref = O.linear_f64(x.float().numpy(), O.gguf_dequantize(O.random_gguf_blocks(qt, n, k, seed=seed), qt, n, k))
        y = lin[name](x.cuda())
        assert O.max_abs_rel(y.float().cpu().numpy(), ref) <= 2e-3, name
    w = mk.int8_tensors()
    il = load_int8_linears(ST_PATH, "cuda")["blocks.0.attn.wq"]
    x = torch.randn(40, 128, generator=g).to(torch.float16)
    ref = O.int8_convrot_linear_ref(x.float().numpy(), w["blocks.0.attn.wq.weight"],
                                    w["blocks.0.attn.wq.weight_scale"], None, group=128)
    y = il(x.cuda(), convrot=True, convrot_groupsize=128)
    assert O.max_abs_rel(y.float().cpu().numpy(), ref) <= 2e-3
