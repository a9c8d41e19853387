"""Regenerates `tiny.gguf` and `tiny_int8.safetensors`, written by the third-party reference
writers (gguf-py 0.19.0 `GGUFWriter`, safetensors 0.7.0 `save_file`), which pin the checkpoint
readers of qlin.checkpoint:

    python tests/golden/make_checkpoint_files.py

tiny.gguf: Q8_0 [64, 256], Q4_K [32, 512], IQ4_NL [16, 128] raw blocks (oracle seeds 1, 2, 3), an
F16 matrix [16, 64] and an F32 vector [256] (not linears), and metadata of every value kind.
tiny_int8.safetensors: blocks.0.attn.wq.weight int8 [48, 128] + .weight_scale f32 [48], an
unpaired int8 matrix, an F16 tensor.  The tests read only the committed files.
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "..", ".."))

from oracle import qlin_oracle as O  # noqa: E402

GGUF_TENSORS = [("blk.0.attn_qkv.weight", 8, 64, 256, 1), ("blk.0.ffn_down.weight", 12, 32, 512, 2),
                ("blk.1.attn_out.weight", 20, 16, 128, 3)]


def int8_tensors():
    rng = np.random.default_rng(4)
    return {"blocks.0.attn.wq.weight": rng.integers(-127, 128, (48, 128)).astype(np.int8),
            "blocks.0.attn.wq.weight_scale": (np.abs(rng.normal(0, 0.02, 48)) / 127).astype(np.float32),
            "blocks.0.unpaired.weight": rng.integers(-127, 128, (8, 32)).astype(np.int8),
            "blocks.0.norm.bias": rng.normal(size=(4, 4)).astype(np.float16)}


def main():
    import gguf
    from safetensors.numpy import save_file

    w = gguf.GGUFWriter(os.path.join(HERE, "tiny.gguf"), "qlin-test")
    w.add_string("general.name", "tiny")
    w.add_uint32("qlin.test.u32", 7)
    w.add_int64("qlin.test.i64", -3)
    w.add_float32("qlin.test.f32", 0.5)
    w.add_bool("qlin.test.bool", True)
    w.add_array("qlin.test.array", [1, 2, 3])
    for name, qt, n, k, seed in GGUF_TENSORS:
        raw = O.random_gguf_blocks(qt, n, k, seed=seed)
        w.add_tensor(name, raw, raw_dtype=gguf.GGMLQuantizationType(qt))
    w.add_tensor("blk.0.proj.weight", np.arange(16 * 64, dtype=np.float16).reshape(16, 64))
    w.add_tensor("blk.0.norm.weight", np.linspace(-1, 1, 256, dtype=np.float32))
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    save_file(int8_tensors(), os.path.join(HERE, "tiny_int8.safetensors"), metadata={"format": "pt"})


if __name__ == "__main__":
    main()
