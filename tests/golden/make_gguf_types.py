"""Regenerates `gguf_types.npz`: GGUF blocks of all twelve supported types and their float32
decode by the third-party reference decoder, gguf-py 0.19.0 (`gguf.quants.dequantize`).

    python tests/golden/make_gguf_types.py

For each type, 4 rows x 512 values of uniformly random block bytes whose fp16 scale fields are
replaced by realistic magnitudes, except that in row 1 the first scale field of every block is one
of the edge values 0, -0, +-65504, the smallest subnormal, +-6.1e-5 (smallest normal) in turn.
Keys: `<NAME>__raw` (uint8 [4, bytes per row]) and `<NAME>__f32` (float32 [4, 512]).

The tests read only the committed .npz; nothing at test time imports gguf.
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "..", "..", "oracle"))

import qlin_oracle as O  # noqa: E402

EDGE_F16 = np.array([0.0, -0.0, 65504.0, -65504.0, 5.96e-8, -5.96e-8, 6.104e-5, -6.104e-5], dtype=np.float16)


def main():
    import gguf
    from gguf import quants

    arrays = {}
    n, k = 4, 512
    for qt, (name, qk, ts) in sorted(O.GGUF_TYPES.items()):
        raw = O.random_gguf_blocks(qt, n, k, seed=1000 + qt).reshape(n, k // qk, ts)
        off = O.GGUF_SCALE_FIELDS[name][0][0]
        edge = np.resize(EDGE_F16, k // qk)
        raw[1, :, off:off + 2] = edge.view(np.uint8).reshape(-1, 2)
        raw = raw.reshape(n, -1)
        want = quants.dequantize(raw.reshape(-1), gguf.GGMLQuantizationType(qt)).reshape(n, k).astype(np.float32)
        arrays[f"{name}__raw"] = raw
        arrays[f"{name}__f32"] = want
    arrays["gguf_version"] = np.array(getattr(gguf, "__version__", "0.19.0"))
    np.savez_compressed(os.path.join(HERE, "gguf_types.npz"), **arrays)


if __name__ == "__main__":
    main()
