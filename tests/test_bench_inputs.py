"""The bench's input module packs the benchmark weight layouts byte for byte as the oracle does,
and its GGUF blocks decode to finite weights of the intended magnitude (CPU)."""
import numpy as np
import torch

import bench_inputs as BI
from oracle import qlin_oracle as O


def test_packings_equal_the_oracle():
    g = torch.Generator().manual_seed(0)
    q4 = torch.randint(-8, 8, (6, 128), generator=g, dtype=torch.int32)
    assert np.array_equal(BI.pack_w4(q4).numpy(), O.pack_w4_uniform(q4.numpy()).view(np.uint8))
    q6 = torch.randint(-32, 32, (6, 128), generator=g, dtype=torch.int32)
    assert np.array_equal(BI.pack_w6(q6).numpy(), O.pack_w6_interleaved(q6.numpy()))
    for bits in (4, 6):
        codes = torch.randint(0, 1 << bits, (5, 64), generator=g, dtype=torch.int32)
        assert np.array_equal(BI.pack_kitchen(codes, bits).numpy().view(np.uint8),
                              O.pack_codes_kitchen(codes.numpy(), bits).view(np.uint8))


def test_gguf_blocks_decode_to_sane_weights():
    for qtype in BI.GGUF_TYPES:
        assert BI.GGUF_TYPES[qtype] == O.GGUF_TYPES[qtype]
        raw = BI.gguf_blocks(qtype, 8, 512, seed=qtype)
        w = O.gguf_dequantize(raw, qtype, 8, 512)
        assert np.isfinite(w).all() and 1e-4 < np.abs(w).max() < 1.0, (qtype, np.abs(w).max())
    for qtype in (8, 2):
        x, raw = BI.cfg1_gguf(16, 256, 64, qtype=qtype, seed=1)
        w = O.gguf_dequantize(raw, qtype, 64, 256)
        assert x.dtype == torch.float16 and np.isfinite(w).all() and np.abs(w).max() < 0.2
