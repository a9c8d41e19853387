"""qlin_gguf_linear_noalloc: the GGUF linear for callers that cannot allocate device memory at
call time (a host without a caching allocator, where cudaMalloc would synchronize the device, or
one with an allocation-free steady state).  It takes its scratch from a fixed 16 MiB device array
inside the library instead of a caller workspace.

Checked through the C ABI against the existing entry point (qlin_gguf_linear with a caller
workspace) on two calls in a row with different inputs, so a second call cannot pass by reading
what the first left in the shared scratch.  This file is collected last on purpose."""
import numpy as np
import pytest
import torch

from oracle import qlin_oracle as O

pytestmark = pytest.mark.gpu


def _call_existing(lib, x, packed, row_exp, qtype, n, bias, y):
    m, k = x.shape
    ws_bytes = lib.qlin_gguf_linear_workspace(m, n, k, 1 if x.dtype == torch.float16 else 2, k)
    ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=x.device)
    return lib.qlin_gguf_linear(x.data_ptr(), 1 if x.dtype == torch.float16 else 2, m, k, k, packed.data_ptr(),
                                row_exp.data_ptr(), qtype, n, bias.data_ptr(), 1, y.data_ptr(), 1, n, ws.data_ptr(),
                                ws_bytes, torch.cuda.current_stream().cuda_stream)


def _call_noalloc(lib, x, packed, row_exp, qtype, n, bias, y):
    m, k = x.shape
    return lib.qlin_gguf_linear_noalloc(x.data_ptr(), 1 if x.dtype == torch.float16 else 2, m, k, k,
                                        packed.data_ptr(), row_exp.data_ptr(), qtype, n, bias.data_ptr(), 1,
                                        y.data_ptr(), 1, n, torch.cuda.current_stream().cuda_stream)


def test_noalloc_matches_workspace_entry_point_on_two_calls():
    assert torch.cuda.is_available(), "needs a CUDA device"
    import qlin
    lib = qlin.lib
    dev = torch.device("cuda", 0)
    # (qtype, m, n, k, x dtype): the first case runs split-K partials through the scratch, the
    # second also the bf16 -> fp16 activation copy.
    cases = [(8, 48, 384, 2048, torch.float16), (12, 200, 256, 1536, torch.bfloat16)]
    for i, (qtype, m, n, k, xdt) in enumerate(cases):
        g = torch.Generator().manual_seed(100 + i)
        x = torch.randn(m, k, generator=g).to(xdt).to(dev)
        raw = torch.from_numpy(O.random_gguf_blocks(qtype, n, k, seed=200 + i)).to(dev)
        bias = (torch.randn(n, generator=g) * 0.1).to(torch.float16).to(dev)
        packed, row_exp = qlin.repack_gguf(raw, qtype, (n, k))
        y_ref = torch.full((m, n), float("nan"), dtype=torch.float16, device=dev)
        y_new = torch.full((m, n), float("nan"), dtype=torch.float16, device=dev)
        assert _call_existing(lib, x, packed, row_exp, qtype, n, bias, y_ref) == 0, lib.qlin_last_error()
        assert _call_noalloc(lib, x, packed, row_exp, qtype, n, bias, y_new) == 0, lib.qlin_last_error()
        torch.cuda.synchronize()
        a = y_new.float().cpu().numpy()
        b = y_ref.float().cpu().numpy()
        assert np.isfinite(a).all()
        assert O.max_abs_rel(a, b) <= 2e-3
        # and both against the float64 reference
        ref = O.linear_f64(x.float().cpu().numpy(), O.gguf_dequantize(raw.cpu().numpy(), qtype, n, k),
                           bias.float().cpu().numpy())
        assert O.max_abs_rel(a, ref) <= 2e-3
    code, where = qlin.device_status()
    assert code == 0, where


def test_noalloc_rejects_calls_beyond_the_scratch_limit():
    import qlin
    lib = qlin.lib
    dev = torch.device("cuda", 0)
    m, n, k = 4096, 256, 3072  # bf16 input: the fp16 copy alone needs 24 MiB > 16 MiB
    x = torch.zeros(m, k, dtype=torch.bfloat16, device=dev)
    raw = torch.from_numpy(O.random_gguf_blocks(8, n, k, seed=1)).to(dev)
    packed, row_exp = qlin.repack_gguf(raw, 8, (n, k))
    bias = torch.zeros(n, dtype=torch.float16, device=dev)
    y = torch.zeros(m, n, dtype=torch.float16, device=dev)
    rc = _call_noalloc(lib, x, packed, row_exp, 8, n, bias, y)
    assert rc == 2
    assert b"16 MiB" in lib.qlin_last_error()
