#!/usr/bin/env python
"""Quantized-linear TFLOP/s and % roofline at M=4096, K=3072, N=12288, per format, on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

A step is one call of the reference-facing operator over one batch: the INT8 ConvRot weight-only
linear of the benchmark configuration (X fp16 [4096, 3072] with 1% outlier channels, W int8
[12288, 3072] stored rotated, Hadamard block 128, per-channel fp16 scale, fp16 bias, fp16 out).
`value` is whole-job TFLOP/s (2*M*K*N per step, summed over ranks) with inputs resident in HBM;
`e2e` is the same op through the public API with the step's activations copied from pinned host
memory and its output copied back inside the timed region.  Every timed step is preceded by an
L2 flush (a 512 MB write) outside its CUDA-event window.  `formats` times every other weight
format at the same shape (one GPU).

With --gpus N (N > 1, one process per GPU under torchrun) the line's `value` is configuration 5
instead: the 60-block MMDiT linear stack with every weight sharded along N over the GPUs and the
outputs all-gathered over NVLink (strong scaling, time = max over ranks); the replicated headline
op moves to `replicated_cfg2`, and `mmdit_stack` carries the per-N breakdown (compute, exchange,
overlap, the all-outputs-gathered variant, the M-split replica control).

--impl reference times the reference's CPU dequantize + matmul path (restated in oracle/) on the
host cores instead, on the same workload.
"""
import argparse
import json
import os
import re
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "mac-kernels-public_b200")
for _p in (ROOT, PKG):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import numpy as np  # noqa: E402
import torch  # noqa: E402

import bench_inputs as BI  # noqa: E402

M, K, N = 4096, 3072, 12288
GROUP = 128
REF_BUDGET_S = 150.0  # reference arm: bound on the host-side run (warm-up + timed steps), seconds
FLOPS = 2.0 * M * K * N
METRIC = "quantized-linear TFLOP/s and % roofline at M=4096,K=3072,N=12288 per format"


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        p = json.load(open(path))
        return {"hbm_gbs": p["hbm_gbs"], "tflops": p["bf16_tflops"], "tflops_sustained": p.get("bf16_tflops_sustained"),
                "source": "measured"}
    return {"hbm_gbs": 6650.0, "tflops": 1590.0, "tflops_sustained": 1400.0, "source": "fallback"}


def workload_config(world):
    """The `config` of both arms' JSON lines (identical, so the two lines describe one workload)."""
    if world == 1:
        return {"workload": "int8_convrot_linear M=4096 K=3072 N=12288 group=128 fp16 out", "format": "int8_convrot",
                "hadamard": "sylvester-128", "l2": "GPU arm: flushed before every step; host arm: n/a",
                "parallelism": "1 GPU"}
    return {"workload": "mmdit_stack: 60 blocks x (QKV 3072->9216, out 3072->3072, up 3072->12288 Q4_K; "
                        "down 12288->3072 Q6_K), 4608 tokens",
            "format": "gguf q4_k + q6_k", "l2": "GPU arm: flushed before every step; host arm: n/a",
            "parallelism": f"N-sharded over {world} GPUs (weights split along N, outputs all-gathered over NVLink)"}


def profile_traffic(name):
    """Per-launch DRAM bytes recorded from an ncu capture in profiles/<name>.md, or None."""
    path = os.path.join(ROOT, "profiles", name + ".md")
    if not os.path.exists(path):
        return None
    m = re.search(r"traffic_bytes_per_launch:\s*([0-9.eE+]+)", open(path).read())
    return float(m.group(1)) if m else None


class ClockSampler:
    """nvidia-smi clock / throttle-reason samples every 100 ms while running."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device):
        self.device = device
        self.proc = None
        self.path = None

    def __enter__(self):
        try:
            bus = torch.cuda.get_device_properties(self.device).pci_bus_id
            ident = ["--id=" + bus] if bus else []
        except Exception:
            ident = []
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(["nvidia-smi", *ident, f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "100"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        rows = []
        if self.path and os.path.exists(self.path):
            for line in open(self.path):
                parts = [p.strip() for p in line.split(",")]
                if len(parts) >= 9:
                    rows.append(parts)
            os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        smax = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        load = [s for s in sm if smax and s > 0.5 * max(smax)] or sm
        return {"sm_mhz": statistics.median(load) if load else None, "sm_max_mhz": max(smax) if smax else None,
                "reasons": reasons, "samples": len(rows)}


def timed_steps(fn, steps, warmup, flush, stream):
    """Per-step device times (ms) with CUDA events on `stream`, L2 flushed before every step."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    times = []
    for _ in range(steps):
        flush.fill_(1)
        s = torch.cuda.Event(enable_timing=True)
        e = torch.cuda.Event(enable_timing=True)
        s.record(stream)
        fn()
        e.record(stream)
        times.append((s, e))
    torch.cuda.synchronize()
    return [s.elapsed_time(e) for s, e in times]


def roofline_time_s(flops, nbytes, pk):
    return max(nbytes / (pk["hbm_gbs"] * 1e9), flops / (pk["tflops"] * 1e12))


def cpu_reference_step(x_cpu, q_cpu, s_cpu, b_cpu, rows):
    """The reference's CPU path (dequantize the stored weight per call, fp32 linear), restated in
    oracle/: W = rotate(q * s) in fp32 torch, Y = X[:rows] . W^T + b."""
    from oracle import qlin_oracle as O
    w = O.rotate_rows(q_cpu.float() * s_cpu.float()[:, None], GROUP)
    return torch.nn.functional.linear(x_cpu[:rows].float(), w, b_cpu.float())


KIND = "restatement"  # the reference's CPU path restated in oracle/qlin_oracle.py (the reference's own
                     # port cannot build the Sylvester-128 rotation of the benchmark configuration)


def cpu_baseline(steps=2, rows=M):
    torch.set_num_threads(os.cpu_count() or 1)
    x, q, s, b = BI.cfg2_int8_convrot(M, K, N, seed=0)
    cpu_reference_step(x, q, s, b, 16)  # warm the BLAS threads
    t0 = time.perf_counter()
    for _ in range(steps):
        cpu_reference_step(x, q, s, b, rows)
    dt = (time.perf_counter() - t0) / steps
    return {"value": 2.0 * rows * K * N / dt / 1e12, "unit": "TFLOP/s", "cores": torch.get_num_threads(),
            "kind": KIND,
            "sample": f"{steps} full steps ({rows} of {M} token rows), weight dequantized (q*s, rotate) per step, "
                      f"fp32 torch on {torch.get_num_threads()} threads ({dt:.2f} s/step)"}


class _StackReferenceStep:
    """The reference's CPU path for one MMDiT block of configuration 5 (ComfyUI-GGUF's stock path:
    every GGUF weight dequantized per call, then an fp32 linear), restated in oracle/: the four
    linears QKV, out, up, down on all 4608 tokens, each over the first `frac` of its output
    channels (the block's weights are drawn once)."""

    def __init__(self, frac=1.0):
        from oracle import qlin_oracle as O
        self.O = O
        hid, self.tokens = 3072, 4608
        self.lin = [(12, 3 * hid, hid), (12, hid, hid), (12, 4 * hid, hid), (14, hid, 4 * hid)]
        self.raw = [BI.gguf_blocks(qt, n, k, seed=i) for i, (qt, n, k) in enumerate(self.lin)]
        g = torch.Generator().manual_seed(7)
        self.x = {k: torch.randn(self.tokens, k, generator=g) for k in (hid, 4 * hid)}
        self.frac = frac

    def flops(self):
        return sum(2.0 * self.tokens * self.rows(n) * k for _, n, k in self.lin)

    def rows(self, n):
        return max(256, int(n * self.frac) // 256 * 256)

    def __call__(self):
        for (qt, n, k), raw in zip(self.lin, self.raw):
            r = self.rows(n)
            w = torch.from_numpy(self.O.gguf_dequantize(raw[:r], qt, r, k))
            torch.nn.functional.linear(self.x[k], w)


def run_reference(args, rank, world):
    """The reference arm: the CPU path timed on the host cores for exactly `--steps` steps after
    `--warmup` untimed ones, on the workload our arm's line reports (one GPU: the INT8 ConvRot
    linear of configuration 2; several: one block of the configuration-5 stack).  A step covers the
    whole workload unit (all M token rows; all of a block's output channels) unless that would make
    the run longer than REF_BUDGET_S; then every step, warm-up and timed alike, covers the same
    smaller sample (a multiple of 256 rows / channels), sized from the first full-size step's time.
    Under torchrun only rank 0 runs it."""
    if rank != 0:
        return
    steps, warm = max(1, args.steps), max(0, args.warmup)
    torch.set_num_threads(os.cpu_count() or 1)
    if world == 1:
        x, q, s, b = BI.cfg2_int8_convrot(M, K, N, seed=0)
        state = {"rows": M}
        step = lambda: cpu_reference_step(x, q, s, b, state["rows"])  # noqa: E731
        flops = lambda: 2.0 * state["rows"] * K * N  # noqa: E731
        shrink = lambda f: state.update(rows=max(256, min(M, int(M * f) // 256 * 256)))  # noqa: E731
        describe = lambda: (f"{state['rows']} of {M} token rows per step; weight dequantized (q*s, rotate) per "  # noqa: E731
                            f"step; fp32 torch")
    else:
        step = _StackReferenceStep()
        flops = step.flops
        shrink = lambda f: setattr(step, "frac", min(1.0, f))  # noqa: E731
        describe = lambda: (f"one MMDiT block per step (4 GGUF linears, 4608 tokens, {100 * step.frac:.0f}% of "  # noqa: E731
                            f"each layer's output channels); weights dequantized per step (gguf-py restated); "
                            f"fp32 torch")
    done_warm = 0
    if warm > 0:
        t0 = time.perf_counter()
        step()
        t_full = time.perf_counter() - t0
        done_warm = 1
        left = warm - 1 + steps
        if left * t_full > REF_BUDGET_S:
            shrink(REF_BUDGET_S / (left * t_full))
    for _ in range(warm - done_warm):
        step()
    times = []
    for _ in range(steps):
        t0 = time.perf_counter()
        step()
        times.append(time.perf_counter() - t0)
    dt = statistics.mean(times)
    value = flops() / dt / 1e12
    line = {"metric": METRIC, "value": value, "unit": "TFLOP/s", "impl": "reference", "n_gpus": world,
            "steps": steps, "warmup": warm, "ms_per_step": dt * 1e3, "higher_is_better": True,
            "scaling": "weak" if world == 1 else "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "config": workload_config(world),
            "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": torch.get_num_threads(), "kind": KIND,
                             "sample": f"{steps} timed steps; " + describe()},
            "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def graph_steps(fn, steps, warmup, flush, stream):
    """Like timed_steps, but the op is captured once in a CUDA graph and replayed, so small ops are
    timed on the device without host launch gaps."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        fn()
    torch.cuda.synchronize()
    return timed_steps(g.replay, steps, 2, flush, stream)


def cold_chain_us(make_fn, copies, steps, flush, stream):
    """Per-call device time (us) of a small op with its weights cold in L2: `copies` calls, each on
    its own copy of the weights (together larger than L2), captured back to back in one CUDA graph;
    L2 is flushed before every replay and the replay time is divided by the number of calls.  This
    is how a model runs a stack of small-M linears (launch gaps inside a graph included), with every
    weight byte read from HBM."""
    fns = [make_fn(i) for i in range(copies)]
    for f in fns:
        f()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for f in fns:
            f()
    torch.cuda.synchronize()
    return statistics.mean(timed_steps(g.replay, steps, 2, flush, stream)) * 1e3 / copies


def int8_peak_tops(dev):
    """Dense int8 tensor peak measured the way MEASURED_PEAKS.json measures bf16: torch._int_mm at
    8192^3, best of 10 after warm-up."""
    a = torch.randint(-128, 127, (8192, 8192), dtype=torch.int8, device=dev)
    b = torch.randint(-128, 127, (8192, 8192), dtype=torch.int8, device=dev)
    for _ in range(3):
        torch._int_mm(a, b.t())
    torch.cuda.synchronize()
    best = float("inf")
    for _ in range(10):
        s = torch.cuda.Event(enable_timing=True)
        e = torch.cuda.Event(enable_timing=True)
        s.record()
        torch._int_mm(a, b.t())
        e.record()
        torch.cuda.synchronize()
        best = min(best, s.elapsed_time(e))
    del a, b
    return 2.0 * 8192 ** 3 / (best * 1e-3) / 1e12


def _w4a8_case(m, k, n, bits, grp, g, dev):
    x = torch.randn(m, k, generator=g).to(torch.float16).to(dev)
    lo, hi = (-8, 8) if bits == 4 else (-32, 32)
    wq = torch.randint(lo, hi, (n, k), generator=g, dtype=torch.int32)
    w = (BI.pack_w4(wq) if bits == 4 else BI.pack_w6(wq)).to(dev)
    s = (torch.randn(n, k // grp, generator=g).abs() * 0.02 / (7 if bits == 4 else 31)).to(torch.float16).to(dev)
    return x, w, s


def format_sweep(dev, steps, warmup, flush, stream, pk, int8_peak):
    """Every other weight format at the same (M, K, N), and the other benchmark configurations:
    device TFLOP/s (TOPS for the int8 tensor path) and roofline fractions."""
    import qlin
    out, cfgs = {}, {}
    g = torch.Generator().manual_seed(1)
    x = torch.randn(M, K, generator=g).to(torch.float16).to(dev)
    for qt, name in sorted((qt, "gguf_" + v[0].lower()) for qt, v in BI.GGUF_TYPES.items()):
        raw = torch.from_numpy(BI.gguf_blocks(qt, N, K, seed=qt)).to(dev)
        packed, _ = qlin.repack_gguf(raw, qt, (N, K))
        fn = lambda: qlin.gguf_linear(x, raw, qt, (N, K))  # noqa: E731
        t = statistics.mean(timed_steps(fn, steps, warmup, flush, stream))
        nbytes = raw.numel() + M * K * 2 + M * N * 2
        rt = roofline_time_s(FLOPS, nbytes, pk)
        out[name] = {"tflops": FLOPS / (t * 1e-3) / 1e12, "ms": t, "roofline_frac": rt / (t * 1e-3), "bound": "tensor"}
        del raw, packed
    pk8 = dict(pk, tflops=int8_peak)
    for bits, grp, name in ((4, 128, "w4a8_g128"), (6, 64, "w6a8_g64")):
        xx, w, s = _w4a8_case(M, K, N, bits, grp, g, dev)
        fn = lambda: qlin.w4a8_linear(xx, w, s, bits=bits, group_size=grp)  # noqa: E731
        t = statistics.mean(timed_steps(fn, steps, warmup, flush, stream))
        nbytes = w.numel() + s.numel() * 2 + M * K * 2 + M * N * 2
        rt = roofline_time_s(FLOPS, nbytes, pk8)
        out[name] = {"tops": FLOPS / (t * 1e-3) / 1e12, "ms": t, "roofline_frac": rt / (t * 1e-3),
                     "bound": "tensor (kind::i8, measured int8 peak)"}
    # The other benchmark configurations (reported for completeness; the headline is configuration 2).
    for qt, name in ((8, "cfg1_gguf_q8_0_256x3072x3072"), (2, "cfg1_gguf_q4_0_256x3072x3072")):
        xs, raw_np = BI.cfg1_gguf(256, 3072, 3072, qtype=qt, seed=0)
        xs = xs.to(dev)
        raw = torch.from_numpy(raw_np).to(dev)
        fn = lambda: qlin.gguf_linear(xs, raw, qt, (3072, 3072))  # noqa: E731
        t = statistics.mean(graph_steps(fn, steps, warmup, flush, stream))
        fl = 2.0 * 256 * 3072 * 3072
        nbytes = raw.numel() + 256 * 3072 * 2 * 2
        cfgs[name] = {"tflops": fl / (t * 1e-3) / 1e12, "us": t * 1e3,
                      "roofline_frac": roofline_time_s(fl, nbytes, pk) / (t * 1e-3),
                      "timing": "cuda graph replay of one call, L2 flushed"}
        # the same linear in a stack: 16 calls on 16 weight copies (160 MB, cold in L2) in one graph
        raws = [raw.clone() for _ in range(16)]
        tc = cold_chain_us(lambda i: (lambda: qlin.gguf_linear(xs, raws[i], qt, (3072, 3072))), 16, steps, flush,
                           stream)
        cfgs[name]["chain"] = {"us": tc, "tflops": fl / (tc * 1e-6) / 1e12,
                               "roofline_frac": roofline_time_s(fl, nbytes, pk) / (tc * 1e-6),
                               "timing": "16 calls on 16 weight copies per CUDA graph, L2 flushed per replay"}
        del raws
    # Small M (text tokens, adapter side paths): HBM-bound weight streaming, one launch.
    small = [(8, 3072, 3072, m, f"cfg1_small_gguf_q8_0_{m}x3072x3072") for m in (1, 16, 64)]
    small += [(12, 3072, 12288, 1, "small_m_gguf_q4_k_1x3072x12288"), (2, 3072, 3072, 1, "small_m_gguf_q4_0_1x3072x3072")]
    for qt, k, n, m, name in small:
        xs, raw_np = BI.cfg1_gguf(m, k, n, qtype=qt, seed=0)
        xs = xs.to(dev)
        raw = torch.from_numpy(raw_np).to(dev)
        fn = lambda: qlin.gguf_linear(xs, raw, qt, (n, k))  # noqa: E731
        t = statistics.mean(graph_steps(fn, steps, warmup, flush, stream))
        fl = 2.0 * m * k * n
        nbytes = raw.numel() + m * k * 2 + m * n * 2
        cfgs[name] = {"us": t * 1e3, "weight_stream_gbs": raw.numel() / (t * 1e-3) / 1e9,
                      "algorithmic_gbs": nbytes / (t * 1e-3) / 1e9,
                      "roofline_frac": roofline_time_s(fl, nbytes, pk) / (t * 1e-3), "bound": "hbm",
                      "timing": "cuda graph replay of one call, L2 flushed"}
        copies = max(16, int(3 * 126e6 // raw.numel()) + 1)  # together about three times L2
        raws = [raw.clone() for _ in range(copies)]
        tc = cold_chain_us(lambda i: (lambda: qlin.gguf_linear(xs, raws[i], qt, (n, k))), copies, steps, flush,
                           stream)
        cfgs[name]["chain"] = {"us": tc, "weight_stream_gbs": raw.numel() / (tc * 1e-6) / 1e9,
                               "roofline_frac": roofline_time_s(fl, nbytes, pk) / (tc * 1e-6),
                               "timing": f"{copies} calls on {copies} weight copies per CUDA graph, L2 flushed per "
                                         "replay (every weight byte from HBM)"}
        del raw, raws
    for (m, k, n, bits, grp), name in (((4096, 12288, 3072, 4, 128), "cfg3_w4a8_4096x12288x3072"),
                                       ((3240, 5120, 13824, 6, 64), "cfg4_w6a8_fwd_3240x5120x13824"),
                                       ((3240, 13824, 5120, 6, 64), "cfg4_w6a8_rev_3240x13824x5120")):
        xx, w, s = _w4a8_case(m, k, n, bits, grp, g, dev)
        fn = lambda: qlin.w4a8_linear(xx, w, s, bits=bits, group_size=grp)  # noqa: E731
        t = statistics.mean(timed_steps(fn, steps, warmup, flush, stream))
        fl = 2.0 * m * k * n
        nbytes = w.numel() + s.numel() * 2 + m * k * 2 + m * n * 2
        cfgs[name] = {"tops": fl / (t * 1e-3) / 1e12, "ms": t,
                      "roofline_frac": roofline_time_s(fl, nbytes, pk8) / (t * 1e-3)}
        del xx, w, s
    return out, cfgs


def qlin_status():
    import qlin
    return qlin.device_status()


def _max_over_ranks(v, dev, world):
    if world == 1:
        return v
    t = torch.tensor([v], device=dev)
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return float(t.item())


def _timed_replays(fn, steps, warmup, flush, stream, dev, world):
    """Mean device time (ms) of `steps` calls after `warmup`, bracketed by a barrier and a device
    synchronize on both sides, max over ranks."""
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    ms = statistics.mean(timed_steps(fn, steps, warmup, flush, stream))
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    return _max_over_ranks(ms, dev, world)


def _shard_linear_chain(st, x, dev):
    """A workload of the rank's shard linears: every block's gguf_linear_slabs calls of the
    NCCL-transport forward, in its order and shapes, on inputs that stay resident (the block input
    for linears reading it, random gathered-layout slabs for the others).  It contains no
    collective, so its time is the compute side of the stack."""
    import qlin
    kw = dict(dtype=torch.float16, device=dev)
    gen = torch.Generator(device=dev).manual_seed(5)
    ins, outs = {}, {}
    for name, _, _, n, k, src, _, _ in st.layers:
        if src == "x":
            ins[name] = x[:st.mc].unsqueeze(0)
        else:
            ins[name] = torch.randn(st.p, st.mc, k // st.p, generator=gen, **kw)
        outs[name] = torch.empty(st.mc, n // st.p, **kw)

    def run():
        for layer in st.blocks:
            for name, _, _, n, _, _, _, _ in st.layers:
                qtype, _, _, packed, row_exp = layer[name]
                for _c in range(st.chunks):
                    qlin.gguf_linear_slabs(ins[name], packed, row_exp, qtype, n // st.p, out=outs[name])
    return run


def _allgather_chain(st, dev):
    """A workload of NCCL all-gathers alone: every gathered output of the forward, per block and
    chunk, gathered back to back on the current stream ([mc, n/p] local -> [p, mc, n/p])."""
    kw = dict(dtype=torch.float16, device=dev)
    bufs = [(torch.zeros(st.mc, n // st.p, **kw), torch.empty(st.p * st.mc, n // st.p, **kw))
            for _, _, _, n, _, _, _, g in st.layers if g]

    def run():
        for _ in st.blocks:
            for loc, gat in bufs:
                for _c in range(st.chunks):
                    torch.distributed.all_gather_into_tensor(gat, loc, group=st.group)
    return run


def _graphed_chain(run):
    """run() once eagerly (communicators, workspaces), then captured into a CUDA graph."""
    run()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        run()
    torch.cuda.synchronize()
    return g


def run_mmdit(args, world, dev, flush, stream, steps, warmup, clk=None):
    """Configuration 5: the MMDiT block linear stack (60 blocks of QKV / out / MLP-up Q4_K and
    MLP-down Q6_K GGUF linears, 4608 tokens, hidden 3072), weights sharded along N over the ranks
    (strong scaling: the total work is fixed), outputs a later linear reads all-gathered into
    column slabs by the GEMM epilogues' stores into every rank's buffer over NVLink ("peer", the
    default) or by NCCL all-gathers on a side stream ("nccl").  Times are the max over ranks.

    With several GPUs it also reports, per forward: the same stack over NCCL, two workloads of
    their own that bound it -- the rank's shard linears back to back on resident inputs (compute)
    and NCCL all-gathers of the same sizes back to back (exchange) -- the overlap those imply, the
    variant that gathers every output (QKV's too), and the M-split replica control (every GPU holds
    all weights and runs 4608 / N tokens, no exchange)."""
    from qlin.sharded import ShardedStack
    transport = args.mmdit_transport
    tokens, hidden, blocks = 4608, 3072, args.mmdit_blocks
    # chunks only pay off when a separate gather overlaps the next chunk's GEMM
    chunks = args.mmdit_chunks or (4 if world > 1 and transport == "nccl" else 1)
    x = torch.randn(tokens, hidden, generator=torch.Generator().manual_seed(7)).to(torch.float16).to(dev)

    def graphed(st, **kw):
        for _ in range(2):
            st.forward(x, **kw)
        torch.cuda.synchronize()
        st.capture(x, **kw)  # one CUDA graph for the whole forward, NCCL gathers included
        torch.cuda.synchronize()

    st = ShardedStack(blocks=blocks, tokens=tokens, hidden=hidden, chunks=chunks, device=dev, transport=transport,
                      gather=args.mmdit_gather)
    graphed(st)
    finite = all(bool(torch.isfinite(o).all()) for o in st.graph_output)
    if clk is not None:
        clk.__enter__()
    ms = _timed_replays(st.replay, steps, warmup, flush, stream, dev, world)
    if clk is not None:
        clk.__exit__(None, None, None)
    out = {"tflops": st.flops() / (ms * 1e-3) / 1e12, "ms_per_forward": ms, "blocks": blocks, "chunks": chunks,
           "n_gpus": world, "scaling": "strong", "timing": "cuda graph replay, max over ranks",
           "transport": st.transport if world > 1 else "none", "gather": args.mmdit_gather,
           "launches_per_forward": st.launches_per_forward(), "output_finite": finite,
           "nvlink_bytes_in_per_rank_per_forward": st.gathered_bytes_per_forward(),
           "config": f"{tokens} tokens, hidden {hidden}, QKV/out/up Q4_K + down Q6_K, N-sharded over {world} GPUs, "
                     f"gathered outputs: {args.mmdit_gather}"}

    # end to end: the block input copied from pinned host memory, the forward, the output back
    xh = x.cpu().pin_memory()
    yh = torch.empty(len(st.graph_output), *st.graph_output[0].shape, dtype=torch.float16).pin_memory()

    def e2e():
        st.graph_input.copy_(xh, non_blocking=True)
        st.replay()
        for c, o in enumerate(st.graph_output):
            yh[c].copy_(o, non_blocking=True)

    e2e_ms = _timed_replays(e2e, max(3, steps // 2), 2, flush, stream, dev, world)
    out["e2e"] = {"value": st.flops() / (e2e_ms * 1e-3) / 1e12, "unit": "TFLOP/s", "ms": e2e_ms,
                  "h2d_bytes_per_step": xh.numel() * 2, "d2h_bytes_per_step": yh.numel() * 2}
    code, where = qlin_status()
    if code:
        raise SystemExit(f"MMDiT stack: a kernel gave up a bounded wait (status {code}, where {where:#x})")
    st.close()  # graphs holding NCCL calls go before the process group does; peer buffers after a barrier

    if world > 1 and not args.no_mmdit_breakdown:
        shared = lambda b, name, base, qtype, n_loc, k, rows: st.blocks[b][name][3:5]  # noqa: E731
        sub = max(3, steps // 2)
        # the same stack over NCCL; its GEMMs alone; its all-gathers alone
        nc = ShardedStack(blocks=blocks, tokens=tokens, hidden=hidden, chunks=chunks, device=dev, transport="nccl",
                          gather=args.mmdit_gather, weights=shared)
        graphed(nc)
        t_nccl = _timed_replays(nc.replay, sub, 2, flush, stream, dev, world)
        nc.release()
        g_comp = _graphed_chain(_shard_linear_chain(nc, x, dev))
        t_comp = _timed_replays(g_comp.replay, sub, 2, flush, stream, dev, world)
        g_comm = _graphed_chain(_allgather_chain(nc, dev))
        t_comm = _timed_replays(g_comm.replay, sub, 2, flush, stream, dev, world)
        del g_comp, g_comm  # graphs holding NCCL calls go before the process group
        nc.close()
        del nc
        gbytes = st.gathered_bytes_per_forward()
        out["breakdown"] = {
            "compute_ms": t_comp, "comm_ms_nccl_alone": t_comm, "total_ms": ms, "nccl_transport_ms": t_nccl,
            "overlap_frac": max(0.0, (t_comp + t_comm - ms) / t_comm) if t_comm > 0 else None,
            "nccl_allgather_gbs_per_rank_in": gbytes / (t_comm * 1e-3) / 1e9 if t_comm > 0 else None,
            "nvlink_floor_ms": gbytes / 770e9 * 1e3,
            "tensor_floor_ms": st.flops() / world / (peaks()["tflops"] * 1e12) * 1e3,
            # measured, not floors: compute when the stack runs within 10 % of its GEMMs alone; else the
            # NVLink floor when that is above the GEMMs; else the exchange and its cross-rank waits
            "limiter": ("compute" if ms <= 1.1 * t_comp else
                        "nvlink" if gbytes / 770e9 * 1e3 > t_comp else "exchange (not hidden behind the GEMMs)"),
            "note": "compute = this rank's shard linears of every block back to back on resident inputs of their "
                    "shapes (no collective in that workload); comm = NCCL all-gathers of the forward's sizes back "
                    "to back; nvlink floor = bytes each rank receives / 770 GB/s (measured peer copy)"}
        # every output gathered (QKV's too)
        if args.mmdit_gather != "all":
            al = ShardedStack(blocks=blocks, tokens=tokens, hidden=hidden, chunks=chunks, device=dev,
                              transport=transport, gather="all")
            graphed(al)
            t_all = _timed_replays(al.replay, sub, 2, flush, stream, dev, world)
            out["gather_all"] = {"tflops": al.flops() / (t_all * 1e-3) / 1e12, "ms_per_forward": t_all,
                                 "nvlink_bytes_in_per_rank_per_forward": al.gathered_bytes_per_forward()}
            al.close()
            del al
        # M-split replica control: all weights on every GPU, tokens / N each, no exchange
        rp = ShardedStack(blocks=blocks, tokens=tokens // world, hidden=hidden, chunks=1, device=dev, replica=True,
                          gather=args.mmdit_gather)
        graphed(rp)
        t_rep = _timed_replays(rp.replay, sub, 2, flush, stream, dev, world)
        out["m_split_replicas"] = {"tflops": world * rp.flops() / (t_rep * 1e-3) / 1e12, "ms_per_forward": t_rep,
                                   "tokens_per_gpu": tokens // world,
                                   "weights_per_gpu_gb": sum(v[3].numel() for b in rp.blocks for v in b.values()) / 1e9}
        rp.close()
        del rp
    del st
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    return out


def run_ours(args, rank, world):
    import qlin
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", 0)))
    torch.cuda.set_device(dev)
    stream = torch.cuda.current_stream(dev)
    pk = peaks()
    x, q, s, b = BI.cfg2_int8_convrot(M, K, N, seed=rank)
    xd, qd, sd, bd = x.to(dev), q.to(dev), s.to(dev), b.to(dev)
    flush = torch.empty(512 * 1024 * 1024, dtype=torch.uint8, device=dev)

    def step():
        return qlin.int8_linear(xd, qd, sd, bd, torch.float16, convrot=True, convrot_groupsize=GROUP)

    y = step()
    torch.cuda.synchronize()
    # parity before timing on rows from every token tile (61 apart, the last row of every 192-row
    # span, the last row), all output channels, against the float64 oracle (the checker)
    from oracle import qlin_oracle as O
    rows = sorted(set(range(0, M, 61)) | set(range(191, M, 192)) | {M - 1})
    ref = O.int8_convrot_linear_ref(x[rows].float().numpy(), q.numpy(), s.float().numpy(), b.float().numpy(),
                                    group=GROUP)
    got = y[rows].float().cpu().numpy()
    err = O.max_abs_rel(got, ref)
    if err > 2e-3 or not np.isfinite(got).all():
        raise SystemExit(f"parity check failed before timing: max-abs-rel {err} over {len(rows)} sampled rows")

    # Dominant kernel alone: the fused dequantize + GEMM on the already rotated fp16 operand,
    # timed before the loaded phase below (at the clocks of a kernel run alone), so its
    # denominator is the burst bf16 peak of MEASURED_PEAKS.json.
    xr, f = qlin.prologue_f16(xd, GROUP)
    xr_in = (xr[:, :K].float() * torch.exp2(f.float())[:, None]).to(torch.float16).contiguous()
    gemm = lambda: qlin.int8_linear(xr_in, qd, sd, bd, torch.float16, convrot=False)  # noqa: E731
    with ClockSampler(dev) as clk_gemm:
        t_gemm = statistics.mean(timed_steps(gemm, args.steps, args.warmup, flush, stream))
    achieved = FLOPS / (t_gemm * 1e-3) / 1e12
    traffic = profile_traffic("int8_convrot_gemm_cfg2")
    peak = pk["tflops"]
    roofline = {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                "frac": achieved / peak, "traffic": traffic,
                "algorithmic_bytes": q.numel() + 4 * N + M * K * 2 + M * N * 2,
                "peak_source": pk["source"] + " burst (kernel timed alone, before the loaded phase)",
                "kernel": "qgemm_f16_kernel<DecInt8> (planner: 192-token tiles, CTA pairs at this shape)",
                "kernel_ms": t_gemm, "kernel_clocks": clk_gemm.summary()}

    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    with ClockSampler(dev) as clk:
        # ~1 s of back-to-back steps so the clock samples see the GPU under this load, then the
        # timed steps
        t_end = time.perf_counter() + 1.0
        while time.perf_counter() < t_end:
            for _ in range(50):
                step()
            torch.cuda.synchronize()
        times = timed_steps(step, args.steps, args.warmup, flush, stream)
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    ms = statistics.mean(times)
    if world > 1:
        t = torch.tensor([ms], device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms = float(t.item())
    value = world * FLOPS / (ms * 1e-3) / 1e12

    algo_bytes = q.numel() + N * 2 + N * 2 + M * K * 2 + M * N * 2
    roof_t = roofline_time_s(FLOPS, algo_bytes, pk)

    # End to end through the public API: host X -> device, op, device Y -> host, per step.
    xh = x.pin_memory()
    yh = torch.empty(M, N, dtype=torch.float16).pin_memory()

    def e2e_step():
        # the host-memory entry point: copies in, op and copies out overlap chunk by chunk
        qlin.int8_linear_streamed(xh, qd, sd, bd, out=yh, convrot=True, convrot_groupsize=GROUP, chunks=8)

    t_e2e = statistics.mean(timed_steps(e2e_step, max(3, args.steps // 2), 2, flush, stream))
    if world > 1:
        t = torch.tensor([t_e2e], device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        t_e2e = float(t.item())

    formats, configs, int8_peak = {}, {}, None
    if not args.no_formats:
        int8_peak = int8_peak_tops(dev)
        formats, configs = format_sweep(dev, max(3, args.steps // 4), 3, flush, stream, pk, int8_peak)
    formats["int8_convrot_g128"] = {"tflops": FLOPS / (ms * 1e-3) / 1e12, "ms": ms,
                                    "roofline_frac": roof_t / (ms * 1e-3), "bound": "tensor"}
    if not args.no_formats:
        # unmerged rank-128 LoRA fused into the same GEMM (flops of the base linear only)
        gl = torch.Generator().manual_seed(5)
        down = (torch.randn(128, K, generator=gl) / K ** 0.5).half().to(dev)
        up = (torch.randn(N, 128, generator=gl) * 0.02).half().to(dev)
        fn = lambda: qlin.int8_linear(xd, qd, sd, bd, torch.float16, convrot=True, convrot_groupsize=GROUP,  # noqa: E731
                                      lora_down=down, lora_up=up, lora_scale=1.0)
        t = statistics.mean(timed_steps(fn, max(3, args.steps // 2), args.warmup, flush, stream))
        formats["int8_convrot_g128_lora_r128_fused"] = {"tflops": FLOPS / (t * 1e-3) / 1e12, "ms": t,
                                                         "overhead_vs_no_lora": t / ms - 1.0}
        # input gradient of the same frozen weight: dy [M, N] fp16 -> dx [M, K] (the transposed
        # weight copy is made once, before timing, as a training loop would)
        dy = torch.randn(M, N, generator=gl).half().to(dev)
        qlin.int8_linear_grad_input(dy, qd, sd, True, GROUP)
        fn = lambda: qlin.int8_linear_grad_input(dy, qd, sd, True, GROUP)  # noqa: E731
        t = statistics.mean(timed_steps(fn, max(3, args.steps // 2), args.warmup, flush, stream))
        formats["int8_convrot_g128_grad_input"] = {"tflops": FLOPS / (t * 1e-3) / 1e12, "ms": t,
                                                    "vs_forward_time": t / ms,
                                                    "note": "dx = dy . W, dy fp16 [4096, 12288] -> dx fp16 [4096, 3072]"}
        # the kitchen's default rotation (H4 Kronecker, 256): forward op and input gradient
        fn = lambda: qlin.int8_linear(xd, qd, sd, bd, torch.float16, convrot=True, convrot_groupsize=256)  # noqa: E731
        t256 = statistics.mean(timed_steps(fn, max(3, args.steps // 2), args.warmup, flush, stream))
        formats["int8_convrot_g256"] = {"tflops": FLOPS / (t256 * 1e-3) / 1e12, "ms": t256}
        fn = lambda: qlin.int8_linear_grad_input(dy, qd, sd, True, 256)  # noqa: E731
        t = statistics.mean(timed_steps(fn, max(3, args.steps // 2), args.warmup, flush, stream))
        formats["int8_convrot_g256_grad_input"] = {"tflops": FLOPS / (t * 1e-3) / 1e12, "ms": t,
                                                    "vs_forward_time": t / t256,
                                                    "note": "H4-256 rotates in a separate pass over fp32 dx"}
        # the kitchen's W4A8 / W6A8 layouts at the same shape: the packed codes decoded per call into a
        # transient int8 grid, then the INT8 GEMM; against the GEMM on an already decoded grid
        for bits, name in ((4, "kitchen_w4a8_cb_g16"), (6, "kitchen_w6a8_g16")):
            codes = torch.randint(0, 1 << bits, (N, K), generator=gl, dtype=torch.int64)
            qdata = BI.pack_kitchen(codes, bits).to(dev)
            s_rel = (torch.rand(N, K // 16, generator=gl) * 12 + 2).to(torch.float8_e4m3fn).to(dev)
            s_ch = (torch.rand(N, generator=gl) * 1e-3 + 1e-4).to(dev)
            cb = (torch.sort(torch.randn(16, generator=gl)).values * 3).to(dev) if bits == 4 else None
            fn = lambda: qlin.w4a8_int8_linear(xd, qdata, s_rel, s_ch, cb, None, bd, 16, GROUP, torch.float16)  # noqa: E731
            t_k = statistics.mean(timed_steps(fn, max(3, args.steps // 2), args.warmup, flush, stream))
            from qlin._w4a8 import kitchen_grid
            grid = kitchen_grid(qdata, s_rel, cb, 16)
            fn = lambda: qlin.int8_linear(xd, grid, s_ch, bd, torch.float16, convrot=True, convrot_groupsize=GROUP)  # noqa: E731
            t_g = statistics.mean(timed_steps(fn, max(3, args.steps // 2), args.warmup, flush, stream))
            formats[name] = {"tflops": FLOPS / (t_k * 1e-3) / 1e12, "ms": t_k, "predecoded_grid_ms": t_g,
                             "vs_predecoded_grid": t_k / t_g,
                             "resident_bytes": qdata.numel() + s_rel.numel() + 4 * N + (64 if cb is not None else 0),
                             "note": "codes decoded to a transient int8 grid every call (nothing cached)"}
            del grid, qdata, s_rel

    mmdit, clk_stack = None, None
    if world > 1:
        # several GPUs: the headline is the N-sharded configuration-5 stack, timed for exactly the
        # requested steps
        clk_stack = ClockSampler(dev)
        mmdit = run_mmdit(args, world, dev, flush, stream, args.steps, args.warmup, clk=clk_stack)
    elif not args.no_mmdit:
        mmdit = run_mmdit(args, world, dev, flush, stream, max(2, args.steps // 8), 1)

    base = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        base = cpu_baseline()

    if rank == 0:
        line = {"metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "f16 (int8 weights decoded exactly to fp16, fp32 accumulate)",
                "data": "synthetic (seeded; configuration 2 shapes and distributions)",
                "config": workload_config(world),
                "roofline": roofline,
                "roofline_op": {"bound": "tensor", "time_frac": roof_t / (ms * 1e-3),
                                "note": "whole op (rotation prologue + GEMM) vs max(bytes/HBM, flops/peak)"},
                "e2e": {"value": world * FLOPS / (t_e2e * 1e-3) / 1e12, "unit": "TFLOP/s",
                        "h2d_bytes_per_step": M * K * 2, "d2h_bytes_per_step": M * N * 2},
                "cpu_baseline": base, "formats": formats, "configs": configs, "mmdit_stack": mmdit,
                "int8_peak_tops_measured": int8_peak, "gpu_launches": 2 * args.steps,
                "parity_max_abs_rel": err, "clocks": clk.summary()}
        if world > 1:
            # the replicated configuration-2 op moves to its own key; the stack is the line
            line["replicated_cfg2"] = {"tflops": value, "ms": ms, "e2e_tflops": line["e2e"]["value"],
                                       "scaling": "weak", "note": "one independent replica of the headline op per GPU"}
            line.update(value=mmdit["tflops"], ms_per_step=mmdit["ms_per_forward"], scaling="strong",
                        dtype="f16 (GGUF Q4_K / Q6_K decoded to fp16, fp32 accumulate)",
                        data="synthetic (seeded; configuration 5 shapes, random legal GGUF blocks)",
                        e2e={k: mmdit["e2e"][k] for k in ("value", "unit", "h2d_bytes_per_step", "d2h_bytes_per_step")},
                        gpu_launches=mmdit["launches_per_forward"] * args.steps, clocks=clk_stack.summary())
            line["mmdit_stack"] = mmdit
            line.pop("roofline_op")
            line["roofline_stack"] = {k: mmdit.get("breakdown", {}).get(k) for k in
                                      ("nvlink_floor_ms", "tensor_floor_ms", "limiter")}
            if mmdit.get("breakdown"):
                floor = max(mmdit["breakdown"]["nvlink_floor_ms"], mmdit["breakdown"]["tensor_floor_ms"])
                line["roofline_stack"]["time_frac"] = floor / mmdit["ms_per_forward"]
        print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-formats", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-mmdit", action="store_true")
    ap.add_argument("--mmdit-blocks", type=int, default=60)
    ap.add_argument("--mmdit-chunks", type=int, default=0)
    ap.add_argument("--mmdit-transport", choices=("peer", "nccl"), default="peer")
    ap.add_argument("--mmdit-gather", choices=("consumed", "all"), default="consumed")
    ap.add_argument("--no-mmdit-breakdown", action="store_true")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if world > 1 and args.impl == "ours":
        import datetime
        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", 0)))
        # NCCL's own log lines (its version banner and communicator lines, when NCCL_DEBUG asks for
        # them) go to stderr: stdout carries only the JSON line of rank 0.
        os.environ.setdefault("NCCL_DEBUG_FILE", "/dev/stderr")
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                             device_id=torch.device("cuda", int(os.environ.get("LOCAL_RANK", 0))))
        args.no_formats = True  # the format sweep is a 1-GPU measurement
    try:
        if args.impl == "reference":
            run_reference(args, rank, world)
        else:
            run_ours(args, rank, world)
    finally:
        if world > 1 and args.impl == "ours" and torch.distributed.is_initialized():
            torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
