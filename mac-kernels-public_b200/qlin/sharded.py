"""N-sharded MMDiT block linear stack across the GPUs of one node (benchmark configuration 5).

Each rank holds a row shard of every weight -- GGUF blocks never straddle rows at these widths, so
a shard is a row selection of the raw tensor -- and computes its column shard of every output.
The outputs a later linear reads are all-gathered into column slabs [p][M][N/p], which the next
GEMM reads in place through a 3-D TMA map (no transpose pass).  Tokens may be split into chunks
that flow through the layers independently, so chunk c's exchange overlaps chunk c+1's GEMM.

Per block (hidden 3072): QKV 3072->9216, out 3072->3072, MLP up 3072->12288 (Q4_K) and MLP down
12288->3072 (Q6_K).  Attention and the MLP activation are not part of the linear stack.  Which
outputs are gathered (`gather`):
  "consumed" (default)  the QKV weight is sharded by heads -- rank r holds the Q, K and V rows of
          its own heads -- because attention is head-local: q, k and v need no exchange, and only
          attention's output, column-sharded like V, must be gathered before the out projection.
          That gather is modelled by gathering the V projection itself (same shape, M x hidden),
          and the out projection reads it.  Out, up and down outputs are gathered: the next linear
          reads all of them.  On one GPU the out projection reads the V columns of the QKV output.
  "all"   every output is gathered, QKV's too (the out projection then reads the block input);
          the V-for-attention stand-in is not needed.
Both do the same flops.

Transports for the gathers:
  "nccl"  the GEMM writes its local shard; an NCCL all-gather (side stream) assembles the slabs.
  "peer"  qlin_gguf_linear_allgather: the GEMM's epilogue stores every finished tile straight
          into all ranks' gathered buffers (CUDA-IPC mappings over NVLink), so the exchange
          overlaps the GEMM tile by tile, and a flag protocol between the ranks' kernels replaces
          the collective (no NCCL on the data path, one launch per linear).
"""
from __future__ import annotations

import math

import torch

import qlin

# base weights of one block: (name, GGUF type, rows, cols) as multiples of hidden
_BASE = {"qkv": (12, 3, 1), "out": (12, 1, 1), "up": (12, 4, 1), "down": (14, 1, 4)}
_BASE_INDEX = {"qkv": 0, "out": 1, "up": 2, "down": 3}


def layers(hidden=3072, gather="consumed", world=1):
    """One block's linears in launch order, as tuples
    (name, base, qtype, n, k, src, col0, gathered):
      base      the block weight whose rows this linear uses ("qkv", "out", "up", "down")
      n, k      output channels summed over all ranks, input features
      src       the linear whose output is this one's input ("x" = the block input)
      col0      first column of src's output that is read (one GPU: V inside QKV)
      gathered  whether the output is all-gathered for a later reader."""
    h = hidden
    tail = [("up", "up", 12, 4 * h, h, "out", 0, True), ("down", "down", 14, h, 4 * h, "up", 0, True)]
    if gather == "all":
        return [("qkv", "qkv", 12, 3 * h, h, "x", 0, True), ("out", "out", 12, h, h, "x", 0, True)] + tail
    if gather != "consumed":
        raise ValueError(f"unknown gather set {gather!r}")
    if world == 1:
        return [("qkv", "qkv", 12, 3 * h, h, "x", 0, False), ("out", "out", 12, h, h, "qkv", 2 * h, False)] + tail
    # v first: its all-gather kernel is the one that waits for the previous block's exchange to
    # land before anything reads the block input
    return [("v", "qkv", 12, h, h, "x", 0, True), ("qk", "qkv", 12, 2 * h, h, "x", 0, False),
            ("out", "out", 12, h, h, "v", 0, True)] + tail


def shard_rows(name, base, hidden, rank, world):
    """Rows of the base weight that rank `rank` holds for linear `name`: a contiguous 1/world of
    the rows, except for QKV, whose rows are grouped by heads -- rank r takes rows
    [r*h/p, (r+1)*h/p) of each of the Q, K and V blocks (h = hidden) -- in the order the linear's
    name lists them (qkv, qk or v)."""
    n_full = _BASE[base][1] * hidden
    if base != "qkv":
        loc = n_full // world
        return torch.arange(rank * loc, (rank + 1) * loc)
    loc = hidden // world
    part = {c: torch.arange(i * hidden + rank * loc, i * hidden + (rank + 1) * loc) for i, c in enumerate("qkv")}
    return torch.cat([part[c] for c in name])


_FIELDS = {12: ([0, 2], 5e-5), 14: ([208], 3e-5), 8: ([0], 0.02 / 127), 2: ([0], 0.02 / 7)}
# byte offsets of the fp16 block-scale fields (d, dmin) per type
_SCALE_OFFSETS = {12: [0, 2], 14: [208], 8: [0], 2: [0]}


def random_gguf_rows(qtype, n, k, gen, device):
    """Random legal blocks for an [n, k] weight: uniform bytes with the fp16 scale fields replaced by
    |N(0, 1)| * magnitude, on the device.  Q4_K blocks get dmin = 7.5 * d, so that with uniform codes
    and sub-block scales a block's weights d * sc * q - dmin * m average zero; otherwise every weight
    shares a positive offset that amplifies any common component of the activations about K-fold
    per layer."""
    name, qk, ts = qlin.GGUF_TYPES[qtype]
    nb = n * (k // qk)
    raw = torch.randint(0, 256, (nb, ts), dtype=torch.uint8, device=device, generator=gen)
    offs, mag = _FIELDS[qtype]
    for off in offs:
        d = (torch.randn(nb, device=device, generator=gen).abs() * mag).to(torch.float16)
        raw[:, off:off + 2] = d.view(torch.uint8).view(nb, 2)
    if qtype == 12:
        d = raw[:, 0:2].contiguous().view(torch.float16).float()
        raw[:, 2:4] = (d * 7.5).to(torch.float16).view(torch.uint8)
    return raw.view(n, (k // qk) * ts)


def base_weight(seed, block, base, hidden, device):
    """The full raw GGUF weight `base` of block `block` (the same on every rank).

    Random blocks amplify or damp activations by a layer-dependent factor (a 12288-wide Q6_K
    down projection about 3x), which over 60 blocks would run the stack's activations out of the
    fp16 range.  On a CUDA device each weight is therefore calibrated once: its gain on a fixed
    random probe, rms(x . W^T) / rms(x), is divided out of the fp16 block-scale fields (d, and dmin
    where the type has one; each rounded to fp16 again), so the stack keeps its activations in
    range over all 60 blocks.  The weights stay legal random GGUF blocks of the configuration's
    types."""
    qtype, rn, ck = _BASE[base]
    n, k = rn * hidden, ck * hidden
    gen = torch.Generator(device=device)
    gen.manual_seed(seed * 100003 + block * 16 + _BASE_INDEX[base])
    raw = random_gguf_rows(qtype, n, k, gen, device)
    if torch.device(device).type != "cuda":
        return raw
    probe = torch.randn(64, k, generator=torch.Generator().manual_seed(11)).to(torch.float16).to(device)
    y = qlin.gguf_linear(probe, raw, qtype, (n, k), out_dtype=torch.float32)
    gain = (y.square().mean().sqrt() / probe.float().square().mean().sqrt()).item()
    if gain > 0 and math.isfinite(gain) and abs(math.log2(gain)) > 0.01:
        name, qk, ts = qlin.GGUF_TYPES[qtype]
        rows = raw.view(-1, ts)
        for off in _SCALE_OFFSETS[qtype]:
            field = rows[:, off:off + 2].contiguous().view(torch.float16)
            rows[:, off:off + 2] = (field.float() / gain).to(torch.float16).view(torch.uint8)
    return raw


class ShardedStack:
    """`blocks` MMDiT blocks of GGUF linears, output channels split over the ranks of `group`.

    op(x_slabs, packed, row_exp, qtype, n, out) computes one shard GEMM; it defaults to
    qlin.gguf_linear_slabs (tests on CPU ranks pass a reference stand-in to check the plumbing).
    weights(block, name, base, qtype, n_loc, k, rows) may supply (packed, row_exp) per linear; by
    default every rank draws the full base weight from the seed and keeps its rows.
    replica=True runs the whole stack on this rank alone (all weights, no exchange): the M-split
    control, where every GPU takes its share of the tokens."""

    def __init__(self, blocks=60, tokens=4608, hidden=3072, chunks=4, group=None, device=None, seed=0, op=None,
                 weights=None, transport="nccl", gather="consumed", replica=False):
        dist = torch.distributed
        self.group = group
        multi_rank = dist.is_initialized() and not replica
        self.p = dist.get_world_size(group) if multi_rank else 1
        self.r = dist.get_rank(group) if multi_rank else 0
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        self.cuda = self.device.type == "cuda"
        self.gather = gather
        self.layers = layers(hidden, gather, self.p)
        if tokens % chunks:
            raise ValueError("tokens must split evenly into chunks")
        self.tokens, self.hidden, self.chunks, self.mc = tokens, hidden, chunks, tokens // chunks
        for name, _, _, n, _, _, _, _ in self.layers:
            if n % (64 * self.p):
                raise ValueError(f"{name}: {n} output channels do not split into {self.p} shards of 64-column slabs")
        self.op = op or (lambda x, packed, row_exp, qtype, n, out: qlin.gguf_linear_slabs(x, packed, row_exp, qtype, n,
                                                                                           out=out))
        self.blocks = []
        for b in range(blocks):
            layer, full = {}, {}
            for name, base, qtype, n, k, _, _, _ in self.layers:
                rows = shard_rows(name, base, hidden, self.r, self.p)
                n_loc = n // self.p
                if weights is not None:
                    packed, row_exp = weights(b, name, base, qtype, n_loc, k, rows)
                else:
                    if base not in full:
                        full[base] = base_weight(seed, b, base, hidden, self.device)
                    shard = full[base][rows.to(self.device)].contiguous()
                    packed, row_exp = qlin.repack_gguf(shard, qtype, (n_loc, k))
                    del shard
                layer[name] = (qtype, n, k, packed, row_exp)
            del full
            self.blocks.append(layer)
        if transport not in ("nccl", "peer"):
            raise ValueError(f"unknown transport {transport!r}")
        self.transport = transport if self.p > 1 else "nccl"
        kw = dict(dtype=torch.float16, device=self.device)
        if self.transport == "peer":
            self._init_peer()
            return
        # Per chunk: local output [mc, n/p] and gathered slabs [p, mc, n/p] per gathered linear.
        self.local = {name: [torch.empty(self.mc, n // self.p, **kw) for _ in range(chunks)]
                      for name, _, _, n, _, _, _, _ in self.layers}
        self.gathered = {name: [torch.empty(self.p, self.mc, n // self.p, **kw) for _ in range(chunks)]
                         for name, _, _, n, _, _, _, g in self.layers if g} if self.p > 1 else None
        # CUDA: gathers run on a side stream ordered by events.  CPU ranks (plumbing tests) run
        # everything in order on the host.
        multi = self.p > 1 and self.cuda
        names = [name for name, *_ in self.layers]
        self.comm = torch.cuda.Stream(device=self.device) if multi else None
        self.done = {name: [torch.cuda.Event() for _ in range(chunks)] for name in names} if multi else None
        self.ready = {name: [torch.cuda.Event() for _ in range(chunks)] for name in names} if multi else None

    def _init_peer(self):
        """Gathered buffers every rank stores into, [chunks][p][mc][n/p] per gathered linear, local
        outputs of the others, and the ranks' flag pads."""
        from .peer import PeerBuffer
        if not self.cuda:
            raise ValueError("the peer transport needs CUDA devices")
        kw = dict(dtype=torch.float16, device=self.device)
        self.bufs, self.gathered, self.local, self.y_ranks = {}, {}, {}, {}
        for name, _, _, n, _, _, _, gathered in self.layers:
            n_loc = n // self.p
            if not gathered:
                self.local[name] = [torch.empty(self.mc, n_loc, **kw) for _ in range(self.chunks)]
                continue
            slab = self.mc * n_loc * 2
            self.bufs[name] = PeerBuffer(self.chunks * self.p * slab, self.group, self.device)
            self.gathered[name] = [self.bufs[name].view((self.p, self.mc, n_loc), torch.float16,
                                                        offset=c * self.p * slab) for c in range(self.chunks)]
            self.y_ranks[name] = [[self.bufs[name].ptr(j, (c * self.p + self.r) * slab) for j in range(self.p)]
                                  for c in range(self.chunks)]
        self.pads = PeerBuffer(256, self.group, self.device)
        self.sync_ranks = [self.pads.ptr(j) for j in range(self.p)]
        self.comm = self.done = self.ready = None
        torch.cuda.synchronize(self.device)
        torch.distributed.barrier(group=self.group)

    def close(self):
        """Frees the peer buffers (after a barrier, so no rank still stores into them)."""
        self.release()
        if self.transport == "peer" and getattr(self, "pads", None) is not None:
            torch.cuda.synchronize(self.device)
            torch.distributed.barrier(group=self.group)
            for b in list(self.bufs.values()) + [self.pads]:
                b.close()
            self.pads = None

    def capture(self, x, **kw):
        """Records forward(x, **kw) once into a CUDA graph (GEMM launches, events and NCCL
        all-gathers); replay() then re-runs it without host launch overhead.  Run forward() at least
        once first so the communicators exist.  Call release() before the process group is
        destroyed."""
        self.graph_input = x
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.graph_output = self.forward(self.graph_input, **kw)
        return self.graph_output

    def replay(self):
        self.graph.replay()
        return self.graph_output

    def release(self):
        self.graph = None
        self.graph_output = None

    def flops(self):
        return len(self.blocks) * sum(2.0 * self.tokens * n * k for _, _, _, n, k, _, _, _ in self.layers)

    def launches_per_forward(self):
        return len(self.blocks) * len(self.layers) * self.chunks

    def gathered_bytes_per_forward(self):
        """Bytes every rank receives per forward: (p - 1) / p of each gathered output."""
        cols = sum(n for _, _, _, n, _, _, _, g in self.layers if g)
        return len(self.blocks) * self.tokens * cols * 2 * (self.p - 1) // self.p if self.p > 1 else 0

    def _src(self, src, col0, k, c, inp):
        """Chunk c of the input of a linear reading `src` (from column col0, k columns) as slabs."""
        if src == "x":
            return inp[c]
        if self.p == 1:
            return self.local[src][c][:, col0:col0 + k].unsqueeze(0)
        return self.gathered[src][c]

    def forward(self, x):
        """x: [tokens, hidden] fp16 on this rank's device (the same on every rank).  Returns the
        last block's output as chunk slabs ([p, mc, hidden/p] each, or [1, mc, hidden] on one GPU)."""
        if self.transport == "peer":
            return self._forward_peer(x)
        multi = self.comm is not None
        gather = self.p > 1
        comp = torch.cuda.current_stream(self.device) if self.cuda else None
        if multi and gather:
            self.comm.wait_stream(comp)  # (forked only when used: a graph capture must rejoin it)
        inp = [x[c * self.mc:(c + 1) * self.mc].unsqueeze(0) for c in range(self.chunks)]
        inp_ready = [None] * self.chunks
        # Events recorded during this forward; gathers of the previous forward are already ordered
        # before this one by the join at its end (and a CUDA graph may only wait on its own events).
        recorded = set()
        for layer in self.blocks:
            for name, _, _, n, k, src, col0, gathered in self.layers:
                qtype, _, _, packed, row_exp = layer[name]
                for c in range(self.chunks):
                    if multi and gather:
                        ready = inp_ready[c] if src == "x" else self.ready[src][c]
                        if ready is not None:
                            comp.wait_event(ready)
                        if (name, c) in recorded:
                            comp.wait_event(self.ready[name][c])  # the previous gather of this buffer is done
                    self.op(self._src(src, col0, k, c, inp), packed, row_exp, qtype, n // self.p, self.local[name][c])
                    if not (gathered and gather):
                        continue
                    if multi:
                        self.done[name][c].record(comp)
                        with torch.cuda.stream(self.comm):
                            self.comm.wait_event(self.done[name][c])
                            torch.distributed.all_gather_into_tensor(self.gathered[name][c].view(-1, n // self.p),
                                                                     self.local[name][c], group=self.group)
                            self.ready[name][c].record(self.comm)
                        recorded.add((name, c))
                    else:
                        torch.distributed.all_gather_into_tensor(self.gathered[name][c].view(-1, n // self.p),
                                                                 self.local[name][c], group=self.group)
            last = self.layers[-1][0]
            inp = [self._src(last, 0, self.hidden, c, inp) for c in range(self.chunks)]
            inp_ready = self.ready[last] if (multi and gather) else [None] * self.chunks
        if multi and gather:
            comp.wait_stream(self.comm)
        return inp

    def _forward_peer(self, x):
        inp = [x[c * self.mc:(c + 1) * self.mc].unsqueeze(0) for c in range(self.chunks)]
        for layer in self.blocks:
            for name, _, _, n, k, src, col0, gathered in self.layers:
                qtype, _, _, packed, row_exp = layer[name]
                for c in range(self.chunks):
                    xs = inp[c] if src == "x" else self.gathered[src][c]
                    if gathered:
                        qlin.gguf_linear_allgather(xs, packed, row_exp, qtype, n // self.p, self.y_ranks[name][c],
                                                   self.sync_ranks, self.r)
                    else:
                        # a local output read by nobody later in the block; the gather kernel
                        # launched before it on this stream already waited for the block input
                        qlin.gguf_linear_slabs(xs, packed, row_exp, qtype, n // self.p, out=self.local[name][c])
            inp = self.gathered[self.layers[-1][0]]
        # the last all-gather's stores from the other ranks land before anything reads the output
        qlin.peer_wait(self.sync_ranks, self.r, device=self.device)
        return list(inp)
