"""N-sharded MMDiT block linear stack across the GPUs of one node (benchmark configuration 5).

Each rank holds output rows [r*N/p, (r+1)*N/p) of every weight -- GGUF blocks never straddle rows
at these widths, so a shard is a row slice of the raw tensor -- and computes its column shard of
every output.  An NCCL all-gather assembles the full activation for the next linear as p column
slabs [p][M][N/p]; the GEMM reads that layout in place through a 3-D TMA map, so no transpose pass
is needed.  Tokens are split into chunks that flow through the layers independently: chunk c's
all-gather (on a side stream) overlaps chunk c+1's GEMM.

Two transports for the gathers:
  "nccl"  the GEMM writes its local shard; an NCCL all-gather (side stream) assembles the slabs.
  "peer"  qlin_gguf_linear_allgather: the GEMM's epilogue stores every finished tile straight
          into all ranks' gathered buffers (CUDA-IPC mappings over NVLink), so the exchange
          overlaps the GEMM tile by tile, and a flag protocol between the ranks' kernels replaces
          the collective (no NCCL on the data path, one launch per linear).

Per block (hidden 3072): QKV 3072->9216 (Q4_K), out 3072->3072 (Q4_K), MLP up 3072->12288
(Q4_K), MLP down 12288->3072 (Q6_K).  Attention and the activation function are not part of the
linear stack: the out projection reads the block input in place of the attention output, and the
down projection reads the up projection's output directly.  All four outputs are gathered.
"""
from __future__ import annotations

import torch

import qlin


def layers(hidden=3072):
    """(name, GGUF type, N, K) of the four linears of one block."""
    return (("qkv", 12, 3 * hidden, hidden), ("out", 12, hidden, hidden), ("up", 12, 4 * hidden, hidden),
            ("down", 14, hidden, 4 * hidden))


LAYERS = layers()
_FIELDS = {12: ([0, 2], 5e-5), 14: ([208], 3e-5), 8: ([0], 0.02 / 127), 2: ([0], 0.02 / 7)}


def random_gguf_rows(qtype, n, k, gen, device):
    """Random legal blocks for an [n, k] weight: uniform bytes with the fp16 scale fields replaced by
    |N(0, 1)| * magnitude, on the device."""
    name, qk, ts = qlin.GGUF_TYPES[qtype]
    nb = n * (k // qk)
    raw = torch.randint(0, 256, (nb, ts), dtype=torch.uint8, device=device, generator=gen)
    offs, mag = _FIELDS[qtype]
    for off in offs:
        d = (torch.randn(nb, device=device, generator=gen).abs() * mag).to(torch.float16)
        raw[:, off:off + 2] = d.view(torch.uint8).view(nb, 2)
    return raw.view(n, (k // qk) * ts)


class ShardedStack:
    """`blocks` MMDiT blocks of GGUF linears, output channels split over the ranks of `group`.

    op(x_slabs, packed, row_exp, qtype, n, out) computes one shard GEMM; it defaults to
    qlin.gguf_linear_slabs (tests on CPU ranks pass a reference stand-in to check the plumbing)."""

    def __init__(self, blocks=60, tokens=4608, hidden=3072, chunks=4, group=None, device=None, seed=0, op=None,
                 weights=None, transport="nccl"):
        dist = torch.distributed
        self.group = group
        self.p = dist.get_world_size(group) if dist.is_initialized() else 1
        self.r = dist.get_rank(group) if dist.is_initialized() else 0
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        self.cuda = self.device.type == "cuda"
        self.layers = layers(hidden)
        if tokens % chunks:
            raise ValueError("tokens must split evenly into chunks")
        self.tokens, self.hidden, self.chunks, self.mc = tokens, hidden, chunks, tokens // chunks
        for _, _, n, _ in self.layers:
            if n % (64 * self.p):
                raise ValueError(f"{n} output channels do not split into {self.p} shards of 64-column slabs")
        self.op = op or (lambda x, packed, row_exp, qtype, n, out: qlin.gguf_linear_slabs(x, packed, row_exp, qtype, n,
                                                                                           out=out))
        self.blocks = []
        for b in range(blocks):
            layer = {}
            for li, (name, qtype, n, k) in enumerate(self.layers):
                n_loc = n // self.p
                if weights is not None:
                    packed, row_exp = weights(b, name, qtype, n, k, self.r, self.p)
                else:
                    gen = torch.Generator(device=self.device)
                    gen.manual_seed(seed * 100003 + b * 16 + li)
                    full = random_gguf_rows(qtype, n, k, gen, self.device)
                    shard = full[self.r * n_loc:(self.r + 1) * n_loc].contiguous()
                    del full
                    packed, row_exp = qlin.repack_gguf(shard, qtype, (n_loc, k))
                    del shard
                layer[name] = (qtype, n, k, packed, row_exp)
            self.blocks.append(layer)
        if transport not in ("nccl", "peer"):
            raise ValueError(f"unknown transport {transport!r}")
        self.transport = transport if self.p > 1 else "nccl"
        if self.transport == "peer":
            self._init_peer()
            return
        # Per chunk: local output [mc, n/p] and gathered slabs [p, mc, n/p] per layer kind.
        kw = dict(dtype=torch.float16, device=self.device)
        self.local = {name: [torch.empty(self.mc, n // self.p, **kw) for _ in range(chunks)]
                      for name, _, n, _ in self.layers}
        self.gathered = {name: [torch.empty(self.p, self.mc, n // self.p, **kw) for _ in range(chunks)]
                         for name, _, n, _ in self.layers} if self.p > 1 else None
        # CUDA: gathers run on a side stream ordered by events.  CPU ranks (plumbing tests) run
        # everything in order on the host.
        multi = self.p > 1 and self.cuda
        self.comm = torch.cuda.Stream(device=self.device) if multi else None
        self.done = {name: [torch.cuda.Event() for _ in range(chunks)] for name, _, _, _ in self.layers} if multi else None
        self.ready = {name: [torch.cuda.Event() for _ in range(chunks)] for name, _, _, _ in self.layers} if multi else None

    def _init_peer(self):
        """Gathered buffers every rank stores into, [chunks][p][mc][n/p] per layer kind, and the
        ranks' flag pads."""
        from .peer import PeerBuffer
        if not self.cuda:
            raise ValueError("the peer transport needs CUDA devices")
        self.bufs, self.gathered, self.local = {}, {}, None
        for name, _, n, _ in self.layers:
            slab = self.mc * (n // self.p) * 2
            self.bufs[name] = PeerBuffer(self.chunks * self.p * slab, self.group, self.device)
            self.gathered[name] = [self.bufs[name].view((self.p, self.mc, n // self.p), torch.float16,
                                                        offset=c * self.p * slab) for c in range(self.chunks)]
        self.pads = PeerBuffer(256, self.group, self.device)
        self.sync_ranks = [self.pads.ptr(j) for j in range(self.p)]
        self.y_ranks = {name: [[self.bufs[name].ptr(j, (c * self.p + self.r) * self.mc * (n // self.p) * 2)
                                for j in range(self.p)] for c in range(self.chunks)]
                        for name, _, n, _ in self.layers}
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

    def capture(self, x):
        """Records forward(x) once into a CUDA graph (GEMM launches, events and NCCL all-gathers);
        replay() then re-runs it without host launch overhead.  Run forward() at least once first
        so the communicators exist.  Call release() before the process group is destroyed."""
        self.graph_input = x
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.graph_output = self.forward(self.graph_input)
        return self.graph_output

    def replay(self):
        self.graph.replay()
        return self.graph_output

    def release(self):
        self.graph = None
        self.graph_output = None

    def flops(self):
        return len(self.blocks) * sum(2.0 * self.tokens * n * k for _, _, n, k in self.layers)

    def _slabs(self, name, c):
        """Chunk c of the gathered output of layer `name` as [p, mc, n/p] (or [1, mc, n] on one GPU)."""
        if self.p == 1:
            return self.local[name][c].unsqueeze(0)
        return self.gathered[name][c]

    def forward(self, x):
        """x: [tokens, hidden] fp16 on this rank's device (the same on every rank).  Returns the
        last block's output as chunk slabs ([p, mc, hidden/p] each, or [1, mc, hidden] on one GPU)."""
        if self.transport == "peer":
            return self._forward_peer(x)
        multi = self.comm is not None
        comp = torch.cuda.current_stream(self.device) if self.cuda else None
        if multi:
            self.comm.wait_stream(comp)
        inp = [x[c * self.mc:(c + 1) * self.mc].unsqueeze(0) for c in range(self.chunks)]
        inp_ready = [None] * self.chunks
        # Events recorded during this forward; gathers of the previous forward are already ordered
        # before this one by the join at its end (and a CUDA graph may only wait on its own events).
        recorded = set()
        for layer in self.blocks:
            srcs = {"qkv": (inp, inp_ready), "out": (inp, inp_ready)}
            for name, _, _, _ in self.layers:
                if name == "up":
                    srcs["up"] = ([self._slabs("out", c) for c in range(self.chunks)],
                                  self.ready["out"] if multi else [None] * self.chunks)
                if name == "down":
                    srcs["down"] = ([self._slabs("up", c) for c in range(self.chunks)],
                                    self.ready["up"] if multi else [None] * self.chunks)
                src, src_ready = srcs[name]
                qtype, n, k, packed, row_exp = layer[name]
                for c in range(self.chunks):
                    if multi:
                        if src_ready[c] is not None:
                            comp.wait_event(src_ready[c])
                        if (name, c) in recorded:
                            comp.wait_event(self.ready[name][c])  # the previous gather of this buffer is done
                    self.op(src[c], packed, row_exp, qtype, n // self.p, self.local[name][c])
                    if multi:
                        self.done[name][c].record(comp)
                        with torch.cuda.stream(self.comm):
                            self.comm.wait_event(self.done[name][c])
                            torch.distributed.all_gather_into_tensor(self.gathered[name][c].view(-1, n // self.p),
                                                                     self.local[name][c], group=self.group)
                            self.ready[name][c].record(self.comm)
                        recorded.add((name, c))
                    elif self.p > 1:
                        torch.distributed.all_gather_into_tensor(self.gathered[name][c].view(-1, n // self.p),
                                                                 self.local[name][c], group=self.group)
            inp = [self._slabs("down", c) for c in range(self.chunks)]
            inp_ready = self.ready["down"] if multi else [None] * self.chunks
        if multi:
            comp.wait_stream(self.comm)
        return inp

    def _forward_peer(self, x):
        inp = [x[c * self.mc:(c + 1) * self.mc].unsqueeze(0) for c in range(self.chunks)]
        for layer in self.blocks:
            src = {"qkv": inp, "out": inp}
            for name, _, _, _ in self.layers:
                if name == "up":
                    src["up"] = self.gathered["out"]
                if name == "down":
                    src["down"] = self.gathered["up"]
                qtype, n, k, packed, row_exp = layer[name]
                for c in range(self.chunks):
                    qlin.gguf_linear_allgather(src[name][c], packed, row_exp, qtype, n // self.p,
                                               self.y_ranks[name][c], self.sync_ranks, self.r)
            inp = self.gathered["down"]
        return list(inp)
