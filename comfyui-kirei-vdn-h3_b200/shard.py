"""Head sharding of the VDN-H3 block over the GPUs of one node.

Every per-head computation of the block is independent: the q/k/v columns, the gate and
beta columns, the short-conv channels, the alpha / output-gate ``up`` rows, the frame
statistics, the factor, the scan and the readout.  Rank r of a group of g GPUs owns heads
[r*H/g, (r+1)*H/g) and computes them over the whole sequence (a head's frame recurrence
never crosses GPUs).  The ``down`` projections of alpha and the output gate (hidden ->
head_dim) are replicated.

The per-head outputs [S, 2*H/g*D] (gated softmax | branch readout) are then exchanged,
in ``chunks`` pipelined steps (RowExchange):

1. all-to-all by row block: in chunk c rank r receives its block of rows from every rank's
   heads, as [g][rows][2*H/g*D];
2. the output projection (out_proj + to_out_linear over K = 2*H*D) runs on those rows,
   reading the receive buffer in place as a grouped-K operand against the output weight
   whose columns were permuted once into the same rank-major order;
3. all-gather of the projected rows (asynchronous, overlapping the next chunk's projection)
   returns the full [S, hidden] output on every rank, which is what the patched
   ``attn.forward`` returns (hybrid.py:409-579 semantics).

The reference runs each block on one GPU; this module has no reference counterpart.
Collectives use ``torch.distributed`` (NCCL over NVLink on the GPU box, gloo in the CPU
tests); remote data always lands in local HBM before a kernel reads it.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass(frozen=True)
class HeadShard:
    """This rank's slice of the heads of one block."""

    rank: int
    world: int
    heads: int
    group: object = None  # torch.distributed process group (None = default group)

    def __post_init__(self):
        if self.world < 1 or not 0 <= self.rank < self.world:
            raise ValueError(f"rank {self.rank} outside a group of {self.world}")
        if self.heads % self.world:
            raise ValueError(f"{self.heads} heads do not split evenly over {self.world} GPUs")

    @property
    def heads_local(self) -> int:
        return self.heads // self.world

    @property
    def head0(self) -> int:
        return self.rank * self.heads_local

    @property
    def head_slice(self) -> slice:
        return slice(self.head0, self.head0 + self.heads_local)

    def row_block(self, seq_len: int) -> int:
        return -(-int(seq_len) // self.world)

    def rows_of(self, seq_len: int, rank: int | None = None) -> tuple[int, int]:
        """(first row, row count) of ``rank``'s block of the output projection."""
        r = self.rank if rank is None else int(rank)
        sb = self.row_block(seq_len)
        r0 = r * sb
        return r0, max(0, min(sb, int(seq_len) - r0))


def qkv_row_index(heads: int, dim: int, head_slice: slice) -> torch.Tensor:
    """Rows of W_qkv [3*H*D, hidden] that produce the q, k and v columns of the local heads."""
    inner = heads * dim
    cols = torch.arange(head_slice.start * dim, head_slice.stop * dim)
    return torch.cat([cols, cols + inner, cols + 2 * inner])


# Branch weights indexed by head (first axis H) or by channel h*D + d (first axis H*D,
# or the second axis of to_out_linear); everything else (norm, the down projections) is
# shared by all heads.  Names follow the reference's weight map (weights.py).
_HEAD_ROWS = ("beta_proj.weight", "alpha.A_log", "softmax_gate.up.weight", "softmax_gate.up.bias")
_CHANNEL_ROWS = ("alpha.dt_bias", "alpha.up.weight", "output_gate.up.weight", "output_gate.up.bias")
_CHANNEL_COLS = ("to_out_linear.weight",)


def slice_branch_weights(w, heads: int, dim: int, head_slice: slice) -> dict:
    """The branch weight map restricted to ``head_slice`` (a map for H/g heads).  Quantised
    ``to_out_linear`` masters are dropped: the row-split projection uses the full matrix."""
    hs = head_slice
    cs = slice(hs.start * dim, hs.stop * dim)
    out = {}
    for name, t in w.items():
        if name in _HEAD_ROWS:
            out[name] = t[hs]
        elif name in _CHANNEL_ROWS or name.startswith("short_conv."):
            out[name] = t[cs]
        elif name in _CHANNEL_COLS:
            out[name] = t[:, cs]
        elif name.startswith("to_out_linear."):
            continue
        else:
            out[name] = t
    return out


def rank_major_out_weight(out_w: torch.Tensor, to_out: torch.Tensor | None, heads: int, dim: int,
                          world: int) -> torch.Tensor:
    """[W_out | W_to_out] ([hidden, 2*H*D]) with its K columns reordered rank-major:
    for each rank r, r's heads of W_out, then r's heads of W_to_out -- the order in
    which the all-to-all receive buffer [g][rows][2*H/g*D] lays K out."""
    hidden = out_w.shape[0]
    if to_out is None:
        to_out = torch.zeros_like(out_w)
    hl = heads // world
    parts = []
    for r in range(world):
        cs = slice(r * hl * dim, (r + 1) * hl * dim)
        parts += [out_w[:, cs], to_out[:, cs]]
    w = torch.cat(parts, 1)
    assert w.shape == (hidden, 2 * heads * dim)
    return w


class RowExchange:
    """Buffers and collectives of one sequence length, pipelined over ``chunks``.

    Rows are cut into g * chunks blocks of ``cs`` rows, chunk-major: chunk c holds blocks
    c*g .. c*g + g - 1 and rank r owns block c*g + r of every chunk.  ``send`` is the rank's
    per-head output [g*chunks*cs, width] in natural row order (rows past S stay zero), so
    chunk c is one contiguous all-to-all send buffer; ``recv[c]`` is its result [g, cs,
    width].  The output projection of chunk c runs while chunk c+1 is exchanged, and the
    projected rows of chunk c are all-gathered (into a contiguous slab of the output, thanks
    to the chunk-major order) while chunk c+1 is projected."""

    def __init__(self, shard: HeadShard, seq_len: int, width: int, hidden: int, device, dtype=torch.bfloat16,
                 chunks: int = 1):
        self.shard = shard
        self.seq_len = int(seq_len)
        g = shard.world
        self.chunks = max(1, int(chunks))
        self.cs = -(-self.seq_len // (g * self.chunks))
        self.send = torch.zeros(g * self.chunks * self.cs, width, device=device, dtype=dtype)
        self.recv = torch.empty(self.chunks, g, self.cs, width, device=device, dtype=dtype)
        self.hidden = int(hidden)
        self._works = []

    @property
    def sb(self) -> int:  # rows of one block
        return self.cs

    def rows_of(self, chunk: int, rank: int | None = None) -> tuple[int, int]:
        """(first row, row count) of ``rank``'s block of ``chunk``."""
        r = self.shard.rank if rank is None else int(rank)
        r0 = (chunk * self.shard.world + r) * self.cs
        return r0, max(0, min(self.cs, self.seq_len - r0))

    def chunk_rows(self, chunk: int) -> tuple[int, int]:
        """[first, end) rows of ``chunk`` over all ranks (end clipped to the sequence)."""
        g, cs = self.shard.world, self.cs
        return chunk * g * cs, min(self.seq_len, (chunk + 1) * g * cs)

    def exchange_chunk(self, chunk: int):
        """Queue the all-to-all of one chunk (asynchronous; the collective waits for the work
        queued on the current stream so far, so it can start while later chunks are computed)."""
        import torch.distributed as dist

        g, cs = self.shard.world, self.cs
        c = chunk
        if c != len(self._works):
            raise RuntimeError("exchange chunks must be queued in order")
        self._works.append(dist.all_to_all_single(self.recv[c].view(g * cs, -1),
                                                  self.send[c * g * cs:(c + 1) * g * cs], group=self.shard.group,
                                                  async_op=True))

    def exchange(self):
        """Queue the all-to-all of every chunk not queued yet (asynchronous; each is waited on
        before use)."""
        for c in range(len(self._works), self.chunks):
            self.exchange_chunk(c)

    def project_and_gather(self, project, out: torch.Tensor | None = None) -> torch.Tensor:
        """Run ``project(recv[c], rows, out_rows, row0)`` on this rank's block of every chunk and
        all-gather the chunk; returns the [S, hidden] output.  ``project`` is called on
        every rank, with rows == 0 on a rank past the end of a short sequence, so that
        collectives it issues (the fp8 amax reduction) stay matched across ranks."""
        import torch.distributed as dist

        g, cs = self.shard.world, self.cs
        total = g * self.chunks * cs
        if out is None or out.shape != (total, self.hidden):
            out = torch.empty(total, self.hidden, device=self.send.device, dtype=self.send.dtype)
        self.exchange()
        gathers = []
        for c in range(self.chunks):
            self._works[c].wait()  # the compute stream waits for this chunk's exchange
            r0, n = self.rows_of(c)
            mine = out[r0:r0 + cs]
            project(self.recv[c], n, mine, r0)
            gathers.append(dist.all_gather_into_tensor(out[c * g * cs:(c + 1) * g * cs], mine,
                                                       group=self.shard.group, async_op=True))
        for w in gathers:
            w.wait()
        self._works = []
        return out[:self.seq_len]


class HeadGather:
    """The exchange the north star describes: every rank all-gathers the per-head outputs
    [S, 2*H/g*D] of every rank, chunk by chunk of rows, and projects all S rows itself (the
    output projection replicated on every rank, so no gather of projected rows follows).
    Same interface as ``RowExchange``: ``send`` holds this rank's per-head outputs in natural
    row order, ``recv[c]`` is chunk c as [g][cs][width] (rank-major K, the grouped-K GEMM's
    operand), and ``project_and_gather(project)`` returns the [S, hidden] output.

    Per rank it receives (g-1)/g * S * 2*H*D values and projects S rows; the row split
    receives (g-1)/g^2 of that plus the projected rows' all-gather, and projects S/g rows."""

    def __init__(self, shard: HeadShard, seq_len: int, width: int, hidden: int, device, dtype=torch.bfloat16,
                 chunks: int = 1):
        self.shard = shard
        self.seq_len = int(seq_len)
        g = shard.world
        self.chunks = max(1, int(chunks))
        self.cs = -(-self.seq_len // self.chunks)
        self.send = torch.zeros(self.chunks * self.cs, width, device=device, dtype=dtype)
        self.recv = torch.empty(self.chunks, g, self.cs, width, device=device, dtype=dtype)
        self.hidden = int(hidden)
        self._works = []

    def rows_of(self, chunk: int, rank: int | None = None) -> tuple[int, int]:
        """(first row, row count) this rank projects in ``chunk``: all of the chunk's rows."""
        r0 = chunk * self.cs
        return r0, max(0, min(self.cs, self.seq_len - r0))

    def chunk_rows(self, chunk: int) -> tuple[int, int]:
        r0 = chunk * self.cs
        return r0, min(self.seq_len, r0 + self.cs)

    def exchange_chunk(self, chunk: int):
        """Queue the all-gather of one chunk (asynchronous, ordered after the work queued on the
        current stream so far)."""
        import torch.distributed as dist

        g, cs = self.shard.world, self.cs
        c = chunk
        if c != len(self._works):
            raise RuntimeError("exchange chunks must be queued in order")
        self._works.append(dist.all_gather_into_tensor(self.recv[c].view(g * cs, -1), self.send[c * cs:(c + 1) * cs],
                                                       group=self.shard.group, async_op=True))

    def exchange(self):
        for c in range(len(self._works), self.chunks):
            self.exchange_chunk(c)

    def project_and_gather(self, project, out: torch.Tensor | None = None) -> torch.Tensor:
        """Run ``project(recv[c], rows, out_rows, row0)`` on every chunk (every rank projects
        every row); returns the [S, hidden] output."""
        total = self.chunks * self.cs
        if out is None or out.shape != (total, self.hidden):
            out = torch.empty(total, self.hidden, device=self.send.device, dtype=self.send.dtype)
        self.exchange()
        for c in range(self.chunks):
            self._works[c].wait()
            r0, n = self.rows_of(c)
            project(self.recv[c], n, out[r0:r0 + self.cs], r0)
        self._works = []
        return out[:self.seq_len]


EXCHANGES = {"rows": RowExchange, "heads": HeadGather}


def concat_rows(recv: torch.Tensor, rows: int) -> torch.Tensor:
    """[g, Sb, width] -> [rows, g*width]: the grouped-K operand as one matrix (the layout
    the quantised projections need, and the CPU tests' reading of the operand)."""
    g, _, w = recv.shape
    return recv[:, :rows].permute(1, 0, 2).reshape(rows, g * w)


def split_heads_outputs(a: torch.Tensor, world: int, inner_local: int) -> tuple[torch.Tensor, torch.Tensor]:
    """Undo the rank-major K order of ``concat_rows``: [rows, g*2*inner_l] ->
    (flat [rows, H*D], branch [rows, H*D]) in head order."""
    rows = a.shape[0]
    v = a.view(rows, world, 2, inner_local)
    return v[:, :, 0].reshape(rows, world * inner_local), v[:, :, 1].reshape(rows, world * inner_local)


def default_shard(heads: int, group=None) -> HeadShard | None:
    """HeadShard over ``group`` (the default group when None) if torch.distributed is
    initialised with more than one rank, else None."""
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()):
        return None
    world = dist.get_world_size(group)
    if world <= 1:
        return None
    return HeadShard(dist.get_rank(group), world, int(heads), group)


__all__ = ["EXCHANGES", "HeadGather", "HeadShard", "RowExchange", "concat_rows", "default_shard", "qkv_row_index",
           "rank_major_out_weight", "slice_branch_weights", "split_heads_outputs"]
