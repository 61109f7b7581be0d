"""The MiniMax-H3 DiT block around the hybrid attention, on sm_100a.

Replaces the fused block forward of block_kernels.py (``make_fast_block_forward``,
:149-240) with the same contract: ``forward(x, t_emb, mod_segments, rope_freqs,
transformer_options=None, attention=None)``.  The reference runs five torch.compile'd
pointwise passes around attention and the MLP; here the whole block is

    h   = adaln_rmsnorm(x, norm1, scale_msa, shift_msa)        one row kernel
    x1  = x + gate_msa * attention(h)                          gated residual fused into the
                                                               attention's output projection
    h2  = adaln_rmsnorm(x1, norm2, scale_mlp, shift_mlp)       one row kernel (int8 codes too)
    a   = act(h2 fc1^T + b1)                                   GELU / SwiGLU in the fc1 epilogue
    out = x1 + gate_mlp * (a fc2^T + b2)                       gated residual in the fc2 epilogue

with every modulation table indexed per token by the row group of its segment
(block_kernels.py:34-60).  With the heads sharded over GPUs, the MLP runs token-parallel
on each rank's row block of the output projection, before the rows are all-gathered, so
the block costs one all-to-all and one all-gather however large the MLP.

The MLP runs in bf16 or INT8 (per-output-channel weights, per-token activations: the
config-2 scheme); SwiGLU is the reference's activation (block_kernels.py:113-115), GELU
(erf) the one BASELINE's 50-block configuration asks for.
"""

from __future__ import annotations

from collections import OrderedDict

import torch

from . import _lib
from .hybrid import STREAM_IO_KEY, B200State, FusedBlock, GatedResidual, StreamIO, _weight_of, gemm_block, rope_table
from .layout import current_layout
from .projection import QuantizedMatrix, quantize_weight

MLP_ACTIVATIONS = ("swiglu", "gelu")
_ACT_CODE = {"gelu": 2, "swiglu": 3}
SWIGLU_BLOCK = 128  # fc1 rows are interleaved in 128-row gate / up blocks: one GEMM tile holds a pair
MOD_NAMES = ("shift_msa", "scale_msa", "gate_msa", "shift_mlp", "scale_mlp", "gate_mlp")


def segment_indices(segments, rows: int, device) -> torch.Tensor:
    """Modulation row of every token as int32 [rows] (block_kernels.py:34-60): ``segments``
    (start, stop, row) must cover [0, rows) contiguously; ``row`` is an int, a 0-d tensor
    or a tensor of stop - start values."""
    ids = torch.empty(int(rows), dtype=torch.int32)
    covered = 0
    for raw_start, raw_stop, row in segments:
        start, stop = int(raw_start), int(raw_stop)
        if start != covered or stop < start or stop > rows:
            raise ValueError("MiniMax-H3 modulation segments must cover the sequence contiguously")
        count = stop - start
        if isinstance(row, torch.Tensor):
            row = row.detach().to("cpu", torch.int64)
            if row.ndim == 0:
                ids[start:stop] = int(row)
            elif row.numel() == count:
                ids[start:stop] = row.reshape(-1).to(torch.int32)
            else:
                raise ValueError(
                    f"modulation row tensor for [{start}:{stop}] has {row.numel()} values, expected {count}")
        else:
            ids[start:stop] = int(row)
        covered = stop
    if covered != rows:
        raise ValueError(f"MiniMax-H3 modulation segments cover {covered}/{rows} rows")
    return ids.to(device)


class SegmentIndexCache:
    """LRU of device row-group vectors for segment lists of plain ints (block_kernels.py:25-79);
    tensor-valued segments are rebuilt every call."""

    def __init__(self, limit: int = 16):
        self.limit = int(limit)
        self._ids: OrderedDict = OrderedDict()

    def indices(self, segments, rows: int, device) -> torch.Tensor:
        if any(isinstance(r, torch.Tensor) for _, _, r in segments):
            return segment_indices(segments, rows, device)
        dev = torch.device(device)
        key = (tuple((int(a), int(b), int(r)) for a, b, r in segments), int(rows), dev.type, dev.index)
        ids = self._ids.get(key)
        if ids is None:
            ids = segment_indices(key[0], rows, dev)
            self._ids[key] = ids
            while len(self._ids) > self.limit:
                self._ids.popitem(last=False)
        else:
            self._ids.move_to_end(key)
        return ids

    def clear(self):
        self._ids.clear()

    release = clear


def interleave_swiglu_rows(w: torch.Tensor, block: int = SWIGLU_BLOCK) -> torch.Tensor:
    """fc1 rows [gate; up] ([2F, ...], F % block == 0) -> [g_0 .. g_127, u_0 .. u_127, g_128, ...]
    so that one 256-row GEMM tile holds the gate block and its up block."""
    F2 = w.shape[0]
    if F2 % (2 * block):
        raise ValueError(f"SwiGLU fc1 has {F2} rows; the B200 MLP needs a multiple of {2 * block}")
    F = F2 // 2
    g, u = w[:F], w[F:]
    return torch.stack([g.reshape(F // block, block, *w.shape[1:]), u.reshape(F // block, block, *w.shape[1:])],
                       1).reshape(w.shape)


def _mods_device(mods, hidden, device):
    if len(mods) != 6:
        raise ValueError("adaln_proj must return (shift_msa, scale_msa, gate_msa, shift_mlp, scale_mlp, gate_mlp)")
    out = []
    for name, t in zip(MOD_NAMES, mods):
        t = t.detach().to(device, torch.bfloat16)
        t = t.reshape(-1, hidden).contiguous()
        out.append(t)
    return out


class B200DiTBlock:
    """Device weights of one DiT block (its attention is a :class:`FusedBlock`)."""

    def __init__(self, attn: FusedBlock, norm1_w, norm1_eps, norm2_w, norm2_eps, fc1_w, fc1_b, fc2_w, fc2_b,
                 device, *, activation="swiglu", precision="bf16", workspaces: dict | None = None):
        if activation not in MLP_ACTIVATIONS:
            raise ValueError(f"unsupported MLP activation {activation!r}")
        if precision not in ("bf16", "int8"):
            raise ValueError("the B200 MLP runs in bf16 or int8")
        dev = torch.device(device)
        hidden = attn.geo.hidden
        ffn = fc2_w.shape[1]
        if fc2_w.shape[0] != hidden or fc1_w.shape[1] != hidden:
            raise ValueError("MLP weights do not match the block's hidden size")
        if fc1_w.shape[0] != (2 * ffn if activation == "swiglu" else ffn):
            raise ValueError(f"fc1 has {fc1_w.shape[0]} rows; {activation} with fc2 of {ffn} columns needs "
                             f"{2 * ffn if activation == 'swiglu' else ffn}")
        self.attn = attn
        self.device = dev
        self.hidden, self.ffn = hidden, ffn
        self.activation = activation
        self.precision = precision
        self.eps1, self.eps2 = float(norm1_eps), float(norm2_eps)
        self.norm1 = norm1_w.detach().to(dev, torch.float32).contiguous()
        self.norm2 = norm2_w.detach().to(dev, torch.float32).contiguous()
        w1 = fc1_w.detach()
        b1 = fc1_b.detach() if fc1_b is not None else None
        if activation == "swiglu":
            w1 = interleave_swiglu_rows(w1)
            b1 = interleave_swiglu_rows(b1) if b1 is not None else None
        self.b1 = b1.to(dev, torch.float32).contiguous() if b1 is not None else None
        self.b2 = fc2_b.detach().to(dev, torch.float32).contiguous() if fc2_b is not None else None
        if precision == "bf16":
            self.w1 = w1.to(dev, torch.bfloat16).contiguous()
            self.w2 = fc2_w.detach().to(dev, torch.bfloat16).contiguous()
        else:
            self.w1 = quantize_weight(w1, "int8", dev)
            self.w2 = quantize_weight(fc2_w, "int8", dev)
        self._ws: dict = workspaces if workspaces is not None else {}  # shareable by like blocks
        self._ws_key = ("dit", hidden, ffn, precision)

    def workspace(self, rows: int) -> dict:
        """Buffers for ``rows`` rows (the pre-norm output, reused by both pre-norms, and the
        MLP activation); a larger workspace already held serves fewer rows."""
        ws = self._ws.get(self._ws_key)
        if ws is None or ws["h"].shape[0] < rows:
            dev, H, F = self.device, self.hidden, self.ffn
            ws = {"h": torch.empty(rows, H, device=dev, dtype=torch.bfloat16),
                  "a": torch.empty(rows, F, device=dev, dtype=torch.bfloat16)}
            if self.precision == "int8":
                ws["hq"] = QuantizedMatrix(torch.empty(rows, H, device=dev, dtype=torch.int8),
                                           torch.empty(rows, device=dev, dtype=torch.float32), "int8")
                ws["aq"] = QuantizedMatrix(torch.empty(rows, F, device=dev, dtype=torch.int8),
                                           torch.empty(rows, device=dev, dtype=torch.float32), "int8")
                ws["amax"] = torch.empty(rows, device=dev, dtype=torch.float32)
            self._ws[self._ws_key] = ws  # one row count at a time
        return ws

    # ------------------------------------------------------------------ kernels
    def _adaln(self, x, w, eps, scale, shift, group, out=None, q: QuantizedMatrix | None = None, stream=None):
        rows = x.shape[0]
        _lib.call("vdn_adaln_rmsnorm", x.data_ptr(), x.stride(0), rows, self.hidden, w.data_ptr(), float(eps),
                  scale.data_ptr(), shift.data_ptr(), scale.stride(0), group.data_ptr(), _lib.ptr(out),
                  out.stride(0) if out is not None else 0, _lib.ptr(q.data if q is not None else None),
                  q.data.stride(0) if q is not None else 0, _lib.ptr(q.scale if q is not None else None), stream)

    def mlp_rows(self, x1, group, mods, status, stream):
        """In place on the residual rows x1 [n, hidden]: x1 += gate_mlp * MLP(pre-norm(x1))."""
        n = x1.shape[0]
        if n == 0:
            return
        ws = self.workspace(n)
        shift, scale, gate = mods[3], mods[4], mods[5]
        act = _ACT_CODE[self.activation]
        res = GatedResidual(x1, gate, group)
        a = ws["a"][:n]
        if self.precision == "bf16":
            h = ws["h"][:n]
            self._adaln(x1, self.norm2, self.eps2, scale, shift, group, out=h, stream=stream)
            gemm_block(0, h, self.w1, a, col_bias=self.b1, act=act, status=status, stream=stream, rows=n)
            gemm_block(0, a, self.w2, x1, col_bias=self.b2, residual=res, status=status, stream=stream, rows=n)
            return
        hq = QuantizedMatrix(ws["hq"].data[:n], ws["hq"].scale[:n], "int8")
        self._adaln(x1, self.norm2, self.eps2, scale, shift, group, q=hq, stream=stream)
        # fc1's epilogue records each row's max |activation|, so the per-token int8 of the
        # activation for fc2 is one streaming pass
        amax = ws["amax"][:n]
        amax.zero_()
        gemm_block(2, hq.data, self.w1.data, a, row_scale=hq.scale, col_scale=self.w1.scale, col_bias=self.b1,
                   act=act, row_amax=amax, status=status, stream=stream, rows=n)
        aq = QuantizedMatrix(ws["aq"].data[:n], ws["aq"].scale[:n], "int8")
        _lib.call("vdn_quant_int8_rows_amax", a.data_ptr(), a.stride(0), n, self.ffn, amax.data_ptr(),
                  aq.data.data_ptr(), aq.data.stride(0), aq.scale.data_ptr(), stream)
        gemm_block(2, aq.data, self.w2.data, x1, row_scale=aq.scale, col_scale=self.w2.scale, col_bias=self.b2,
                   residual=res, status=status, stream=stream, rows=n)

    def forward(self, x, mods, group, layout, plans, status, *, out=None, io: StreamIO | None = None,
                **attn_kwargs) -> torch.Tensor:
        """x [S, hidden] bf16 (the residual stream), mods: the six adaln tables
        [groups, hidden], group [S] int32 -> the block output [S, hidden] bf16.  ``io``: x
        arrives and the output leaves by row blocks (``StreamIO``)."""
        _lib.require_cuda(x)
        compute = torch.cuda.current_stream(x.device)
        if io is not None and (x.dtype != torch.bfloat16 or x.stride(-1) != 1):
            io.wait_all(compute)
        if x.dtype != torch.bfloat16 or x.stride(-1) != 1:
            x = x.to(torch.bfloat16).contiguous()
        S = x.shape[0]
        stream = _lib.stream_handle(x.device)
        mods = _mods_device(mods, self.hidden, x.device)
        group = group.to(x.device, torch.int32).contiguous()
        h = self.workspace(S)["h"][:S]
        inner_io = None
        if io is not None and len(io.in_blocks) > 1:
            # pre-norm each row block as it lands; the attention then follows on this stream
            for k, (r0, r1) in enumerate(io.bounds()):
                io.wait(compute, k)
                self._adaln(x[r0:r1], self.norm1, self.eps1, mods[1], mods[0], group[r0:r1], out=h[r0:r1],
                            stream=stream)
            inner_io = StreamIO([(r1, None) for r1, _ in io.in_blocks], io.out_ready)
        else:
            if io is not None:
                io.wait_all(compute)
            self._adaln(x, self.norm1, self.eps1, mods[1], mods[0], group, out=h, stream=stream)
        residual = GatedResidual(x, mods[2], group)

        def mlp(rows_view, row0, n):
            self.mlp_rows(rows_view, group[row0:row0 + n], mods, status, stream)

        return self.attn.forward(h, layout, plans, status, out=out, residual=residual, row_epilogue=mlp, io=inner_io,
                                 **attn_kwargs)


def _dit_cache(state: B200State) -> dict:
    cache = getattr(state, "dit_blocks", None)
    if cache is None:
        cache = state.dit_blocks = {}
        state.segment_cache = SegmentIndexCache()
    return cache


def dit_block(state: B200State, block, index: int, device) -> B200DiTBlock:
    """The B200 weights of ``block`` (a ComfyUI MiniMax-H3 DiTBlock: norm1, attn, norm2,
    mlp.fc1 / mlp.fc2, adaln_proj), built once per state."""
    cache = _dit_cache(state)
    db = cache.get(index)
    if db is None:
        fb = state.fused_block(block.attn, index, device)
        mlp = block.mlp
        cfg = state.config
        db = B200DiTBlock(fb, _weight_of(block.norm1), getattr(block.norm1, "eps", 1e-6), _weight_of(block.norm2),
                          getattr(block.norm2, "eps", 1e-6), _weight_of(mlp.fc1), getattr(mlp.fc1, "bias", None),
                          _weight_of(mlp.fc2), getattr(mlp.fc2, "bias", None), device,
                          activation=str(cfg.get("mlp_activation", "swiglu")),
                          precision=str(cfg.get("mlp_precision", "int8" if state.projection_precision == "int8"
                                                else "bf16")), workspaces=state.workspaces)
        cache[index] = db
    return db


def make_fast_block_forward(block, state: B200State, block_index: int):
    """Drop-in ``DiTBlock.forward`` (block_kernels.py:149-240) on the B200 kernels.  As in the
    reference, a call with an ``attention`` override, or with no published VDN layout, runs
    the block's own forward."""
    original_forward = block.forward
    config = state.config

    def forward(x, t_emb, mod_segments, rope_freqs, transformer_options=None, attention=None):
        layout = current_layout(required=False)
        if attention is not None or layout is None:
            return original_forward(x, t_emb, mod_segments, rope_freqs,
                                    transformer_options=transformer_options or {}, attention=attention)
        if int(x.shape[0]) != layout.seq_len:
            raise RuntimeError(f"VDN layout has {layout.seq_len} rows but the block received {x.shape[0]}")
        _lib.require_cuda(x)
        db = dit_block(state, block, block_index, x.device)
        group = state.segment_cache.indices(mod_segments, x.shape[0], x.device)
        mods = block.adaln_proj(t_emb)
        status = state.device_status(x.device)
        out = db.forward(x, mods, group, layout, state.window_plans, status,
                         io=(transformer_options or {}).get(STREAM_IO_KEY),
                         linear_enabled=bool(config.get("linear_enabled", True)),
                         rope=rope_table(rope_freqs, layout.seq_len, state.head_dim, x.device))
        return out.to(x.dtype)

    forward._vdn_h3_fast_block = True
    forward._vdn_h3_block_index = int(block_index)
    forward._vdn_h3_original = original_forward
    return forward


__all__ = ["B200DiTBlock", "MLP_ACTIVATIONS", "SegmentIndexCache", "dit_block", "interleave_swiglu_rows",
           "make_fast_block_forward", "segment_indices"]
