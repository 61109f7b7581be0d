"""The VDN-H3 hybrid attention block on sm_100a (replaces vdn_h3/hybrid.py's operator).

``make_vdn_forward(attn, state, block_index)`` returns the same patched
``attn.forward(x, rope_freqs=None, transformer_options=None)`` the reference installs
(hybrid.py:409-579): layout from the request ContextVar, QKV, the linear branch on the
raw video q/k/v, q/k RMSNorm, exact window softmax, per-token head gate, out_proj and
the branch delta added on the video rows.

On the device one block forward is four phases, all on the caller's stream:

1. one tcgen05 GEMM of x against [W_qkv; W_gate; W_beta; W_og_down; W_alpha_down]
   writing raw q/k/v (bf16), per-head RMS-normalised q/k (bf16), the side projections
   (fp32) and the branch's q features (silu + L2, frame-head-token layout) from a single
   pass over x;
2. the branch kernels (features, alpha, statistics, Cholesky inverse, fused scan,
   gather/readout/RMSNorm/output gate) writing the branch rows of a [S, H*D] buffer;
3. the block-sparse window attention kernel with the gate fused in its epilogue;
4. one tcgen05 GEMM over K = 2*H*D of [gated softmax | branch] against
   [W_out | W_to_out]: out_proj, to_out_linear and the delta add in one pass when both
   projections are bf16; otherwise out_proj then to_out_linear (each in its own
   arithmetic) with an addend epilogue.

With a ``HeadShard`` (one process per GPU, torch.distributed) phases 1-3 run on this
rank's heads only, the attention chunk by chunk of rows with each chunk's exchange queued
behind it, and phase 4 becomes either all-to-all by row block, the output projection on
the rank's rows and an all-gather of the rows, or an all-gather of the per-head outputs and
the whole projection on every rank (shard.py).
"""

from __future__ import annotations

from collections.abc import Mapping
from dataclasses import dataclass

import torch

from . import _lib
from .branch import DELTA_RULES, BranchDeviceWeights, BranchWorkspace, cholesky_runtime_scope, run_branch
from .layout import VDNLayout, current_layout
from .projection import (CONVROT_KEY, KIND, QuantizedMatrix, dequantize_projection_weight, quantize_rows_int8,
                         quantize_rows_int8_convrot, quantize_tensor_fp8, quantize_weight)
from .shard import (EXCHANGES, HeadShard, RowExchange, concat_rows, default_shard, qkv_row_index, rank_major_out_weight,
                    slice_branch_weights, split_heads_outputs)
from .window import ATTENTION_BACKENDS, WindowPlanCache, launch_window_attention

STREAM_IO_KEY = "vdn_b200_io"  # transformer_options entry carrying a StreamIO (HostStreamer)
AUX_ALIGN = 32  # side columns padded to 32: 128-byte fp32 rows, and no extra 256-column GEMM tile
EXCHANGE_CHUNKS = 4  # pipelined exchange / projection / gather steps of the head-sharded block
EXCHANGE_MIN_ROWS = 512  # rows per rank and chunk (one wave of projection tiles); fewer: one step
# Work items per CTA below which the chunks of a head-sharded block share one attention launch:
# a persistent launch of few items per CTA loses its tail to the unevenly sized items (at 4 GPUs,
# config 1, four launches of 260 items made the kernel 1.3x slower per head than one launch).
ATTN_ITEMS_PER_CTA = 6


_SM_COUNT: dict = {}


def _sm_count(device) -> int:
    key = torch.device(device).index
    if key not in _SM_COUNT:
        _SM_COUNT[key] = torch.cuda.get_device_properties(device).multi_processor_count
    return _SM_COUNT[key]

# Branch settings a node config may leave out, with the values the reference falls back to:
# the node builds each block's branch from the config with these defaults (nodes.py:98-116)
# and the operator reads enable_text_state from the branch, then from the config with the
# same default (hybrid.py:449-451).
BRANCH_SETTING_DEFAULTS = {"delta_rule": "vdn_solve", "bridge": "alpha", "short_conv": (),
                           "enable_text_state": False}


def branch_setting(branch, config: Mapping, name: str):
    """A branch setting as the reference resolves it: the branch object's own attribute when
    the block's branch is an object (``LinearBranch`` / ``B200LinearBranch`` carry
    delta_rule, bridge, short_conv, enable_text_state), else the node config's value, else
    the reference default."""
    if branch is not None and not isinstance(branch, Mapping) and hasattr(branch, name):
        value = getattr(branch, name)
    else:
        value = config.get(name, BRANCH_SETTING_DEFAULTS[name])
    if name == "short_conv":
        return tuple(value)
    if name == "enable_text_state":
        return bool(value)
    return str(value)


def _weight_of(module_or_tensor):
    w = getattr(module_or_tensor, "weight", module_or_tensor)
    return w.detach()


@dataclass
class RopeTable:
    """``rope_freqs`` in the form the RoPE kernel reads: fp32 [rows or 1, rot/2 * 4] on the
    device, ``ld`` floats between rows (0: one set of matrices for every row)."""

    freqs: torch.Tensor
    rot: int
    ld: int


def rope_table(rope_freqs, seq: int, head_dim: int, device) -> RopeTable | None:
    """Canonical device form of the ``rope_freqs`` a block receives (hybrid.py:271-292 reads
    rot_dim = 2 * rope_freqs.shape[-3]; the trailing [rot/2, 2, 2] are ComfyUI's per-pair
    rotation matrices).  Leading dimensions must broadcast over the heads: after dropping
    size-1 dimensions they are empty (one table for all rows) or [seq]."""
    if rope_freqs is None:
        return None
    f = rope_freqs
    if not isinstance(f, torch.Tensor):
        raise TypeError(f"rope_freqs must be a tensor, got {type(f).__name__}")
    if f.ndim < 3 or tuple(f.shape[-2:]) != (2, 2):
        raise ValueError(f"rope_freqs must end in [rot/2, 2, 2], got {tuple(f.shape)}")
    half = int(f.shape[-3])
    rot = 2 * half
    if half < 1 or rot > head_dim:
        raise ValueError(f"rope rot_dim {rot} must be in [2, head_dim={head_dim}]")
    lead = [int(d) for d in f.shape[:-3] if d != 1]
    if not lead:
        n = 1
    elif lead == [seq]:
        n = seq
    else:
        raise ValueError(f"rope_freqs leading dims {tuple(f.shape[:-3])} must be one table or one per row "
                         f"({seq} rows), broadcast over heads")
    f = f.detach().to(device=device, dtype=torch.float32).reshape(n, half * 4).contiguous()
    return RopeTable(f, rot, 0 if n == 1 else half * 4)


@dataclass
class GatedResidual:
    """``x + gate[group[row]] * y`` fused into the projection that makes y (the DiT block's
    post-branch residual, block_kernels.py:92-93): x [S, hidden] bf16, gate [groups, hidden]
    bf16, group [S] int32."""

    x: torch.Tensor
    gate: torch.Tensor
    group: torch.Tensor

    def rows(self, r0: int, n: int) -> "GatedResidual":
        return GatedResidual(self.x[r0:r0 + n], self.gate, self.group[r0:r0 + n])


class StreamIO:
    """Row-block hand-over between host copies and one block forward (``HostStreamer``):
    ``in_blocks`` = [(row_end, event), ...] cover x in order, each event recorded when that
    block's copy-in landed; the block projects each row block as soon as it may and calls
    ``out_ready(out, row0, rows)`` once each block of its output is final.  A forward that
    cannot work by blocks waits for every block first (``wait_all``)."""

    def __init__(self, in_blocks, out_ready=None):
        self.in_blocks = list(in_blocks)
        self.out_ready = out_ready
        self.waited = 0

    def bounds(self):
        r0 = 0
        for r1, _ in self.in_blocks:
            yield r0, r1
            r0 = r1

    def wait(self, stream, k: int):
        ev = self.in_blocks[k][1]
        if ev is not None:  # None: the block was produced on the compute stream itself
            stream.wait_event(ev)
        self.waited = max(self.waited, k + 1)

    def wait_all(self, stream):
        if self.in_blocks and self.waited < len(self.in_blocks):
            self.wait(stream, len(self.in_blocks) - 1)  # one copy stream: the last block lands last
            self.waited = len(self.in_blocks)

    @property
    def complete(self) -> bool:
        return self.waited >= len(self.in_blocks)


def gemm_block(kind, a, w, out, *, a2=None, k_split=0, grouped=None, alpha=1.0, dev_scales=(None, None),
               row_scale=None, col_scale=None, col_bias=None, act=0, residual: GatedResidual | None = None,
               addend=None, row_amax=None, status, stream, rows=None, k=None):
    """One ``vdn_gemm_block`` call: out[:rows] = (residual or addend) + gate * act(scales * a w^T + bias).
    ``grouped`` = (groups, kg, group_stride) reads ``a`` as a grouped-K operand; ``row_amax``
    (zeroed fp32 [rows]) receives each output row's max |value|."""
    M = a.shape[-2] if rows is None else int(rows)
    K = (k if k is not None else (grouped[0] * grouped[1] if grouped else a.shape[-1] + (0 if a2 is None else
                                                                                          a2.shape[-1])))
    N = w.shape[0]
    groups, kg, gstride = grouped if grouped else (0, 0, 0)
    lda = a.stride(-2)
    res = residual.x if residual is not None else addend
    _lib.call("vdn_gemm_block", kind, a.data_ptr(), lda, _lib.ptr(a2), a2.stride(0) if a2 is not None else 0,
              int(k_split), int(gstride), int(kg), w.data_ptr(), w.stride(0), out.data_ptr(), out.stride(0), M, N, K,
              float(alpha), _lib.ptr(dev_scales[0]), _lib.ptr(dev_scales[1]), _lib.ptr(row_scale), _lib.ptr(col_scale),
              _lib.ptr(col_bias), int(act), _lib.ptr(res), res.stride(0) if res is not None else 0,
              _lib.ptr(residual.group if residual is not None else None),
              _lib.ptr(residual.gate if residual is not None else None),
              residual.gate.stride(0) if residual is not None else 0, _lib.ptr(row_amax), status.err_ptr, stream)


@dataclass
class BlockGeometry:
    heads: int
    dim: int
    hidden: int

    @property
    def inner(self):
        return self.heads * self.dim


class FusedBlock:
    """Device weights of one H3 attention block + its VDN branch, laid out for the kernels.

    ``precision`` is the arithmetic of this block's own projections (qkv_proj, out_proj);
    ``to_out_linear`` runs in the representation its map stores, as ``project`` dispatches
    on it (projection.py:259-268): a bf16 ``to_out_linear.weight`` stays bf16 whatever the
    block's precision (the edge blocks fp8.py:198 keeps in bf16), a quantised
    ``to_out_linear.weight_fp8`` runs as int8 or e4m3.  The branch settings (short_conv,
    delta_rule, bridge, enable_text_state) default to the released lineage, which is also
    ``LinearBranch``'s constructor default (branch.py:533-546); ``tile_frames`` > 0 runs the
    branch in frame tiles (runtime.py:421-543, same result)."""

    def __init__(self, qkv_w, q_norm_w, k_norm_w, out_w, branch_w: Mapping, heads, dim, device, *,
                 precision="bf16", eps=1e-6, enable_gate=True, short_conv=("k", "v"), shard: HeadShard | None = None,
                 workspaces: dict | None = None, delta_rule="vdn_solve", bridge="alpha", enable_text_state=True,
                 tile_frames=0, exchange="rows"):
        dev = torch.device(device)
        H_all, D = int(heads), int(dim)
        inner_all = H_all * D
        hidden = int(qkv_w.shape[1])
        if qkv_w.shape[0] != 3 * inner_all or out_w.shape != (hidden, inner_all):
            raise ValueError("attention weights do not match the head geometry")
        if shard is not None and shard.world == 1:
            shard = None
        if shard is not None and shard.heads != H_all:
            raise ValueError("head shard does not match the block's head count")
        self.shard = shard
        hs = shard.head_slice if shard is not None else slice(0, H_all)
        H = hs.stop - hs.start
        inner = H * D
        self.geo = BlockGeometry(H, D, hidden)  # this rank's heads
        self.heads_total = H_all
        self.device = dev
        self.precision = precision
        self.eps = float(eps)
        self.enable_gate = bool(enable_gate)
        self.short_conv = tuple(short_conv)
        if delta_rule not in DELTA_RULES:
            raise ValueError(f"unsupported delta_rule {delta_rule!r}")
        if bridge not in ("alpha", "none"):
            raise ValueError("bridge must be 'alpha' or 'none'")
        if isinstance(tile_frames, bool) or not isinstance(tile_frames, int) or tile_frames < 0:
            raise ValueError("tile_frames must be a non-negative integer")
        self.delta_rule = delta_rule
        self.bridge = bridge
        self.enable_text_state = bool(enable_text_state)
        self.tile_frames = tile_frames
        if exchange not in EXCHANGES:
            raise ValueError(f"unknown head-shard exchange {exchange!r}: one of {sorted(EXCHANGES)}")
        self.exchange = exchange  # head-sharded only: "rows" (all-to-all, row-split projection) or "heads"
        qkv_rows = qkv_row_index(H_all, D, hs)

        def f32(t):
            return t.detach().to(dev, torch.float32).contiguous()

        def b16(t):
            return t.detach().to(dev, torch.bfloat16).contiguous()

        # this rank's view of the branch weights (the full map on one GPU)
        wl = slice_branch_weights(branch_w, H_all, D, hs) if shard is not None else branch_w
        zeros_h = torch.zeros(H, hidden)
        gate_w = wl.get("softmax_gate.up.weight", zeros_h) if enable_gate else zeros_h
        self.gate_bias = f32(wl.get("softmax_gate.up.bias", torch.zeros(H))) if enable_gate else None
        side = [gate_w, wl.get("beta_proj.weight", zeros_h), wl.get("output_gate.down.weight",
                torch.zeros(D, hidden)), wl.get("alpha.down.weight", torch.zeros(D, hidden))]
        n_side = 2 * H + 2 * D
        self.n_aux = (n_side + AUX_ALIGN - 1) // AUX_ALIGN * AUX_ALIGN
        pad = torch.zeros(self.n_aux - n_side, hidden)
        side_w = torch.cat([s.detach().float().cpu() for s in side] + [pad], 0)
        # aux column offsets
        self.col_gate, self.col_beta, self.col_ogd, self.col_ad = 0, H, 2 * H, 2 * H + D
        self.norm_w = torch.cat([f32(q_norm_w), f32(k_norm_w)]).contiguous()
        self.has_branch = "to_out_linear.weight" in branch_w or "to_out_linear.weight_fp8" in branch_w
        to_out = branch_w.get("to_out_linear.weight")
        if to_out is not None and not self.has_branch:
            to_out = None
        # A stored quantised master (the reference's storage of fp8 / int8 projections,
        # fp8.py:168-222, projection.py:139-232) runs as stored: int8 codes with per-channel
        # scales (ConvRot when the map says so), e4m3 codes with a per-tensor scale.  Only an
        # e4m3 master with per-channel scales (fp8.py:88-96 on parts below sm_100) has no
        # kernel here; it is dequantised once to bf16.
        self.w_to_q = None
        self.to_out_convrot = None
        if to_out is None and "to_out_linear.weight_fp8" in branch_w:
            stored = branch_w["to_out_linear.weight_fp8"]
            stored_scale = branch_w["to_out_linear.weight_scale"]
            group = branch_w.get(CONVROT_KEY)
            group = None if group is None else int(group)
            stored_prec = "int8" if stored.dtype == torch.int8 else "fp8"
            if stored_prec == "int8" or (group is None and stored_scale.numel() == 1):
                self.w_to_q = QuantizedMatrix(stored.detach().to(dev).contiguous(),
                                              f32(stored_scale).reshape(-1).contiguous(), stored_prec)
                self.to_out_convrot = group
            else:
                to_out = dequantize_projection_weight(stored, stored_scale, group)
        # "bf16", "int8", "fp8" or None (no branch projection)
        self.to_out_kind = self.w_to_q.precision if self.w_to_q is not None else (
            "bf16" if to_out is not None else None)
        # one K-concat GEMM [flat | branch] x [W_out | W_to_out] when both projections are bf16
        self.concat_out = precision == "bf16" and self.to_out_kind in ("bf16", None)
        self.w_to_b16 = b16(to_out) if to_out is not None and not self.concat_out else None
        if precision == "bf16":
            self.w_big = torch.cat([b16(qkv_w[qkv_rows]), side_w.to(dev, torch.bfloat16)], 0).contiguous()
            if not self.concat_out:
                self.w_out = b16(out_w)
            elif shard is not None:
                # every rank projects all hidden columns of its row block: K in rank-major order
                self.w_out_cat = b16(rank_major_out_weight(out_w.detach().cpu(), None if to_out is None else
                                                           to_out.detach().cpu(), H_all, D, shard.world))
            elif to_out is not None:
                self.w_out_cat = torch.cat([b16(out_w), b16(to_out)], 1).contiguous()
            else:
                self.w_out_cat = torch.cat([b16(out_w), torch.zeros(hidden, inner, device=dev,
                                                                    dtype=torch.bfloat16)], 1).contiguous()
        else:
            # quantise the whole matrix, then keep this rank's rows: the fp8 per-tensor scale
            # stays the one of the full weight
            wq = quantize_weight(qkv_w, precision, dev)
            if shard is not None:
                idx = qkv_rows.to(dev)
                wq = QuantizedMatrix(wq.data[idx].contiguous(),
                                     wq.scale[idx].contiguous() if precision == "int8" else wq.scale, precision)
            self.w_qkv_q = wq
            self.w_side = side_w.to(dev, torch.bfloat16).contiguous()
            self.w_out_q = quantize_weight(out_w, precision, dev)
        self.bw = BranchDeviceWeights.from_dict(wl, H, D, dev, short_conv=self.short_conv) if self.has_branch \
            else None
        # blocks of one model run one after another on one stream: they may share workspaces
        # (pass the same dict), keyed by geometry, precision and shard so only like blocks meet
        self._ws: dict = workspaces if workspaces is not None else {}

    # ------------------------------------------------------------------ workspaces
    def _branch_tile(self, Fb: int):
        """Frames per branch tile, or None for the untiled branch."""
        return self.tile_frames if 0 < self.tile_frames < Fb else None

    def workspace(self, S: int, layout: VDNLayout | None):
        key = (S, None if layout is None else (layout.num_frames, layout.tokens_per_frame, layout.text_len,
                                               layout.anchor_frames),
               self.geo.heads, self.geo.dim, self.geo.hidden, self.precision, self.n_aux,
               None if self.shard is None else (self.shard.rank, self.shard.world, self.exchange), self.bw is not None,
               self.tile_frames)
        ws = self._ws.get(key)
        if ws is None:
            g = self.geo
            dev = self.device
            bf = dict(device=dev, dtype=torch.bfloat16)
            ws = {
                "qkv": torch.empty(S, 3 * g.inner, **bf),
                "qkn": torch.empty(S, 2 * g.inner, **bf),
                "aux": torch.empty(S, self.n_aux, device=dev, dtype=torch.float32),
            }
            if self.shard is not None:
                # per-head outputs [gated softmax | branch] side by side: one all-to-all chunk per rank
                # bf16: four chunks, so the exchange and the gather of one overlap the projection
                # of another; the quantised projections need whole-tensor activation scales (fp8)
                chunks = (EXCHANGE_CHUNKS if self.precision == "bf16" and S >= EXCHANGE_MIN_ROWS * EXCHANGE_CHUNKS *
                          self.shard.world else 1)
                xchg = EXCHANGES[self.exchange](self.shard, S, 2 * g.inner, g.hidden, dev, chunks=chunks)
                ws["xchg"] = xchg
                ws["flat"] = xchg.send[:S, :g.inner]
                ws["branch"] = xchg.send[:S, g.inner:]
                ws["branch_written"] = False
            else:
                ws["flat"] = torch.empty(S, g.inner, **bf)
                ws["branch"] = torch.zeros(S, g.inner, **bf)
            ws["work"] = torch.empty(1, device=dev, dtype=torch.float32)
            if layout is not None and self.bw is not None and not layout.full_cover:
                skip = layout.anchor_frames == "both"
                Fb = layout.num_frames - 2 if skip else layout.num_frames
                if Fb > 0:
                    ws["bws"] = BranchWorkspace(dev, Fb, layout.tokens_per_frame, g.heads, g.dim, layout.text_len,
                                                tile_frames=self._branch_tile(Fb))
            self._ws[key] = ws
        return ws

    def quant_buffer(self, ws, name: str, kind: str, rows: int, k: int) -> QuantizedMatrix:
        """Quantised-activation buffer ``name`` of ``kind`` (int8: per-row scales, fp8: one
        scale) in the shared workspace, allocated on first use: blocks of one model that
        share workspaces may store to_out_linear in different kinds (bf16 edge blocks)."""
        slot = f"{name}_{kind}"
        buf = ws.get(slot)
        if buf is None or buf.data.shape[0] < rows or buf.data.shape[1] != k:
            qdt = torch.int8 if kind == "int8" else torch.float8_e4m3fn
            dev = self.device
            buf = QuantizedMatrix(torch.empty(rows, k, device=dev, dtype=qdt),
                                  torch.empty(rows if kind == "int8" else 1, device=dev, dtype=torch.float32), kind)
            ws[slot] = buf
        return buf

    # ------------------------------------------------------------------ phases
    def _qkv(self, x, ws, status, stream, q_act=None, rows=None):
        """q_act: (buffer, first row, rows, tokens per frame) of the branch q features the
        epilogue writes, or None.  rows = (r0, r1): project only those rows of x (a block of
        the sequence whose copy has landed)."""
        g = self.geo
        r0, r1 = rows if rows is not None else (0, x.shape[0])
        S = r1 - r0
        x = x[r0:r1]
        qkv, qkn, aux = ws["qkv"][r0:r1], ws["qkn"][r0:r1], ws["aux"][r0:r1]
        qa = (None, 0, 0, 0) if q_act is None else (q_act[0].data_ptr(), q_act[1] - r0) + tuple(q_act[2:])
        if self.precision == "bf16":
            _lib.call("vdn_qkv_gemm", 0, x.data_ptr(), x.stride(0), self.w_big.data_ptr(), self.w_big.stride(0), S,
                      g.hidden, g.inner, self.n_aux, g.dim, self.norm_w.data_ptr(), self.eps, 1.0, None, None, None,
                      None, qkv.data_ptr(), qkv.stride(0), qkn.data_ptr(), qkn.stride(0), aux.data_ptr(),
                      aux.stride(0), *qa, status.err_ptr, stream)
            return
        kind = KIND[self.precision]
        xbuf = self.quant_buffer(ws, "xq", self.precision, ws["qkv"].shape[0], g.hidden)
        if self.precision == "int8":
            xq = quantize_rows_int8(x, QuantizedMatrix(xbuf.data[r0:r1], xbuf.scale[r0:r1], "int8"))
            rs, cs, d0, d1 = xq.scale, self.w_qkv_q.scale, None, None
        else:
            xq = quantize_tensor_fp8(x, QuantizedMatrix(xbuf.data[:S], xbuf.scale, "fp8"), ws["work"])
            rs, cs, d0, d1 = None, None, xq.scale, self.w_qkv_q.scale
        _lib.call("vdn_qkv_gemm", kind, xq.data.data_ptr(), xq.data.stride(0), self.w_qkv_q.data.data_ptr(),
                  self.w_qkv_q.data.stride(0), S, g.hidden, g.inner, 0, g.dim, self.norm_w.data_ptr(), self.eps, 1.0,
                  _lib.ptr(d0), _lib.ptr(d1), _lib.ptr(rs), _lib.ptr(cs), qkv.data_ptr(), qkv.stride(0),
                  qkn.data_ptr(), qkn.stride(0), None, 0, *qa, status.err_ptr, stream)
        # side projections stay bf16 -> fp32 (gates, beta, alpha are never quantised: fp8.py:1-12)
        _lib.call("vdn_gemm", 0, x.data_ptr(), x.stride(0), None, 0, 0, self.w_side.data_ptr(),
                  self.w_side.stride(0), aux.data_ptr(), aux.stride(0), 1, S, self.n_aux, g.hidden, 1.0,
                  None, None, None, None, None, 0, None, 0, status.err_ptr, stream)

    def _out(self, ws, out, with_branch, status, stream, residual: GatedResidual | None = None, rows=None):
        """The output projection of rows [r0, r1) (all rows by default)."""
        g = self.geo
        r0, r1 = rows if rows is not None else (0, out.shape[0])
        flat, branch, out = ws["flat"][r0:r1], ws["branch"][r0:r1], out[r0:r1]
        if residual is not None and rows is not None:
            residual = residual.rows(r0, r1 - r0)
        if self.concat_out:
            a2 = branch if with_branch else None
            gemm_block(0, flat, self.w_out_cat, out, a2=a2, k_split=g.inner if with_branch else 0,
                       k=2 * g.inner if with_branch else g.inner, residual=residual, status=status, stream=stream,
                       rows=r1 - r0)
            return
        self._two_pass_out(flat, branch if with_branch else None, ws, out, status, stream, residual=residual)

    def _two_pass_out(self, flat, branch, ws, out, status, stream, amax_reduce=None,
                      residual: GatedResidual | None = None):
        """out = P(flat) W_out^T, then + P'(branch) W_to^T as an addend pass, each in its own
        arithmetic: out_proj in the block's precision, to_out_linear in the kind its map
        stores.  Quantised activations are int8 per row (ConvRot for a ConvRot master) or
        e4m3 per tensor (``amax_reduce`` combines the amax of the ranks' row blocks).  With a
        ``residual`` both passes are gated and the first adds the residual stream."""
        rows = flat.shape[0]
        K = flat.shape[1]

        def project_pass(src, name, kind, w, first, convrot=None):
            res = None
            if residual is not None:
                res = residual if first else GatedResidual(out, residual.gate, residual.group)
            addend = None if (first or res is not None) else out
            if kind == "bf16":
                if rows > 0:
                    gemm_block(0, src, w, out, residual=res, addend=addend, status=status, stream=stream, rows=rows,
                               k=K)
                return
            if rows == 0 and kind == "int8":
                return  # per-row scales: nothing to combine across ranks
            buf = self.quant_buffer(ws, name, kind, rows, K)
            buf = QuantizedMatrix(buf.data[:rows], buf.scale[:rows] if kind == "int8" else buf.scale, kind)
            if kind == "int8":
                qa = quantize_rows_int8(src, buf) if convrot is None else \
                    quantize_rows_int8_convrot(src, buf, group=convrot)
                rs, cs, d0, d1 = qa.scale, w.scale, None, None
            else:
                qa = quantize_tensor_fp8(src, buf, ws["work"], amax_reduce=amax_reduce)
                rs, cs, d0, d1 = None, None, qa.scale, w.scale
            if rows == 0:
                return
            gemm_block(KIND[kind], qa.data, w.data, out, dev_scales=(d0, d1), row_scale=rs, col_scale=cs,
                       residual=res, addend=addend, status=status, stream=stream, rows=rows, k=K)

        if self.precision == "bf16":
            project_pass(flat, "fq", "bf16", self.w_out, True)
        else:
            project_pass(flat, "fq", self.precision, self.w_out_q, True)
        if branch is None or self.to_out_kind is None:
            return
        if self.to_out_kind == "bf16":
            project_pass(branch, "bq", "bf16", self.w_to_b16, False)
        else:
            project_pass(branch, "bq", self.to_out_kind, self.w_to_q, False, self.to_out_convrot)

    def project_rows(self, ws, with_branch, recv, rows, out_rows, status, stream, amax_reduce=None,
                     residual: GatedResidual | None = None):
        """Head-sharded phase 4 on this rank: the output projection of ``rows`` rows from
        the all-to-all receive buffer ``recv`` [ranks, Sb, 2*H/g*D] into ``out_rows``
        (``residual``: already restricted to those rows)."""
        g = self.geo
        world = recv.shape[0]
        if self.concat_out:
            if rows > 0:
                gemm_block(0, recv, self.w_out_cat, out_rows, grouped=(world, 2 * g.inner, recv.stride(0)),
                           residual=residual, status=status, stream=stream, rows=rows)
            return
        flat, branch = split_heads_outputs(concat_rows(recv, rows), world, g.inner)
        self._two_pass_out(flat, branch if with_branch else None, ws, out_rows, status, stream,
                           amax_reduce=amax_reduce, residual=residual)

    def _out_sharded(self, ws, with_branch, status, stream, residual: GatedResidual | None = None,
                     row_epilogue=None) -> torch.Tensor:
        """The exchange of the per-head outputs and the output projection (grouped-K over the
        receive buffer), ``row_epilogue(rows_view, row0, n)`` on the projected rows (the DiT
        block's token-parallel MLP): all-to-all by row block, this rank's rows, all-gather of
        the rows ("rows"); or all-gather of the per-head outputs and every row on every rank
        ("heads")."""
        sh = self.shard
        xchg = ws["xchg"]
        xchg.exchange()  # the chunks the attention launches have not queued yet
        amax_reduce = None
        if self.precision == "fp8" and isinstance(xchg, RowExchange):
            # each rank quantises its row block: the per-tensor amax is the ranks' maximum
            import torch.distributed as dist

            def amax_reduce(t):
                dist.all_reduce(t, op=dist.ReduceOp.MAX, group=sh.group)

        def project(recv, rows, out_rows, row0):
            self.project_rows(ws, with_branch, recv, rows, out_rows, status, stream, amax_reduce,
                              residual.rows(row0, rows) if residual is not None else None)
            if row_epilogue is not None:
                row_epilogue(out_rows[:rows], row0, rows)

        return xchg.project_and_gather(project)

    def forward(self, x: torch.Tensor, layout: VDNLayout, plans: WindowPlanCache, status: _lib.DeviceStatus,
                *, linear_enabled=True, bridge=None, enable_text_state=None, out=None,
                residual: GatedResidual | None = None, row_epilogue=None, io: StreamIO | None = None,
                rope: RopeTable | None = None) -> torch.Tensor:
        """The block output [S, hidden]; with ``residual`` the gated residual stream
        ``residual.x + gate * block(x)`` instead, and ``row_epilogue(rows_view, row0, n)``
        run on the projected rows (in place) before they leave this GPU.  ``io``: x arrives
        and the output leaves by row blocks (see :class:`StreamIO`).  ``rope``: rotary
        embedding of the normalised q / k (``rope_table``)."""
        ws, linear_active = self.forward_heads(x, layout, plans, status, linear_enabled=linear_enabled,
                                               bridge=bridge, enable_text_state=enable_text_state, io=io, rope=rope,
                                               issue_exchange=self.shard is not None)
        stream = _lib.stream_handle(x.device)
        if self.shard is not None:
            full = self._out_sharded(ws, linear_active, status, stream, residual, row_epilogue)
            if out is None:
                return full
            out.copy_(full)
            return out
        if out is None:
            out = torch.empty(x.shape[0], self.geo.hidden, device=x.device, dtype=torch.bfloat16)
        blocks = list(io.bounds()) if io is not None and io.out_ready is not None and self.precision != "fp8" \
            else [(0, out.shape[0])]
        for r0, r1 in blocks:
            self._out(ws, out, linear_active, status, stream, residual, rows=(r0, r1))
            if row_epilogue is not None:
                row_epilogue(out[r0:r1], r0, r1 - r0)
            if io is not None and io.out_ready is not None and len(blocks) > 1:
                io.out_ready(out, r0, r1 - r0)
        return out

    def forward_heads(self, x: torch.Tensor, layout: VDNLayout, plans: WindowPlanCache, status: _lib.DeviceStatus,
                      *, linear_enabled=True, bridge=None, enable_text_state=None, io: StreamIO | None = None,
                      rope: RopeTable | None = None, issue_exchange=False):
        """Phases 1-3 (QKV, branch, window attention) for this rank's heads; returns the
        workspace holding the per-head outputs and whether the branch ran.  ``bridge`` /
        ``enable_text_state``: None takes the block's own settings.  ``issue_exchange``
        (head-sharded, several exchange chunks): the attention runs chunk by chunk of rows and
        each chunk's exchange is queued as soon as its rows are written, so it crosses NVLink
        while the next chunk is computed."""
        g = self.geo
        S = x.shape[0]
        bridge = self.bridge if bridge is None else bridge
        enable_text_state = self.enable_text_state if enable_text_state is None else bool(enable_text_state)
        by_blocks = (io is not None and x.dtype == torch.bfloat16 and x.stride(-1) == 1 and self.shard is None and
                     self.precision != "fp8" and len(io.in_blocks) > 1)
        if io is not None and not by_blocks:
            io.wait_all(torch.cuda.current_stream(x.device))  # fp8 needs the whole tensor's scale
        if x.dtype != torch.bfloat16 or x.stride(-1) != 1:
            x = x.to(torch.bfloat16).contiguous()
        stream = _lib.stream_handle(x.device)
        ws = self.workspace(S, layout)
        linear_active = linear_enabled and not layout.full_cover and self.bw is not None and "bws" in ws
        q_act = None
        if linear_active:
            skip = layout.anchor_frames == "both"
            tpf = layout.tokens_per_frame
            Fb = layout.num_frames - 2 if skip else layout.num_frames
            r0 = layout.video_start + (tpf if skip else 0)
            if "q" not in self.short_conv and ws["bws"].tile_frames is None:
                # q's features need no conv: the QKV epilogue writes them (untiled branch)
                q_act = (ws["bws"].qf, r0, Fb * tpf, tpf)
        if by_blocks:
            # project each row block of x as soon as its copy has landed
            compute = torch.cuda.current_stream(x.device)
            for k, (r0b, r1b) in enumerate(io.bounds()):
                io.wait(compute, k)
                self._qkv(x, ws, status, stream, q_act, rows=(r0b, r1b))
        else:
            self._qkv(x, ws, status, stream, q_act)
        if linear_active:
            rows = slice(r0, r0 + Fb * tpf)
            bounds_b = [(lo - 1, hi - 1) for lo, hi in layout.bounds[1:-1]] if skip else list(layout.bounds)
            qkv, aux = ws["qkv"], ws["aux"]
            kw = dict(q_raw=qkv[rows, :g.inner], k_raw=qkv[rows, g.inner:2 * g.inner],
                      v_raw=qkv[rows, 2 * g.inner:], aux=aux[rows], beta_col0=self.col_beta, ogd_col0=self.col_ogd,
                      ad_col0=self.col_ad, Fb=Fb, tpf=tpf, frame_size=layout.frame_size, bounds=bounds_b,
                      bridge=bridge, out=ws["branch"], out_row0=r0, status=status, short_conv=self.short_conv,
                      delta_rule=self.delta_rule,
                      q_ready=q_act is not None)
            if enable_text_state and layout.text_len > 0:  # hybrid.py:449-451
                ts = slice(layout.text_start, layout.text_start + layout.text_len)
                kw.update(text_k=qkv[ts, g.inner:2 * g.inner], text_v=qkv[ts, 2 * g.inner:], text_aux=aux[ts])
            run_branch(ws["bws"], self.bw, **kw)
        # window softmax with the fused gate
        if layout.full_cover:
            plan = plans.get(S, 0, S, 1, S, [(0, 0)], "none")
        else:
            plan = plans.get(S, layout.video_start, layout.video_end, layout.num_frames, layout.tokens_per_frame,
                             layout.bounds, layout.anchor_frames)
        qkn, qkv = ws["qkn"], ws["qkv"]
        if rope is not None:
            # after the q / k RMSNorm of the QKV epilogue; the branch read the raw projections
            _lib.call("vdn_rope_split_half", qkn.data_ptr(), qkn.stride(0), S, 2 * g.heads, g.dim, rope.rot,
                      rope.freqs.data_ptr(), rope.ld, stream)
        if self.shard is not None:
            # the grouped operand of the sharded projection always spans the branch columns
            if linear_active:
                ws["branch_written"] = True
            elif ws["branch_written"]:
                ws["branch"].zero_()
                ws["branch_written"] = False
        attend = dict(gate_logits=ws["aux"] if self.enable_gate else None, gate_col0=self.col_gate,
                      gate_bias=self.gate_bias)
        operands = (qkn[:, :g.inner], qkn[:, g.inner:], qkv[:, 2 * g.inner:], ws["flat"], plan, g.heads, g.dim,
                    g.dim ** -0.5, status)
        xchg = ws.get("xchg") if issue_exchange else None
        if xchg is not None and xchg.chunks > 1:
            # the attention of consecutive row chunks in as many launches as keep at least
            # ATTN_ITEMS_PER_CTA items per CTA; each launch's chunks are exchanged behind it
            ends = [xchg.chunk_rows(c)[1] for c in range(xchg.chunks)]
            total = plan.n_qtiles * g.heads
            launches = max(1, min(xchg.chunks, total // (ATTN_ITEMS_PER_CTA * _sm_count(x.device))))
            for items, chunks in plan.device_chunk_groups(x.device, g.heads, ends, launches):
                if items.numel():
                    launch_window_attention(*operands, items=items, **attend)
                for c in chunks:
                    xchg.exchange_chunk(c)
        else:
            launch_window_attention(*operands, **attend)
        return ws, linear_active


class B200State:
    """Runtime state of one patched model on the B200 path (counterpart of VDNState,
    hybrid.py:33-150).  ``branches`` holds one weight mapping (or an object exposing it
    as ``.w``) per block.

    ``shard_heads``: False (one GPU per block), True (shard the heads over the default
    torch.distributed group, one process per GPU) or a process group to shard over.
    Every rank then runs the patched forward on the same x and gets the full output.
    ``shard_exchange``: "rows" (all-to-all of the per-head outputs by row block, each rank
    projects its rows, all-gather of the projected rows) or "heads" (all-gather of the
    per-head outputs, every rank projects every row)."""

    def __init__(self, name, config: Mapping, branches, num_heads, head_dim, *, attention_backend="b200",
                 projection_precision="bf16", inference=True, weight_maps=None, shard_heads=False, tile_frames=0,
                 shard_exchange="rows", **_ignored):
        if attention_backend not in ATTENTION_BACKENDS:
            raise ValueError(f"unsupported attention backend {attention_backend!r}")
        if projection_precision not in ("bf16", "fp8", "int8"):
            raise ValueError(f"unsupported projection precision {projection_precision!r}")
        self.name = str(name)
        self.config = dict(config)
        self.num_heads = int(num_heads)
        self.head_dim = int(head_dim)
        self.attention_backend = attention_backend
        self.projection_precision = projection_precision
        self.inference = bool(inference)
        if isinstance(tile_frames, bool) or not isinstance(tile_frames, int) or tile_frames < 0:
            raise ValueError("tile_frames must be a non-negative integer")  # nodes.py:247-248
        self.tile_frames = tile_frames  # the runtime's frame tiling (hybrid.py:51), for branches without their own
        self.shard_exchange = shard_exchange  # "rows" or "heads" (shard.EXCHANGES)
        maps = list(weight_maps) if weight_maps is not None else [
            b if isinstance(b, Mapping) else getattr(b, "w") for b in branches]
        self.branches = list(branches)
        self.weight_maps = maps
        self.window_plans = WindowPlanCache(limit=24)
        self.blocks: dict[int, FusedBlock] = {}
        self.workspaces: dict = {}  # shared by every block of the model
        self.status: dict[str, _lib.DeviceStatus] = {}
        self.forwards = 0
        self.last_attention_backend = None
        self.shard = None
        if shard_heads is not False and shard_heads is not None:
            self.shard = default_shard(self.num_heads, None if shard_heads is True else shard_heads)

    def device_status(self, device) -> _lib.DeviceStatus:
        key = str(device)
        if key not in self.status:
            self.status[key] = _lib.DeviceStatus(device)
        return self.status[key]

    def fused_block(self, attn, index, device) -> FusedBlock:
        fb = self.blocks.get(index)
        if fb is None:
            cfg = self.config
            # each setting from the block's branch object, else the node config, else the
            # reference default (nodes.py:98-116, hybrid.py:449-451)
            owner = self.branches[index] if index < len(self.branches) else None
            setting = {name: branch_setting(owner, cfg, name) for name in BRANCH_SETTING_DEFAULTS}
            tile = getattr(owner, "tile_frames", None) if not isinstance(owner, Mapping) else None
            fb = FusedBlock(_weight_of(attn.qkv_proj), _weight_of(attn.q_norm), _weight_of(attn.k_norm),
                            _weight_of(attn.out_proj), self.weight_maps[index], self.num_heads, self.head_dim,
                            device, precision=self.projection_precision, eps=float(getattr(attn.q_norm, "eps", 1e-6)),
                            enable_gate=bool(cfg.get("enable_softmax_gate", True)), shard=self.shard,
                            workspaces=self.workspaces, tile_frames=int(self.tile_frames if tile is None else tile),
                            exchange=self.shard_exchange, **setting)
            self.blocks[index] = fb
        return fb

    def release(self):
        self.blocks.clear()
        self.workspaces.clear()
        self.window_plans.clear()
        return self


def make_vdn_forward(attn, state: B200State, block_index: int):
    """Patched ``attn.forward`` (hybrid.py:409-579) running the sm_100a block."""
    original_forward = attn.forward
    heads, head_dim = int(attn.heads), int(attn.head_dim)
    if heads != state.num_heads or head_dim != state.head_dim:
        raise RuntimeError("attention geometry disagrees with the VDN state")
    config = state.config

    def vdn_forward(x, rope_freqs=None, transformer_options=None):
        layout = current_layout(required=False)
        if layout is None:
            return original_forward(x, rope_freqs=rope_freqs, transformer_options=transformer_options or {})
        if int(x.shape[0]) != layout.seq_len:
            raise RuntimeError(f"VDN layout has {layout.seq_len} rows but attention received {x.shape[0]}")
        _lib.require_cuda(x)
        rope = rope_table(rope_freqs, layout.seq_len, head_dim, x.device)
        status = state.device_status(x.device)
        block = state.fused_block(attn, block_index, x.device)
        # the branch settings were resolved when the block was built (B200State.fused_block)
        out = block.forward(x, layout, state.window_plans, status,
                            linear_enabled=bool(config.get("linear_enabled", True)),
                            io=(transformer_options or {}).get(STREAM_IO_KEY), rope=rope)
        state.last_attention_backend = "b200_dense" if layout.full_cover else "b200"
        return out.to(x.dtype)

    vdn_forward._vdn_h3_forward = True
    vdn_forward._vdn_h3_original = original_forward
    return vdn_forward


def run_forward_checked(state: B200State, fn, *args, **kwargs):
    """Run one model forward inside the deferred Cholesky scope and check the kernels'
    device status once at the end (the reference's layout wrapper, hybrid.py:216-241)."""
    with cholesky_runtime_scope():
        result = fn(*args, **kwargs)
    for st in state.status.values():
        st.raise_if_failed()
    return result


__all__ = ["BRANCH_SETTING_DEFAULTS", "B200State", "FusedBlock", "RopeTable", "branch_setting", "make_vdn_forward",
           "rope_table", "run_forward_checked"]
