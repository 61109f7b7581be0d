"""Block-sparse window softmax on sm_100a (replaces vdn_h3/window.py's backends).

``window_softmax_b200`` keeps the argument list of ``window_softmax_grouped``
(window.py:277-280) and its exact semantics (window.py:327-344), but runs one persistent
tcgen05 kernel over a host-built plan instead of per-group K/V gathers and SDPA calls.

Plan (built once per geometry, cached like the reference's ``_DecomposedPlan``,
window.py:726-797): query rows are cut into segments where they switch between seeing
every key (text rows, anchor-frame rows) and seeing a frame window, and each segment into
tiles of at most 256 rows; for each tile the key rows visible to any of its rows are merged
into intervals and cut into 128-key tiles that may start at any row.  A key tile carries a mask flag only when some row of the query
tile cannot see all of its keys; the kernel then rebuilds that row's visibility from
the frame index.  Work items (head, query tile) are sorted by key-tile count so the
persistent CTAs stay balanced.
"""

from __future__ import annotations

from collections import OrderedDict
from dataclasses import dataclass

import numpy as np
import torch

from . import _lib
from .layout import ANCHOR_FRAME_MODES, validate_layout

BQ = 256  # query rows per work item: two 128-row tiles that share every key tile
BKV = 128
# Planner cost model, in unmasked key-tile steps: a masked key tile (per-row visibility
# rebuilt in the softmax) and the fixed cost of one work item (Q load, epilogue, handoffs).
MASKED_TILE_COST = 1.1
ITEM_COST = 0.5
# Items at least this many times the median cost can be claimed first (None: plain head-major
# order, which measured slightly faster at config 1 once no query tile mixes dense and windowed rows).
LONG_ITEM_FACTOR = None
ATTENTION_BACKENDS = ("auto", "grouped", "flex", "flash2", "decomposed", "reference", "compat", "b200")


def _merge(intervals):
    out = []
    for a, b in sorted(i for i in intervals if i[0] < i[1]):
        if out and out[-1][1] >= a:
            out[-1] = (out[-1][0], max(out[-1][1], b))
        else:
            out.append((a, b))
    return out


def _contained(a, b, ivs) -> bool:
    return any(x <= a and b <= y for x, y in ivs)


@dataclass
class WindowPlan:
    seq_len: int
    video_start: int
    video_end: int
    num_frames: int
    tokens_per_frame: int
    anchor_rows: bool
    anchor_cols: bool
    frame_lo: np.ndarray  # [F] int32, clamped
    frame_hi: np.ndarray  # [F] int32, clamped
    tile_off: np.ndarray  # [nq + 1] int32
    qtile: np.ndarray  # [nq, 2] int32 per 128-row half: (row0 << 8) | rows (0 rows: empty half)
    ktile: np.ndarray  # [n_ktiles] int32 packed (k0 << 9) | (masked << 8) | (valid - 1)
    tiles_per_q: np.ndarray  # [nq]
    masked_tiles: int
    _device: dict | None = None

    @property
    def n_qtiles(self) -> int:
        return len(self.tiles_per_q)

    def q_halves(self, qt: int) -> list[tuple[int, int]]:
        """[(first row, row count)] of the non-empty 128-row halves of query tile ``qt``."""
        out = []
        for a in range(2):
            code = int(self.qtile[qt, a])
            if code & 0xFF:
                out.append((code >> 8, code & 0xFF))
        return out

    def items(self, heads: int, long_factor: float | None = None) -> np.ndarray:
        """(head << 20) | q_tile in claim order: head-major (the CTAs in flight share one
        head's K/V in L2), the most expensive first within a head.  With a ``long_factor``
        (default ``LONG_ITEM_FACTOR``), the long items (query tiles whose rows see at least
        that many times the median number of key tiles: text rows and anchor frames) of all
        heads come first, head by head, so none of them starts near the end of the queue."""
        long_factor = LONG_ITEM_FACTOR if long_factor is None else long_factor
        cost = self.tiles_per_q.astype(np.int64)
        order = np.argsort(-cost, kind="stable")
        if long_factor is None:
            long_q = np.zeros(len(cost), dtype=bool)
        else:
            long_q = cost >= long_factor * max(float(np.median(cost)), 1.0)
        hs = np.arange(heads, dtype=np.int64)
        first = [(h << 20) | q for h in hs for q in order if long_q[q]]
        rest = [(h << 20) | q for h in hs for q in order if not long_q[q]]
        return np.asarray(first + rest, dtype=np.int64).astype(np.int32)

    def chunk_items(self, heads: int, ends) -> list[np.ndarray]:
        """``items(heads)`` split into consecutive row chunks ending at ``ends`` (ascending,
        the last one the sequence length), keeping the claim order inside each: a query tile
        goes with the chunk of its first row, so once the launches of chunks 0..c are done
        every row before ``ends[c]`` is final (a tile reaching into a later chunk only
        finishes those rows early)."""
        first_row = np.array([min(r0 for r0, _ in self.q_halves(q)) for q in range(self.n_qtiles)], dtype=np.int64)
        chunk_of = np.searchsorted(np.asarray(ends, dtype=np.int64), first_row, side="right")
        items = self.items(heads)
        owner = chunk_of[items & 0xFFFFF]
        return [items[owner == c] for c in range(len(ends))]

    def key_tiles_total(self, heads: int) -> int:
        return int(self.tiles_per_q.sum()) * heads

    def device_arrays(self, device, heads: int) -> dict:
        key = (str(device), heads)
        if self._device is None:
            self._device = {}
        if key not in self._device:
            dev = torch.device(device)
            self._device[key] = {
                "frame_lo": torch.from_numpy(self.frame_lo).to(dev),
                "frame_hi": torch.from_numpy(self.frame_hi).to(dev),
                "tile_off": torch.from_numpy(self.tile_off).to(dev),
                "qtile": torch.from_numpy(np.ascontiguousarray(self.qtile.reshape(-1))).to(dev),
                "ktile": torch.from_numpy(self.ktile).to(dev),
                "items": torch.from_numpy(self.items(heads)).to(dev),
            }
        return self._device[key]

    def device_chunk_items(self, device, heads: int, ends) -> list[torch.Tensor]:
        """``chunk_items`` on the device (cached per chunk boundaries)."""
        d = self.device_arrays(device, heads)
        key = ("chunks", tuple(int(e) for e in ends))
        if key not in d:
            d[key] = [torch.from_numpy(np.ascontiguousarray(it)).to(torch.device(device))
                      for it in self.chunk_items(heads, ends)]
        return d[key]

    def chunk_groups(self, heads: int, ends, launches: int) -> list[tuple[np.ndarray, range]]:
        """``chunk_items`` merged into ``launches`` runs of consecutive chunks (as even as the
        chunk count allows): each run's items, in chunk order, and the chunks it covers.  One
        launch per run keeps enough items per CTA for the persistent grid to balance its tail,
        while the collectives of a run's chunks still start as soon as that run is done."""
        per = self.chunk_items(heads, ends)
        n = len(per)
        runs = max(1, min(int(launches), n))
        bounds = [(n * k) // runs for k in range(runs + 1)]
        return [(np.concatenate(per[a:b]).astype(np.int32) if b > a else np.zeros(0, np.int32), range(a, b))
                for a, b in zip(bounds, bounds[1:])]

    def device_chunk_groups(self, device, heads: int, ends, launches: int) -> list[tuple[torch.Tensor, range]]:
        """``chunk_groups`` on the device (cached per chunk boundaries and launch count)."""
        d = self.device_arrays(device, heads)
        key = ("groups", tuple(int(e) for e in ends), int(launches))
        if key not in d:
            d[key] = [(torch.from_numpy(np.ascontiguousarray(it)).to(torch.device(device)), r)
                      for it, r in self.chunk_groups(heads, ends, launches)]
        return d[key]


HALF = BQ // 2  # rows per MMA half of a work item


def _pair_short_tiles(q_tiles, keys):
    """Query tiles as two 128-row halves [(first row, rows), (first row, rows)]; tiles of at
    most 128 rows whose key tiles are identical (the partial tiles at the ends of the
    every-key segments before and after the video) share one work item, one per half."""
    halves, out_keys, waiting = [], [], {}
    for (r0, r1), kc in zip(q_tiles, keys):
        n = r1 - r0
        if n > HALF:
            halves.append([(r0, HALF), (r0 + HALF, n - HALF)])
            out_keys.append(kc)
            continue
        sig = tuple(kc[0])
        if sig in waiting:
            i = waiting.pop(sig)
            halves[i][1] = (r0, n)
        else:
            waiting[sig] = len(halves)
            halves.append([(r0, n), (r0, 0)])  # an empty second half keeps a valid first row
            out_keys.append(kc)
    return halves, out_keys


def build_window_plan(seq_len, video_start, video_end, num_frames, tokens_per_frame, bounds,
                      anchor_frames, cutting: str = "auto") -> WindowPlan:
    """``cutting``: "class" cuts query tiles at every change of the rows' visible keys,
    "dense" only where rows switch between seeing every key and a window, "auto" keeps the
    cheaper of the two under the planner's cost model."""
    if cutting not in ("auto", "class", "dense"):
        raise ValueError(f"unknown cutting {cutting!r}")
    validate_layout(seq_len, video_start, video_end, num_frames, tokens_per_frame, bounds, anchor_frames)
    S, vs, ve, F, tpf = int(seq_len), int(video_start), int(video_end), int(num_frames), int(tokens_per_frame)
    a_rows = anchor_frames in ("rows", "both")
    a_cols = anchor_frames in ("columns", "both")
    last = F - 1
    lo = np.array([max(int(b[0]), 0) for b in bounds], dtype=np.int32)
    hi = np.array([min(int(b[1]), last) for b in bounds], dtype=np.int32)
    cls_cache: dict[int, list] = {}

    def class_iv(c):
        if c not in cls_cache:
            if c < 0:
                cls_cache[c] = [(0, S)]
            else:
                iv = [(0, vs), (ve, S), (vs + int(lo[c]) * tpf, vs + (int(hi[c]) + 1) * tpf)]
                if a_cols:
                    iv += [(vs, vs + tpf), (ve - tpf, ve)]
                cls_cache[c] = _merge(iv)
        return cls_cache[c]

    def row_class(f):
        """Visible-key class of the rows of frame ``f``: -1 (every key) or its frame window."""
        return -1 if (a_rows and f in (0, last)) else (int(lo[f]), int(hi[f]))

    def tile_keys(r0, r1):
        """Key tiles of query rows [r0, r1): (packed codes, number of masked tiles)."""
        classes = set()
        if r0 < vs or r1 > ve:
            classes.add(-1)
        a, b = max(r0, vs), min(r1, ve)
        if a < b:
            for f in range((a - vs) // tpf, (b - 1 - vs) // tpf + 1):
                classes.add(-1 if row_class(f) == -1 else f)
        ivs = {c: class_iv(c) for c in classes}
        union = _merge([iv for c in classes for iv in ivs[c]])
        codes, n_masked = [], 0
        for x, y in union:
            for k0 in range(x, y, BKV):
                kend = min(k0 + BKV, y)
                m = any(not _contained(k0, kend, ivs[c]) for c in classes)
                n_masked += int(m)
                codes.append((k0 << 9) | (int(m) << 8) | (kend - k0 - 1))
        if not codes:
            raise ValueError(f"query rows [{r0}, {r1}) see no keys")
        return codes, n_masked

    # Row runs of one visible-key class: text rows and anchor-frame rows see every key;
    # consecutive frames with the same window (chunked windows) share a class.
    runs = [0]
    prev = -1 if vs > 0 else None
    for f in range(F):
        c = row_class(f)
        if c != prev:
            runs.append(vs + f * tpf)
            prev = c
    if ve < S and prev != -1:
        runs.append(ve)
    runs = sorted(set(runs) | {S})
    # Two cuttings of the rows into query tiles: at every class change (no masked key tiles,
    # but a partial tile per run), or only where rows switch between seeing every key and a
    # window (tiles may straddle frames and mask some keys).  The cheaper one is kept.
    dense_cuts = {0, S}
    for r0, r1 in zip(runs, runs[1:]):
        f = (r0 - vs) // tpf if vs <= r0 < ve else None
        dense = f is None or row_class(f) == -1
        prev_dense = r0 == 0 or (r0 - 1 < vs or r0 - 1 >= ve or row_class((r0 - 1 - vs) // tpf) == -1)
        if dense != prev_dense:
            dense_cuts.add(r0)
    candidates = {"class": [runs], "dense": [sorted(dense_cuts)], "auto": [runs, sorted(dense_cuts)]}[cutting]
    best = None
    for cuts in candidates:
        q_tiles = [(r0, min(b, r0 + BQ)) for a, b in zip(cuts, cuts[1:]) for r0 in range(a, b, BQ)]
        keys = [tile_keys(r0, r1) for r0, r1 in q_tiles]
        halves, keys = _pair_short_tiles(q_tiles, keys)
        cost = sum(len(c) + (MASKED_TILE_COST - 1.0) * m + ITEM_COST for c, m in keys)
        if best is None or cost < best[0]:
            best = (cost, halves, keys)
    _, halves, keys = best
    nq = len(halves)
    tile_off = np.zeros(nq + 1, dtype=np.int64)
    tile_off[1:] = np.cumsum([len(c) for c, _ in keys])
    qtile = np.array([[(r0 << 8) | n for r0, n in hv] for hv in halves], dtype=np.int64).reshape(nq, 2)
    ktiles = np.asarray([code for c, _ in keys for code in c], dtype=np.int64)
    tiles_per_q = np.array([len(c) for c, _ in keys], dtype=np.int64)
    masked = int(sum(m for _, m in keys))
    return WindowPlan(S, vs, ve, F, tpf, a_rows, a_cols, lo, hi, tile_off.astype(np.int32), qtile.astype(np.int32),
                      ktiles.astype(np.int32), tiles_per_q, masked)


class WindowPlanCache:
    """LRU of plans, owned by one state object (window.py:77-138 keeps plans per model)."""

    def __init__(self, limit: int = 16):
        self.limit = int(limit)
        self._plans: OrderedDict = OrderedDict()

    def get(self, seq_len, video_start, video_end, num_frames, tokens_per_frame, bounds, anchor_frames):
        key = (int(seq_len), int(video_start), int(video_end), int(num_frames), int(tokens_per_frame),
               tuple((int(a), int(b)) for a, b in bounds), str(anchor_frames))
        plan = self._plans.get(key)
        if plan is None:
            plan = build_window_plan(*key)
            self._plans[key] = plan
            while len(self._plans) > self.limit:
                self._plans.popitem(last=False)
        else:
            self._plans.move_to_end(key)
        return plan

    def clear(self):
        self._plans.clear()

    release = clear


_DEFAULT_PLANS = WindowPlanCache()


def _rows_view(t: torch.Tensor, heads: int, dim: int) -> int:
    """Row pitch of a [S, H, D] view whose heads and dims are packed (row-major [S, H*D])."""
    if t.dtype != torch.bfloat16:
        raise ValueError("window attention operands must be bfloat16")
    if t.stride(-1) != 1 or t.stride(-2) != dim:
        raise ValueError("q/k/v must have contiguous [heads, dim] inner layout")
    return t.stride(0)


def launch_window_attention(q, k, v, out, plan: WindowPlan, heads, dim, scale, status: _lib.DeviceStatus,
                            gate_logits=None, gate_col0=0, gate_bias=None, items: torch.Tensor | None = None):
    """Launch the kernel on the current stream (no validation beyond the C-ABI's).
    ``items``: a device subset of the work items (one row chunk, ``device_chunk_items``)."""
    d = plan.device_arrays(q.device, heads)
    if items is None:
        items = d["items"]
    n_items = int(items.numel())
    _lib.call(
        "vdn_window_attention",
        q.data_ptr(), q.stride(0), k.data_ptr(), k.stride(0), v.data_ptr(), v.stride(0),
        plan.seq_len, heads, dim, plan.video_start, plan.video_end, plan.num_frames, plan.tokens_per_frame,
        int(plan.anchor_rows), int(plan.anchor_cols), float(scale),
        d["frame_lo"].data_ptr(), d["frame_hi"].data_ptr(), items.data_ptr(), n_items,
        d["tile_off"].data_ptr(), d["qtile"].data_ptr(), d["ktile"].data_ptr(), out.data_ptr(), out.stride(0),
        _lib.ptr(gate_logits), gate_logits.stride(0) if gate_logits is not None else 0, int(gate_col0),
        _lib.ptr(gate_bias), status.counter_ptr, status.err_ptr, _lib.stream_handle(q.device),
    )


def window_softmax_b200(query, key, value, video_start, video_end, num_frames, tokens_per_frame, bounds, scale,
                        anchor_frames="none", *, gate=None, cache: WindowPlanCache | None = None,
                        status: _lib.DeviceStatus | None = None):
    """Exact window softmax attention, same contract as window_softmax_grouped
    (window.py:277-313).  ``query/key/value``: [S, H, D] bf16 CUDA tensors (strided row
    views of a fused projection are accepted).  ``gate`` optionally fuses the per-token
    head gate: a tuple (logits [S, >=H] fp32 view, bias [H] fp32 or None); the result is
    then ``softmax_out * sigmoid(logits + bias)``.  Returns [S, H, D] bf16.
    """
    if query.ndim != 3 or query.shape != key.shape or query.shape != value.shape:
        raise ValueError("query, key and value must share shape [sequence, heads, dim]")
    _lib.require_cuda(query, key, value)
    S, H, D = query.shape
    plan = (cache or _DEFAULT_PLANS).get(S, video_start, video_end, num_frames, tokens_per_frame, bounds,
                                         anchor_frames)
    for t in (query, key, value):
        _rows_view(t, H, D)
    out = torch.empty(S, H, D, device=query.device, dtype=torch.bfloat16)
    st = status or _lib.DeviceStatus(query.device)
    logits, bias, col0 = None, None, 0
    if gate is not None:
        logits, bias = gate
        if logits.dtype != torch.float32 or logits.stride(-1) != 1:
            raise ValueError("gate logits must be an fp32 row-major view")
        col0 = 0
    launch_window_attention(query, key, value, out, plan, H, D, scale, st, logits, col0, bias)
    if status is None:
        st.raise_if_failed()
    return out


__all__ = [
    "ANCHOR_FRAME_MODES",
    "ATTENTION_BACKENDS",
    "WindowPlan",
    "WindowPlanCache",
    "build_window_plan",
    "launch_window_attention",
    "window_softmax_b200",
]
