"""Video Delta Attention branch on sm_100a (replaces vdn_h3/branch.py + vdn_h3/runtime.py).

``B200LinearBranch`` keeps the reference's constructor knobs (delta_rule, bridge,
a_fp32, short_conv, enable_text_state) and its two entry points:

* ``readout(weights, xv, q_raw, k_raw, v_raw, num_frames, tokens_per_frame, bounds,
  frame_size, text_x, text_k_raw, text_v_raw, skip_ends, *, inference)``
  (branch.py:672-722), returning the branch output before ``to_out_linear``;
* ``projected_delta(..., projector=None)`` (runtime.py:545-607), returning it after.

Both run the same kernel sequence as the fused block (``run_branch``): features, alpha,
frame statistics (+ the text frame), the delta factor, the fused bidirectional scan and the
gather/readout/RMSNorm/gate kernel.  Both delta rules of branch.py:180 run on the device:
``vdn_solve`` (the released lineage, docs/ARCHITECTURE.md:70-82: Cholesky-checked inverse
of I + A) and ``sana_scaled`` (M = I - A/L, injection B/sqrt(L)); the bridge is ``alpha``
or ``none``.
"""

from __future__ import annotations

from contextlib import contextmanager
from contextvars import ContextVar
from dataclasses import dataclass

import torch

from . import _lib

TEXT_STATE_SCALE = 0.5  # branch.py:23
DELTA_RULES = ("vdn_solve", "sana_scaled")  # branch.py:180
_CHOLESKY_CHECKS: ContextVar = ContextVar("vdn_b200_cholesky_checks", default=None)


class InfoRing:
    """Status rows for the factor calls of one branch workspace: each call gets a [rows, H]
    int32 slot of its own (the reference gets a fresh ``info`` from every ``cholesky_ex``,
    branch.py:62-71), so blocks that share a workspace cannot overwrite a status before the
    forward validates it.  Slots come from chunks allocated on first need and return to the
    free list once their scope has validated them; after the first forward no call
    allocates."""

    CHUNK = 16

    def __init__(self, rows: int, heads: int, device):
        self.shape = (int(rows), int(heads))
        self.device = torch.device(device)
        self.chunks: list[torch.Tensor] = []
        self.free: list[torch.Tensor] = []

    def claim(self) -> torch.Tensor:
        if not self.free:
            chunk = torch.zeros(self.CHUNK, *self.shape, device=self.device, dtype=torch.int32)
            self.chunks.append(chunk)
            self.free = [chunk[i] for i in range(self.CHUNK - 1, -1, -1)]
        return self.free.pop()

    def release(self, slot: torch.Tensor):
        self.free.append(slot)


class _CholeskyChecks:
    """Deferred SPD validation of every factorisation of one forward (branch.py:27-45)."""

    def __init__(self):
        self.statuses: list[torch.Tensor] = []
        self.factor_calls = 0
        self.claims: list[tuple[InfoRing, torch.Tensor]] = []

    def release(self):
        for ring, slot in self.claims:
            ring.release(slot)
        self.claims.clear()

    def validate(self):
        if not self.statuses:
            return
        flat = torch.cat([s.reshape(-1) for s in self.statuses])
        bad = torch.nonzero(flat != 0)
        if bad.numel():
            failed = int(bad[0].item())
            for index, status in enumerate(self.statuses):
                if failed < status.numel():
                    minor = int(status.reshape(-1)[failed].item())
                    raise torch.linalg.LinAlgError(
                        f"VDN-H3 Cholesky factor {index}, batch {failed}: "
                        f"leading minor of order {minor} is not positive-definite")
                failed -= status.numel()


@contextmanager
def cholesky_runtime_scope():
    """Collect factor statuses and validate them once when the scope exits (branch.py:48-59)."""
    checks = _CholeskyChecks()
    token = _CHOLESKY_CHECKS.set(checks)
    try:
        yield checks
        checks.validate()
    finally:
        checks.statuses.clear()
        checks.release()
        _CHOLESKY_CHECKS.reset(token)


def claim_factor_status(ring: InfoRing) -> torch.Tensor:
    """A status slot for one branch call's factorisations (text frame and clip frames),
    held until the enclosing scope has validated it (outside a scope: until the call's own
    immediate validation)."""
    slot = ring.claim()
    checks = _CHOLESKY_CHECKS.get()
    if checks is not None:
        checks.claims.append((ring, slot))
    return slot


def record_factor_status(infos: list[torch.Tensor], ring: InfoRing | None = None,
                         slot: torch.Tensor | None = None):
    """Register the status rows of one call's factorisations, in the order the reference
    factors them (the text frame's, then the clip's: branch.py:795-799), for validation:
    deferred to the exit of ``cholesky_runtime_scope`` (branch.py:48-59), else validated now
    (a host sync), ``slot`` going back to ``ring`` afterwards."""
    checks = _CHOLESKY_CHECKS.get()
    if checks is None:
        tmp = _CholeskyChecks()
        tmp.statuses.extend(infos)
        tmp.factor_calls = len(infos)
        try:
            tmp.validate()
        finally:
            if ring is not None and slot is not None:
                ring.release(slot)
    else:
        checks.statuses.extend(infos)
        checks.factor_calls += len(infos)


@dataclass
class BranchDeviceWeights:
    """Branch weights in the layouts the kernels read (fp32 for the small tensors,
    matching the reference's fp32 policy for A_log/dt_bias, weights.py)."""

    heads: int
    dim: int
    og_up: torch.Tensor  # [H*D, D] bf16
    og_bias: torch.Tensor  # [H*D] fp32
    alpha_up: torch.Tensor  # [H*D, D] fp32
    dt_bias: torch.Tensor  # [H*D] fp32
    a_log: torch.Tensor  # [H] fp32
    norm_w: torch.Tensor  # [D] fp32
    conv: dict  # name -> (spatial [C, kh*kw] fp32, kh, kw, temporal [C, taps] fp32, taps)
    beta_w: torch.Tensor  # [H, hidden] bf16
    og_down: torch.Tensor  # [D, hidden] bf16
    alpha_down: torch.Tensor  # [D, hidden] bf16
    to_out: torch.Tensor | None  # [hidden, H*D] bf16

    @staticmethod
    def from_dict(w: dict, heads: int, dim: int, device, head_slice: slice | None = None,
                  short_conv=("k", "v")) -> "BranchDeviceWeights":
        dev = torch.device(device)
        hs = head_slice or slice(0, heads)
        h0, h1 = hs.start, hs.stop
        cs = slice(h0 * dim, h1 * dim)

        def f32(t):
            return t.detach().to(dev, torch.float32).contiguous()

        def b16(t):
            return t.detach().to(dev, torch.bfloat16).contiguous()

        conv = {}
        for name in short_conv:
            sp = w[f"short_conv.{name}_sp.weight"][cs]
            tm = w[f"short_conv.{name}_tm.weight"][cs]
            kh, kw = int(sp.shape[-2]), int(sp.shape[-1])
            conv[name] = (f32(sp.reshape(sp.shape[0], -1)), kh, kw, f32(tm.reshape(tm.shape[0], -1)),
                          int(tm.shape[-1]))
        to_out = w.get("to_out_linear.weight")
        return BranchDeviceWeights(
            heads=h1 - h0, dim=dim,
            og_up=b16(w["output_gate.up.weight"][cs]),
            og_bias=f32(w.get("output_gate.up.bias", torch.zeros(heads * dim))[cs]),
            alpha_up=f32(w["alpha.up.weight"][cs]),
            dt_bias=f32(w["alpha.dt_bias"][cs]),
            a_log=f32(w["alpha.A_log"][hs]),
            norm_w=f32(w["norm.weight"]),
            conv=conv,
            beta_w=b16(w["beta_proj.weight"][hs]),
            og_down=b16(w["output_gate.down.weight"]),
            alpha_down=b16(w["alpha.down.weight"]),
            to_out=b16(to_out) if to_out is not None and not isinstance(to_out, tuple) else None,
        )


class BranchWorkspace:
    """Device buffers of one branch geometry, reused across calls.  ``tile_frames`` (the
    frame-tiled low-memory mode of runtime.py:421-543): the per-row feature buffers hold one
    tile plus its temporal halo (``TILE_HALO`` frames each side) instead of the whole clip;
    the per-frame matrices always cover the clip."""

    def __init__(self, device, Fb, tpf, heads, dim, text_len, tile_frames=None):
        dev = torch.device(device)
        inner = heads * dim
        tile = feature_frames(Fb, tile_frames)
        rows = tile * tpf
        bf = dict(device=dev, dtype=torch.bfloat16)
        f32 = dict(device=dev, dtype=torch.float32)
        self.key = (str(dev), Fb, tpf, heads, dim, text_len, tile_frames)
        self.tile_frames = tile_frames
        self.feature_frames = tile
        self._conv_shape = (rows, inner)
        self._conv_tmp = None  # the spatial conv's output, for the two-kernel path only
        self.qf = torch.empty(tile, heads, tpf, dim, **bf)
        self.kf = torch.empty(tile, heads, tpf, dim, **bf)
        self.vf = torch.empty(tile, heads, tpf, dim, **bf)
        nt = 1 if text_len > 0 else 0
        self.tk = torch.empty(1, heads, max(text_len, 1), dim, **bf)
        self.tv = torch.empty(1, heads, max(text_len, 1), dim, **bf)
        self.alpha = torch.empty(Fb, heads, dim, **f32)
        self.A = torch.empty(Fb + nt, heads, dim, dim, **f32)
        self.B = torch.empty(Fb + nt, heads, dim, dim, **f32)
        self.inv = torch.empty(Fb + nt, heads, dim, dim, **f32)
        # bf16 hi / lo halves of the inverses for the tensor-core scan (head_dim 128)
        self.inv_split = torch.empty(2 if dim == 128 else 0, Fb + nt, heads, dim, dim, **bf)
        self.info_ring = InfoRing(Fb + nt, heads, dev)  # one [Fb + nt, H] status slot per call
        self.s0 = torch.empty(heads, dim, dim, **f32)
        self.prefix = torch.empty(Fb, heads, dim, dim, **f32)
        self.suffix = torch.empty(Fb, heads, dim, dim, **f32)
        self.ogd = torch.empty(rows, dim, **bf)
        # the output gate is materialised only on the head_dim-64 path (128 fuses it into the readout)
        self.og = torch.empty(rows if dim != 128 else 0, inner, **bf)
        self.lohi: dict = {}
        self._side = None

    def conv_buffer(self) -> torch.Tensor:
        """[rows, H*D] bf16 spatial-conv output of the two-kernel feature path (allocated on
        first use: the fused path never needs it)."""
        if self._conv_tmp is None:
            self._conv_tmp = torch.empty(*self._conv_shape, device=self.alpha.device, dtype=torch.bfloat16)
        return self._conv_tmp

    def side_stream(self) -> torch.cuda.Stream:
        """The stream the text state runs on, beside the frames' kernels."""
        if self._side is None:
            self._side = torch.cuda.Stream(self.alpha.device)
        return self._side

    def bounds_arrays(self, bounds):
        key = tuple(bounds)
        if key not in self.lohi:
            dev = self.alpha.device
            lo = torch.tensor([int(b[0]) for b in bounds], dtype=torch.int32, device=dev)
            hi = torch.tensor([int(b[1]) for b in bounds], dtype=torch.int32, device=dev)
            self.lohi[key] = (lo, hi)
        return self.lohi[key]


TILE_HALO = 2  # frames each side: the 5-tap temporal conv's reach (runtime.py:428-430)
# Short conv features in one kernel (vdn_conv_features) where its geometry allows.  Off: on
# the config-1 clip (38 x 22 frames, H = 40) the fused kernel, bound by its one-frame-deep
# prefetch and one 256-thread CTA per SM, measured 1.78 ms per forward for k and v against
# 1.03 ms for the spatial + temporal pair (0.78 ms since their rewrite), which keep more
# warps busy per SM.
FUSED_CONV = False


def fused_conv_ok(src: torch.Tensor, kh: int, kw: int, taps: int, dim: int) -> bool:
    """Whether ``vdn_conv_features`` takes these features (5x5 spatial, 5-tap temporal, head
    dim 64 or 128, 16-byte aligned rows); otherwise the spatial and temporal kernels run."""
    return (FUSED_CONV and kh == 5 and kw == 5 and taps == 5 and dim in (64, 128) and src.data_ptr() % 16 == 0
            and src.stride(0) % 8 == 0 and src.stride(-1) == 1)


def frame_tiles(Fb: int, tile_frames) -> list[tuple[int, int]]:
    """[start, stop) frame tiles of a clip of Fb frames (one tile when ``tile_frames`` is None
    or covers the clip), as runtime.py:452-453 / :516-517 step them."""
    if tile_frames is None or int(tile_frames) >= Fb:
        return [(0, Fb)]
    t = int(tile_frames)
    if t <= 0:
        raise ValueError("tile_frames must be positive")
    return [(a, min(Fb, a + t)) for a in range(0, Fb, t)]


def feature_frames(Fb: int, tile_frames) -> int:
    """Frames a feature buffer holds: the clip, or the largest tile plus its halo."""
    tiles = frame_tiles(Fb, tile_frames)
    if len(tiles) == 1:
        return Fb
    return min(Fb, max(b - a for a, b in tiles) + 2 * TILE_HALO)


def run_branch(ws: BranchWorkspace, bw: BranchDeviceWeights, *, q_raw, k_raw, v_raw, aux, beta_col0, ogd_col0,
               ad_col0, Fb, tpf, frame_size, bounds, bridge, text_k=None, text_v=None, text_aux=None,
               out, out_row0, status: _lib.DeviceStatus, short_conv=("k", "v"), q_ready=False,
               delta_rule="vdn_solve"):
    """Run the branch kernels on the current stream.

    q_raw / k_raw / v_raw: [Fb*tpf, H*D] bf16 row views (pitch = stride(0)) of the raw
    projections of the branch frames; aux: [Fb*tpf, *] fp32 rows holding the beta logits
    (column beta_col0 + h), the output-gate bottleneck (ogd_col0 + j) and the alpha
    bottleneck (ad_col0 + j); text_k / text_v / text_aux: the same for the text rows.
    Writes out[out_row0 + f*tpf + s, h*D + v] (bf16).  q_ready: ws.qf already holds the q
    features of every frame (written by the QKV epilogue).  delta_rule: "vdn_solve" (inverse
    of I + A, injection folded before the product) or "sana_scaled" (M = I - A/tpf, injection
    B/sqrt(tpf) added after it; text state 0.5 B/sqrt(text_len), no factorisation).
    With ``ws.tile_frames`` the clip runs in frame tiles (runtime.py:421-543): features,
    statistics and alpha per tile (the conv'd features with a 2-frame halo each side), the
    factor and the scans over the clip, then features, gate and readout per tile; the result
    is the same as one tile.
    """
    if delta_rule not in DELTA_RULES:
        raise ValueError(f"unknown delta rule: {delta_rule!r}")
    H, D = bw.heads, bw.dim
    inner = H * D
    stream = _lib.stream_handle(out.device)
    gh, gw = frame_size
    call = _lib.call
    tiles = frame_tiles(Fb, ws.tile_frames)
    if q_ready and len(tiles) > 1:
        raise ValueError("q features written by the QKV epilogue need the untiled branch")
    fhsd = H * tpf * D  # elements of one frame of a feature buffer

    def feature(raw, name, dst, l2, a, b):
        """Features of clip frames [a, b) into dst; returns the offset (in frames) of frame a
        inside dst (the conv'd features are computed over a halo that the tile discards)."""
        conv = name in bw.conv and name in short_conv
        ha, hb = (max(0, a - TILE_HALO), min(Fb, b + TILE_HALO)) if conv and len(tiles) > 1 else (a, b)
        src = raw[ha * tpf:hb * tpf]
        nf = hb - ha
        if conv:
            sp, kh, kw, tm, taps = bw.conv[name]
            if fused_conv_ok(src, kh, kw, taps, D):
                # spatial + temporal conv, SiLU and L2 in one pass (no intermediate in HBM)
                call("vdn_conv_features", src.data_ptr(), src.stride(0), sp.data_ptr(), kh, kw, tm.data_ptr(), taps,
                     nf, gh, gw, H, D, int(l2), dst.data_ptr(), stream)
                return a - ha
            conv_tmp = ws.conv_buffer()
            call("vdn_spatial_conv", src.data_ptr(), src.stride(0), sp.data_ptr(), kh, kw, nf, gh, gw, inner,
                 conv_tmp.data_ptr(), conv_tmp.stride(0), stream)
            call("vdn_temporal_act", conv_tmp.data_ptr(), conv_tmp.stride(0), tm.data_ptr(), taps, nf, tpf,
                 H, D, int(l2), dst.data_ptr(), stream)
        else:
            call("vdn_temporal_act", src.data_ptr(), src.stride(0), None, 0, nf, tpf, H, D, int(l2), dst.data_ptr(),
                 stream)
        return a - ha

    aux_ld = aux.stride(0)
    tensor_cores = D == 128  # the tcgen05 statistics/readout kernels are written for head_dim 128

    def stats(kf_ptr, vf_ptr, F_, T_, beta, beta_row0, A_ptr, B_ptr, st=stream):
        bp = beta.data_ptr() + 4 * beta_row0 * beta.stride(0)
        if tensor_cores:
            call("vdn_frame_stats_tc", kf_ptr, vf_ptr, F_, H, T_, bp, beta.stride(0), beta_col0, A_ptr, B_ptr,
                 status.err_ptr, st)
        else:
            call("vdn_frame_stats", kf_ptr, vf_ptr, F_, H, T_, D, bp, beta.stride(0), beta_col0, A_ptr, B_ptr, st)

    has_text = text_k is not None
    s0 = ws.s0 if has_text else None
    mat = D * D * H
    # this call's factor status rows: [Fb] clip frames then the text frame
    info = claim_factor_status(ws.info_ring) if delta_rule == "vdn_solve" else None
    # The text "frame" (its features, statistics, factor and S0) and alpha (launches of 30 to
    # 40-odd CTAs, latency-bound) run on a side stream beside the frames' conv, statistics and
    # factor; the scan waits for them.  Their inputs were written before this call on the
    # caller's stream.
    main = torch.cuda.current_stream(out.device)
    side = ws.side_stream()
    side.wait_stream(main)
    ts = side.cuda_stream
    for a, b in tiles:
        call("vdn_alpha_gate", aux.data_ptr() + 4 * (ad_col0 + a * tpf * aux_ld), aux_ld, b - a, tpf, D,
             bw.alpha_up.data_ptr(), bw.dt_bias.data_ptr(), bw.a_log.data_ptr(), H, D,
             ws.alpha.data_ptr() + 4 * a * H * D, ts)
    if has_text:
        L = text_k.shape[0]
        call("vdn_temporal_act", text_k.data_ptr(), text_k.stride(0), None, 0, 1, L, H, D, 1, ws.tk.data_ptr(), ts)
        call("vdn_temporal_act", text_v.data_ptr(), text_v.stride(0), None, 0, 1, L, H, D, 0, ws.tv.data_ptr(), ts)
        stats(ws.tk.data_ptr(), ws.tv.data_ptr(), 1, L, text_aux, 0, ws.A.data_ptr() + 4 * Fb * mat,
              ws.B.data_ptr() + 4 * Fb * mat, st=ts)
        if delta_rule == "sana_scaled":
            # S0 = 0.5 * B / sqrt(L): no factor of the text matrix is needed
            call("vdn_sana_factor", ws.A.data_ptr() + 4 * Fb * mat, ws.B.data_ptr() + 4 * Fb * mat, 1, H, D, 1.0 / L,
                 None, None, 0, (1.0 / L) ** 0.5, TEXT_STATE_SCALE, ws.s0.data_ptr(), ts)
        else:
            call("vdn_delta_factor", ws.A.data_ptr() + 4 * Fb * mat, ws.B.data_ptr() + 4 * Fb * mat, 1, H, D,
                 ws.inv.data_ptr() + 4 * Fb * mat, info.data_ptr() + 4 * Fb * H, 0, TEXT_STATE_SCALE,
                 ws.s0.data_ptr(), None, ts)
    side_done = torch.cuda.Event()
    side_done.record(side)

    for a, b in tiles:
        ok = feature(k_raw, "k", ws.kf, True, a, b)
        ov = feature(v_raw, "v", ws.vf, False, a, b)
        stats(ws.kf.data_ptr() + 2 * ok * fhsd, ws.vf.data_ptr() + 2 * ov * fhsd, b - a, tpf, aux, a * tpf,
              ws.A.data_ptr() + 4 * a * mat, ws.B.data_ptr() + 4 * a * mat)
    # the frames' factor (the text matrix is factored on the side stream); the inverse halves
    # of the Fb frames, hi then lo, are what the tensor-core scan reads
    split = ws.inv_split.data_ptr() if tensor_cores else None
    if delta_rule == "sana_scaled":
        # python-float scalars as branch.py:167-168 computes them; the C ABI rounds them to fp32
        # as torch does when it multiplies them into an fp32 tensor
        inj_scale = (1.0 / tpf) ** 0.5
        call("vdn_sana_factor", ws.A.data_ptr(), ws.B.data_ptr(), Fb, H, D, 1.0 / tpf,
             None if tensor_cores else ws.inv.data_ptr(), split, -1, 0.0, 0.0, None, stream)
    else:
        inj_scale = 0.0
        call("vdn_delta_factor", ws.A.data_ptr(), ws.B.data_ptr(), Fb, H, D, ws.inv.data_ptr(), info.data_ptr(),
             -1, 0.0, None, split, stream)
    main.wait_event(side_done)
    if info is not None:
        # after the join: an immediate validation (outside a scope) reads the text row too
        record_factor_status(([info[Fb:Fb + 1]] if has_text else []) + [info[:Fb]], ws.info_ring, info)
    if tensor_cores:
        call("vdn_bidir_scan_tc", split, ws.B.data_ptr(), ws.alpha.data_ptr(), _lib.ptr(s0), Fb, Fb, H, inj_scale,
             ws.prefix.data_ptr(), ws.suffix.data_ptr(), status.err_ptr, stream)
    else:
        call("vdn_bidir_scan", ws.inv.data_ptr(), ws.B.data_ptr(), ws.alpha.data_ptr(), _lib.ptr(s0), Fb, H, D,
             inj_scale, ws.prefix.data_ptr(), ws.suffix.data_ptr(), stream)
    lo, hi = ws.bounds_arrays(bounds)
    for a, b in tiles:
        n = (b - a) * tpf
        if q_ready:
            oq = a  # ws.qf holds every frame
        else:
            oq = feature(q_raw, "q", ws.qf, True, a, b)
        q_ptr = ws.qf.data_ptr() + 2 * oq * fhsd
        # output gate: sigmoid(bf16(x W_down^T) W_up^T + b)  (branch.py:754-758)
        call("vdn_cast_rows", aux.data_ptr() + 4 * a * tpf * aux_ld, aux_ld, ogd_col0, n, D, ws.ogd.data_ptr(),
             ws.ogd.stride(0), stream)
        row0 = int(out_row0) + a * tpf
        if tensor_cores:
            # gather, Q S^T, the output-gate up-projection and the epilogue in one kernel
            call("vdn_readout_tc", q_ptr, b - a, H, tpf, ws.prefix.data_ptr(), ws.suffix.data_ptr(),
                 ws.alpha.data_ptr(), _lib.ptr(s0), lo.data_ptr(), hi.data_ptr(), int(bridge == "alpha"),
                 bw.norm_w.data_ptr(), ws.ogd.data_ptr(), bw.og_up.data_ptr(), bw.og_bias.data_ptr(), out.data_ptr(),
                 out.stride(0), row0, a, Fb, status.err_ptr, stream)
            continue
        call("vdn_gemm", 0, ws.ogd.data_ptr(), D, None, 0, 0, bw.og_up.data_ptr(), D, ws.og.data_ptr(), inner, 0,
             n, inner, D, 1.0, None, None, None, None, bw.og_bias.data_ptr(), 1, None, 0, status.err_ptr, stream)
        call("vdn_readout", q_ptr, b - a, H, tpf, D, ws.prefix.data_ptr(), ws.suffix.data_ptr(),
             ws.alpha.data_ptr(), _lib.ptr(s0), lo.data_ptr(), hi.data_ptr(), int(bridge == "alpha"),
             bw.norm_w.data_ptr(), ws.og.data_ptr(), inner, out.data_ptr(), out.stride(0), row0, a, Fb, stream)


class B200LinearBranch:
    """Drop-in for ``LinearBranch`` / ``OptimizedLinearBranch`` (branch.py:533-571,
    runtime.py:237-245) running the sm_100a kernels."""

    def __init__(self, weights, num_heads, head_dim, delta_rule="vdn_solve", bridge="alpha", a_fp32=True,
                 short_conv=("k", "v"), enable_text_state=True, tile_frames=0, **_runtime):
        if delta_rule not in DELTA_RULES:
            raise ValueError(f"unknown delta rule: {delta_rule!r}")
        if bridge not in ("alpha", "none"):
            raise ValueError("bridge must be 'alpha' or 'none'")
        targets = tuple(short_conv)
        if len(set(targets)) != len(targets) or any(t not in ("q", "k", "v") for t in targets):
            raise ValueError("short_conv must be a distinct subset of ('q', 'k', 'v')")
        self.w = weights
        self.num_heads = int(num_heads)
        self.head_dim = int(head_dim)
        self.delta_rule = delta_rule
        self.bridge = bridge
        self.a_fp32 = bool(a_fp32)
        self.short_conv = targets
        self.enable_text_state = bool(enable_text_state)
        if isinstance(tile_frames, bool) or not isinstance(tile_frames, int) or tile_frames < 0:
            raise ValueError("tile_frames must be a non-negative integer")  # nodes.py:247-248
        self.tile_frames = tile_frames
        self._dev_weights: dict = {}
        self._workspaces: dict = {}
        self.status = None

    def detach_weights(self):
        self.w = None

    def release(self):
        self._dev_weights.clear()
        self._workspaces.clear()

    clear = release

    def device_weights(self, weights, device) -> BranchDeviceWeights:
        key = (str(device), id(weights))
        if key not in self._dev_weights:
            self._dev_weights[key] = BranchDeviceWeights.from_dict(weights, self.num_heads, self.head_dim, device,
                                                                   short_conv=self.short_conv)
        return self._dev_weights[key]

    def workspace(self, device, Fb, tpf, text_len, tile_frames=None) -> BranchWorkspace:
        tile = None if tile_frames is None or int(tile_frames) >= Fb else int(tile_frames)
        key = (str(device), Fb, tpf, text_len, tile)
        if key not in self._workspaces:
            self._workspaces[key] = BranchWorkspace(device, Fb, tpf, self.num_heads, self.head_dim, text_len,
                                                    tile_frames=tile)
        return self._workspaces[key]

    def readout(self, weights, xv, q_raw, k_raw, v_raw, num_frames, tokens_per_frame, bounds, frame_size=None,
                text_x=None, text_k_raw=None, text_v_raw=None, skip_ends=False, *, inference=False,
                tile_frames=None):
        """The branch before ``to_out_linear`` (branch.py:672-722).  ``tile_frames``: run the
        branch frames in tiles of that many frames (the low-memory spelling of
        runtime.py:421-543; same result)."""
        expected_rows = num_frames * tokens_per_frame
        if xv.ndim != 2 or xv.shape[0] != expected_rows:
            raise ValueError("xv rows must equal num_frames * tokens_per_frame")
        H, D = self.num_heads, self.head_dim
        expected_qkv = (expected_rows, H, D)
        if q_raw.shape != expected_qkv or k_raw.shape != expected_qkv or v_raw.shape != expected_qkv:
            raise ValueError("raw q/k/v have incompatible video row/head geometry")
        if len(bounds) != num_frames:
            raise ValueError("bounds must contain one entry per frame")
        if frame_size is None and self.short_conv:
            raise ValueError("short convolution requires frame_size")
        _lib.require_cuda(xv, q_raw, k_raw, v_raw)
        dev = xv.device
        out = torch.zeros(expected_rows, H * D, device=dev, dtype=torch.bfloat16)
        if skip_ends:
            if num_frames <= 2:
                return out
            F_b, r0 = num_frames - 2, tokens_per_frame
            bounds_b = [(lo - 1, hi - 1) for lo, hi in bounds[1:-1]]
        else:
            F_b, r0 = num_frames, 0
            bounds_b = list(bounds)
        rows = slice(r0, r0 + F_b * tokens_per_frame)
        bw = self.device_weights(weights, dev)
        text = self.enable_text_state and text_x is not None
        if text and (text_k_raw is None or text_v_raw is None):
            raise ValueError("text state needs both raw text key and value")
        ws = self.workspace(dev, F_b, tokens_per_frame, text_x.shape[0] if text else 0, tile_frames)
        # side projections [beta | og_down | alpha_down] as fp32 (branch.py:736, :743-751, :755)
        w_side = torch.cat([bw.beta_w, bw.og_down, bw.alpha_down], 0).contiguous()
        n_side = w_side.shape[0]
        n_pad = (n_side + 255) // 256 * 256
        st = self.status or _lib.DeviceStatus(dev)

        def side(x):
            xb = x.to(torch.bfloat16).contiguous()
            o = torch.empty(xb.shape[0], n_pad, device=dev, dtype=torch.float32)
            _lib.call("vdn_gemm", 0, xb.data_ptr(), xb.shape[1], None, 0, 0, w_side.data_ptr(), w_side.shape[1],
                      o.data_ptr(), n_pad, 1, xb.shape[0], n_side, xb.shape[1], 1.0, None, None, None, None, None, 0,
                      None, 0, st.err_ptr, _lib.stream_handle(dev))
            return o

        aux = side(xv[rows])

        def flat(t):
            t = t.reshape(t.shape[0], H * D) if t.is_contiguous() else t.contiguous().reshape(t.shape[0], H * D)
            return t.to(torch.bfloat16)

        kw = dict(q_raw=flat(q_raw[rows]), k_raw=flat(k_raw[rows]), v_raw=flat(v_raw[rows]), aux=aux, beta_col0=0,
                  ogd_col0=H, ad_col0=H + D, Fb=F_b, tpf=tokens_per_frame, frame_size=frame_size, bounds=bounds_b,
                  bridge=self.bridge, out=out, out_row0=r0, status=st, short_conv=self.short_conv,
                  delta_rule=self.delta_rule)
        if text:
            kw.update(text_k=flat(text_k_raw), text_v=flat(text_v_raw), text_aux=side(text_x))
        run_branch(ws, bw, **kw)
        if self.status is None:
            st.raise_if_failed()
        return out

    def projected_delta(self, weights, xv, q_raw, k_raw, v_raw, num_frames, tokens_per_frame, bounds, *,
                        frame_size=None, text_x=None, text_k_raw=None, text_v_raw=None, skip_ends=False,
                        inference=False, projector=None, tile_frames=None):
        """Branch output after ``to_out_linear`` (runtime.py:545-607).  As there, an inference
        call with ``tile_frames`` (else the constructor's) > 0 runs in frame tiles."""
        tile = self.tile_frames if tile_frames is None else int(tile_frames)
        readout = self.readout(weights, xv, q_raw, k_raw, v_raw, num_frames, tokens_per_frame, bounds,
                               frame_size=frame_size, text_x=text_x, text_k_raw=text_k_raw, text_v_raw=text_v_raw,
                               skip_ends=skip_ends, inference=inference,
                               tile_frames=tile if inference and tile > 0 else None)
        if projector is None:
            from .projection import project
            return project(readout.to(xv.dtype), weights)
        return projector(readout.to(xv.dtype))


__all__ = ["B200LinearBranch", "BranchDeviceWeights", "BranchWorkspace", "DELTA_RULES", "InfoRing", "TEXT_STATE_SCALE",
           "TILE_HALO", "cholesky_runtime_scope", "claim_factor_status", "feature_frames", "frame_tiles",
           "record_factor_status", "run_branch"]
