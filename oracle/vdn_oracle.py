"""CPU float64 restatement of the VDN-H3 hybrid attention block forward.

TEST INFRASTRUCTURE ONLY.  This module is the parity checker for the CUDA path.
Only ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` / ``--impl
reference`` legs of ``bench.py`` may import it, and only to check or to time a CPU
baseline.  The product path (the ``comfyui-kirei-vdn-h3_b200`` package and its C-ABI
library) never calls into it.

Every function restates the algorithm of hyukudan/ComfyUI-Kirei-VDN-H3 v0.3.3; the
reference file:line it follows is cited in each docstring (paths inside that project).
Arithmetic is float64 throughout so the oracle is an upper-precision stand-in for the
reference's fp32 CPU path and bf16 GPU path alike.

Pinning: ``tests/golden/make_golden.py`` runs the reference itself (its own torch code,
imported read-only where it is mounted) on seeded config-0 inputs and stores the outputs
under ``tests/golden/``; ``tests/test_oracle_golden.py`` checks this module against them.
Parity unpinned for RoPE (``rope_split_half``): the reference hands it to comfy-kitchen's
``rms_rope_split_half_``, which is absent from the reference tree and this image; the
restatement follows ComfyUI's published freqs convention (see the function).  Parity
unpinned for ConvRot int8 (``convrot_rotate``): the reference hands it to comfy-kitchen too;
the restatement follows the published ConvRot method with one fixed Hadamard construction.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np
import torch
import torch.nn.functional as F

F64 = torch.float64
ANCHOR_MODES = ("none", "columns", "rows", "both")
TEXT_STATE_SCALE = 0.5  # branch.py:23
FP8_MAX = 448.0  # fp8.py:30 (float8_e4m3fn max)


_COMPUTE = [F64]
_MATMUL = [None]  # None: GEMM operands in the compute dtype; torch.bfloat16: the reference's bf16 GEMMs


def set_compute_dtype(dtype) -> torch.dtype:
    """Switch the arithmetic dtype (float64 for parity checks; float32 reproduces the
    reference's CPU path for the timed CPU baseline).  Returns the previous dtype."""
    prev = _COMPUTE[0]
    _COMPUTE[0] = dtype
    return prev


def set_matmul_dtype(dtype):
    """Operand dtype of the block's large products: the bf16 projections (``project``) and
    the window attention's two products.  None keeps them in the compute dtype (the parity
    checks); ``torch.bfloat16`` runs them as the reference's bf16 path does on its own
    torch ops -- bf16 operands, bf16 results (hybrid.py:260-268, window.py:197-216) -- with
    the statistics, factor and scans still in the compute dtype (branch.py:197-243 keeps
    them in fp32).  Used to time the reference path at config 1's dtype.  Returns the
    previous setting."""
    prev = _MATMUL[0]
    _MATMUL[0] = dtype
    return prev


def _t(x) -> torch.Tensor:
    if isinstance(x, np.ndarray):
        x = torch.from_numpy(x)
    return x.detach().to("cpu", _COMPUTE[0])


# ---------------------------------------------------------------------------------------
# Geometry (window.py:141-178, layout.py:19-41)
# ---------------------------------------------------------------------------------------

def window_bounds(num_frames: int, radius: int, chunk: int = 0) -> list[tuple[int, int]]:
    """Per-frame inclusive key-frame range (window.py:141-153)."""
    if num_frames < 0 or radius < 0:
        raise ValueError("num_frames and radius must be non-negative")
    out = []
    for f in range(num_frames):
        if chunk <= 0:
            out.append((f - radius, f + radius))
        else:
            base = f // chunk
            out.append(((base - radius) * chunk, (base + radius + 1) * chunk - 1))
    return out


def full_coverage(bounds, num_frames) -> bool:
    """window.py:156-159."""
    return all(lo <= 0 and hi >= num_frames - 1 for lo, hi in bounds)


@dataclass(frozen=True)
class Layout:
    """Packed-sequence geometry (layout.py:19-41)."""

    seq_len: int
    video_start: int
    video_end: int
    num_frames: int
    tokens_per_frame: int
    frame_size: tuple[int, int]
    text_start: int
    text_len: int
    bounds: tuple = ()
    full_cover: bool = False
    anchor_frames: str = "both"


def make_layout(text_len, num_frames, grid, *, radius=1, chunk=5, anchor_frames="both",
                text_first=True) -> Layout:
    gh, gw = grid
    tpf = gh * gw
    video = num_frames * tpf
    if text_first:
        ts, vs = 0, text_len
    else:
        vs, ts = 0, video
    bounds = tuple(window_bounds(num_frames, radius, chunk))
    return Layout(
        seq_len=text_len + video, video_start=vs, video_end=vs + video,
        num_frames=num_frames, tokens_per_frame=tpf, frame_size=(gh, gw),
        text_start=ts, text_len=text_len, bounds=bounds,
        full_cover=full_coverage(bounds, num_frames), anchor_frames=anchor_frames,
    )


# ---------------------------------------------------------------------------------------
# Window softmax (window.py:277-344; tests/test_window.py:41-69)
# ---------------------------------------------------------------------------------------

def allowed_mask(seq, vs, ve, num_frames, tpf, bounds, anchors, rows=None) -> torch.Tensor:
    """Boolean [rows, seq] mask of allowed (query, key) pairs (window.py:327-344);
    all rows when ``rows`` is None."""
    keys = torch.arange(seq)
    qrows = keys if rows is None else torch.as_tensor(rows, dtype=torch.long)
    kglob = (keys < vs) | (keys >= ve)
    qglob = (qrows < vs) | (qrows >= ve)
    kf = torch.div(keys - vs, tpf, rounding_mode="floor")[None, :]
    qf = torch.div(qrows - vs, tpf, rounding_mode="floor")
    lo_f = torch.tensor([max(a, 0) for a, _ in bounds], dtype=torch.long)
    hi_f = torch.tensor([min(b, num_frames - 1) for _, b in bounds], dtype=torch.long)
    qfc = qf.clamp(0, num_frames - 1)
    lo = torch.where(qglob, 0, lo_f[qfc])
    hi = torch.where(qglob, num_frames - 1, hi_f[qfc])
    allowed = qglob[:, None] | kglob[None, :] | ((kf >= lo[:, None]) & (kf <= hi[:, None]))
    if anchors in ("columns", "both"):
        allowed = allowed | ((kf == 0) | (kf == num_frames - 1))
    if anchors in ("rows", "both"):
        allowed = allowed | ((qf[:, None] == 0) | (qf[:, None] == num_frames - 1))
    return allowed


def window_attention(q, k, v, vs, ve, num_frames, tpf, bounds, scale, anchors="none",
                     rows=None, chunk=512) -> torch.Tensor:
    """Exact masked softmax attention (window.py:277-313 semantics), computed in blocks
    of ``chunk`` query rows so memory stays bounded.

    ``q,k,v``: [S, H, D].  ``rows`` optionally restricts which query rows are computed
    (a 1-D index tensor); the result then has one entry per requested row.
    """
    q, k, v = _t(q), _t(k), _t(v)
    seq = q.shape[0]
    rows = torch.arange(seq) if rows is None else torch.as_tensor(rows, dtype=torch.long)
    out = torch.empty(len(rows), q.shape[1], q.shape[2], dtype=q.dtype)
    for i in range(0, len(rows), chunk):
        r = rows[i:i + chunk]
        mask = allowed_mask(seq, vs, ve, num_frames, tpf, bounds, anchors, rows=r)
        logits = torch.einsum("qhd,khd->hqk", q[r], k) * scale
        logits = logits.masked_fill(~mask[None], float("-inf"))
        p = torch.softmax(logits, dim=-1)
        out[i:i + chunk] = torch.einsum("hqk,khd->qhd", p, v)
    return out


def frame_key_sets(num_frames, bounds, anchors):
    """Runs of consecutive frames whose rows see the same key frames (window.py:248-274):
    [(first, stop, frames)], ``frames`` None for anchor-frame rows that see every key."""
    last = num_frames - 1
    runs = []
    for f in range(num_frames):
        if anchors in ("rows", "both") and f in (0, last):
            sig = None
        else:
            sel = set(range(max(bounds[f][0], 0), min(bounds[f][1], last) + 1))
            if anchors in ("columns", "both"):
                sel.update((0, last))
            sig = tuple(sorted(sel))
        if runs and runs[-1][2] == sig and runs[-1][1] == f:
            runs[-1] = (runs[-1][0], f + 1, sig)
        else:
            runs.append((f, f + 1, sig))
    return runs


def _sdpa_rows(q, k, v, scale):
    """softmax(q k^T * scale) v for [rows, H, D] operands, in the matmul dtype when set."""
    md = _MATMUL[0] or q.dtype

    def heads_major(t):  # [rows, H, D] -> contiguous [1, H, rows, D] (the fused CPU kernel's layout)
        return t.to(md).permute(1, 0, 2).contiguous().unsqueeze(0)

    o = F.scaled_dot_product_attention(heads_major(q), heads_major(k), heads_major(v), scale=scale)
    return o[0].permute(1, 0, 2).to(q.dtype)


def window_attention_grouped(q, k, v, vs, ve, num_frames, tpf, bounds, scale, anchors="none",
                             rows=None) -> torch.Tensor:
    """The same exact window softmax as ``window_attention``, computed the way the reference's
    grouped backend does (window.py:277-313): global rows against every key; each run of
    frames with one key set against the gathered [global rows, visible frames] keys only, so
    the work is the allowed pairs rather than the dense square.  ``rows``: restrict the
    output to these query rows (sorted or not); returns [len(rows), H, D] then."""
    q, k, v = _t(q), _t(k), _t(v)
    seq = q.shape[0]
    want = torch.arange(seq) if rows is None else torch.as_tensor(rows, dtype=torch.long)
    need = torch.zeros(seq, dtype=torch.bool)
    need[want] = True
    out = torch.zeros(seq, q.shape[1], q.shape[2], dtype=q.dtype)
    glob = torch.cat([torch.arange(0, vs), torch.arange(ve, seq)])
    g_rows = glob[need[glob]]
    if len(g_rows):
        out[g_rows] = _sdpa_rows(q[g_rows], k, v, scale)
    for first, stop, frames in frame_key_sets(num_frames, bounds, anchors):
        r = torch.arange(vs + first * tpf, vs + stop * tpf)
        r = r[need[r]]
        if not len(r):
            continue
        if frames is None:
            keys = torch.arange(seq)
        else:
            vid = torch.cat([torch.arange(vs + f * tpf, vs + (f + 1) * tpf) for f in frames])
            keys = torch.cat([glob, vid])
        out[r] = _sdpa_rows(q[r], k[keys], v[keys], scale)
    return out[want]


def key_count_per_row(seq, vs, ve, num_frames, tpf, bounds, anchors) -> np.ndarray:
    """Allowed keys per query row, computed from intervals (no [S,S] mask)."""
    out = np.empty(seq, dtype=np.int64)
    glob = vs + (seq - ve)
    out[:vs] = seq
    out[ve:] = seq
    last = num_frames - 1
    for f in range(num_frames):
        s = vs + f * tpf
        if anchors in ("rows", "both") and f in (0, last):
            out[s:s + tpf] = seq
            continue
        lo, hi = max(bounds[f][0], 0), min(bounds[f][1], last)
        frames = set(range(lo, hi + 1))
        if anchors in ("columns", "both"):
            frames.update((0, last))
        out[s:s + tpf] = glob + len(frames) * tpf
    return out


# ---------------------------------------------------------------------------------------
# Branch pieces (kernels.py, branch.py, runtime.py)
# ---------------------------------------------------------------------------------------

def activate(x, l2norm: bool) -> torch.Tensor:
    """SiLU then optional L2 over the last dim, eps 1e-6 (kernels.py:47-51)."""
    y = F.silu(_t(x))
    if l2norm:
        y = y / y.norm(dim=-1, keepdim=True).clamp_min(1e-6)
    return y


def temporal_shift(x, w) -> torch.Tensor:
    """Zero-padded depthwise temporal conv over axis 0 (kernels.py:59-68).

    ``x``: [T, S_frame, C]; ``w``: [C, taps] with taps odd.
    """
    x, w = _t(x), _t(w)
    taps = w.shape[-1]
    pad = taps // 2
    T = x.shape[0]
    # out[t] = sum_j x[t + j - pad] * w[:, j], terms outside [0, T) being zero
    out = x * w[:, pad].view(1, 1, -1)
    for j in range(taps):
        s = j - pad
        if s == 0 or abs(s) >= T:
            continue
        if s > 0:
            out[:T - s] += x[s:] * w[:, j].view(1, 1, -1)
        else:
            out[-s:] += x[:T + s] * w[:, j].view(1, 1, -1)
    return out


def conv_features(tokens, spatial_w, temporal_w, num_frames, frame_size, l2norm) -> torch.Tensor:
    """Depthwise spatial conv per frame, temporal 5-tap conv, SiLU, L2 (branch.py:443-480).

    ``tokens``: [F*gh*gw, H, D]; returns [F, H, gh*gw, D] (the FHSD layout).
    """
    tokens = _t(tokens)
    heads, dim = tokens.shape[-2:]
    gh, gw = frame_size
    ch = heads * dim
    vol = tokens.reshape(num_frames, gh, gw, ch).permute(0, 3, 1, 2)
    sw = _t(spatial_w)
    kh, kw = sw.shape[-2:]
    vol = F.conv2d(vol, sw, padding=(kh // 2, kw // 2), groups=ch)
    flat = vol.permute(0, 2, 3, 1).reshape(num_frames, gh * gw, ch)
    tm = temporal_shift(flat, _t(temporal_w).reshape(ch, -1))
    y = activate(tm.reshape(num_frames, gh * gw, heads, dim), l2norm)
    return y.permute(0, 2, 1, 3).contiguous()


def to_fhsd(tokens, num_frames) -> torch.Tensor:
    t = _t(tokens)
    rows, h, d = t.shape
    return t.reshape(num_frames, rows // num_frames, h, d).permute(0, 2, 1, 3).contiguous()


def frame_statistics(key, value, beta) -> tuple[torch.Tensor, torch.Tensor]:
    """A = sym((beta*K)^T K), B = (beta*V)^T K per frame/head (branch.py:197-243)."""
    key, value, beta = _t(key), _t(value), _t(beta)
    kb = key * beta[..., None]  # [F, H, S, D]: two-operand products keep memory at the input size
    a = kb.transpose(-1, -2) @ key
    a = 0.5 * (a + a.transpose(-1, -2))
    b = (value * beta[..., None]).transpose(-1, -2) @ key
    return a, b


def alpha_gate(frame_mean, w_down, w_up, dt_bias, a_log, heads, dim) -> torch.Tensor:
    """alpha = exp(-exp(A_log) * softplus(up(down(mean)) + dt_bias)) (branch.py:483-491)."""
    m = _t(frame_mean)
    delta = m @ _t(w_down).T
    delta = delta @ _t(w_up).T + _t(dt_bias)
    decay = torch.exp(_t(a_log)).reshape(heads, 1)
    return torch.exp(-decay * F.softplus(delta.reshape(-1, heads, dim)))


def cholesky_info(a) -> torch.Tensor:
    """First failing leading-minor order per matrix of I+A (0 = SPD); cholesky_ex semantics."""
    m = _t(a)
    n = m.shape[-1]
    flat = (m + torch.eye(n, dtype=m.dtype)).reshape(-1, n, n)
    info = torch.zeros(flat.shape[0], dtype=torch.int32)
    for i in range(flat.shape[0]):
        _, inf = torch.linalg.cholesky_ex(flat[i])
        info[i] = int(inf)
    return info.reshape(m.shape[:-2])


def factor_apply(alpha, a, b) -> tuple[torch.Tensor, torch.Tensor]:
    """T = alpha[...,None] * (I+A)^-1, Inj = B (I+A)^-1 via Cholesky (branch.py:148-160)."""
    a, b, alpha = _t(a), _t(b), _t(alpha)
    n = a.shape[-1]
    eye = torch.eye(n, dtype=a.dtype).expand_as(a)
    chol = torch.linalg.cholesky(a + eye)
    inv_chol = torch.linalg.solve_triangular(chol, eye, upper=False, left=True)
    inverse = inv_chol.transpose(-1, -2) @ inv_chol
    return alpha.unsqueeze(-1) * inverse, b @ inverse


def sana_factor_apply(alpha, a, b, tokens) -> tuple[torch.Tensor, torch.Tensor]:
    """T = alpha*(I - A/tpf), Inj = B/sqrt(tpf) (branch.py:163-177)."""
    a, b, alpha = _t(a), _t(b), _t(alpha)
    eye = torch.eye(a.shape[-1], dtype=a.dtype)
    return alpha.unsqueeze(-1) * (eye - a / tokens), b / math.sqrt(tokens)


def run_scans(transition, injection, initial) -> tuple[torch.Tensor, torch.Tensor]:
    """prefix_t = Inj_t + prefix_{t-1} T_t (t up), suffix likewise (t down) (branch.py:297-312)."""
    frames = transition.shape[0]
    prefix = torch.empty_like(injection)
    suffix = torch.empty_like(injection)
    state = initial
    for f in range(frames):
        state = injection[f] + state @ transition[f]
        prefix[f] = state
    state = initial
    for f in range(frames - 1, -1, -1):
        state = injection[f] + state @ transition[f]
        suffix[f] = state
    return prefix, suffix


def gather_linear_state(prefix, suffix, alpha, bounds, bridge="alpha", text_state=None):
    """Window-bridged linear state per frame (branch.py:345-396)."""
    frames = prefix.shape[0]
    log_prefix = torch.cat((torch.zeros_like(alpha[:1]), alpha.clamp_min(1e-12).log().cumsum(0)))
    zero = torch.zeros_like(prefix[0])
    out = []
    for f, (raw_lo, raw_hi) in enumerate(bounds):
        lo, hi = max(raw_lo, 0), min(raw_hi, frames - 1)
        has_before, has_after = raw_lo - 1 >= 0, raw_hi + 1 < frames
        fallback = zero if text_state is None else text_state
        before = prefix[lo - 1] if has_before else fallback
        after = suffix[hi + 1] if has_after else fallback
        if bridge == "alpha":
            before = before * torch.exp(log_prefix[f + 1] - log_prefix[lo]).unsqueeze(1)
            after = after * torch.exp(log_prefix[hi + 1] - log_prefix[f]).unsqueeze(1)
        out.append(before + after)
    return torch.stack(out)


def rope_split_half(x, freqs) -> torch.Tensor:
    """RoPE on [S, H, D] heads, split-half pairing (hybrid.py:271-292 calls comfy-kitchen's
    ``rms_rope_split_half_`` with rot_dim = 2 * freqs.shape[-3]).  PARITY UNPINNED: that
    library is absent, so this restates ComfyUI's freqs convention: freqs [S, rot/2, 2, 2]
    holds per token and pair index j the matrix [[cos, -sin], [sin, cos]] applied as
    out_a = sum_b f[j, a, b] pair_b (comfy/ldm/flux/math.py apply_rope1), with the pair
    (x[j], x[j + rot/2]) instead of the interleaved (x[2j], x[2j + 1]); features >= rot pass
    through."""
    x, f = _t(x), _t(freqs)
    half = f.shape[-3]
    rot = 2 * half
    f = f.reshape(-1, 1, half, 2, 2)  # [S or 1, heads broadcast, half, 2, 2]
    a, b = x[..., :half], x[..., half:rot]
    out = x.clone()
    out[..., :half] = f[..., 0, 0] * a + f[..., 0, 1] * b
    out[..., half:rot] = f[..., 1, 0] * a + f[..., 1, 1] * b
    return out


def make_rope_freqs(seq, rot, *, theta=10000.0, offset=0) -> torch.Tensor:
    """Deterministic synthetic RoPE table [seq, rot/2, 2, 2] (fp32) of 1-D positions
    offset..offset+seq-1 with the usual theta^(-2j/rot) frequencies (the layout ComfyUI's
    ``rope()`` returns, comfy/ldm/flux/math.py)."""
    pos = torch.arange(offset, offset + seq, dtype=torch.float64)
    omega = 1.0 / theta ** (torch.arange(0, rot, 2, dtype=torch.float64) / rot)
    ang = pos[:, None] * omega[None]
    c, s = torch.cos(ang), torch.sin(ang)
    return torch.stack([torch.stack([c, -s], -1), torch.stack([s, c], -1)], -2).float()


def rms_norm(x, weight, eps=1e-6) -> torch.Tensor:
    """x * rsqrt(mean(x^2) + eps) * weight over the last dim (branch.py:494-498)."""
    x = _t(x)
    ms = x.square().mean(dim=-1, keepdim=True)
    return x * torch.rsqrt(ms + eps) * _t(weight)


@dataclass
class BranchConfig:
    """Released-lineage branch structure (docs/ARCHITECTURE.md:70-82, spec.py:297-353)."""

    delta_rule: str = "vdn_solve"
    bridge: str = "alpha"
    short_conv: tuple = ("k", "v")
    enable_text_state: bool = True

    def node_config(self, **extra) -> dict:
        """The node config that builds this branch structure (nodes.py:98-116 reads these
        keys, defaulting to short_conv=() and enable_text_state=False when they are absent),
        with the softmax gate on."""
        return dict(enable_softmax_gate=True, delta_rule=self.delta_rule, bridge=self.bridge,
                    short_conv=tuple(self.short_conv), enable_text_state=self.enable_text_state, **extra)


def text_state(weights, text_x, text_k, text_v, heads, dim, cfg: BranchConfig):
    """Text rows as one extra 'frame', alpha = 1, S0 = 0.5 * Inj (branch.py:649-670)."""
    if not cfg.enable_text_state or text_x is None:
        return None
    length = text_x.shape[0]
    key = activate(text_k, True).reshape(1, length, heads, dim).permute(0, 2, 1, 3)
    val = activate(text_v, False).reshape(1, length, heads, dim).permute(0, 2, 1, 3)
    beta = torch.sigmoid(_t(text_x) @ _t(weights["beta_proj.weight"]).T)
    beta = beta.reshape(1, length, heads).permute(0, 2, 1)
    a, b = frame_statistics(key, val, beta)
    ones = torch.ones(1, heads, dim, dtype=_COMPUTE[0])
    if cfg.delta_rule == "vdn_solve":
        _, inj = factor_apply(ones, a, b)
    else:
        _, inj = sana_factor_apply(ones, a, b, length)
    return TEXT_STATE_SCALE * inj[0]


def branch_readout(weights, xv, q_raw, k_raw, v_raw, num_frames, tpf, bounds, frame_size,
                   heads, dim, cfg: BranchConfig, text_x=None, text_k=None, text_v=None,
                   skip_ends=False, return_parts=False):
    """Linear-branch readout before ``to_out_linear`` (branch.py:672-785; runtime.py:545-607).

    Returns [F*tpf, H*D] (rows of skipped end frames are zero).
    """
    xv = _t(xv)
    rows_total = num_frames * tpf
    if skip_ends:
        if num_frames <= 2:
            return torch.zeros(rows_total, heads * dim, dtype=_COMPUTE[0])
        inner = slice(tpf, (num_frames - 1) * tpf)
        inner_out = branch_readout(
            weights, xv[inner], _t(q_raw)[inner], _t(k_raw)[inner], _t(v_raw)[inner],
            num_frames - 2, tpf, [(lo - 1, hi - 1) for lo, hi in bounds[1:-1]], frame_size,
            heads, dim, cfg, text_x, text_k, text_v, skip_ends=False, return_parts=return_parts,
        )
        parts = None
        if return_parts:
            inner_out, parts = inner_out
        out = torch.zeros(rows_total, heads * dim, dtype=_COMPUTE[0])
        out[inner] = inner_out
        return (out, parts) if return_parts else out
    w = weights

    def feature(tokens, name):
        l2 = name != "v"
        if name in cfg.short_conv:
            return conv_features(tokens, w[f"short_conv.{name}_sp.weight"],
                                 w[f"short_conv.{name}_tm.weight"], num_frames, frame_size, l2)
        return to_fhsd(activate(tokens, l2), num_frames)

    qf, kf, vf = feature(q_raw, "q"), feature(k_raw, "k"), feature(v_raw, "v")
    beta = torch.sigmoid(xv @ _t(w["beta_proj.weight"]).T)
    beta = beta.reshape(num_frames, tpf, heads).permute(0, 2, 1)
    a, b = frame_statistics(kf, vf, beta)
    frame_mean = xv.reshape(num_frames, tpf, -1).mean(dim=1)
    alpha = alpha_gate(frame_mean, w["alpha.down.weight"], w["alpha.up.weight"],
                       w["alpha.dt_bias"], w["alpha.A_log"], heads, dim)
    s0 = text_state(w, text_x, text_k, text_v, heads, dim, cfg)
    if cfg.delta_rule == "vdn_solve":
        trans, inj = factor_apply(alpha, a, b)
    else:
        trans, inj = sana_factor_apply(alpha, a, b, tpf)
    init = torch.zeros_like(inj[0]) if s0 is None else s0
    prefix, suffix = run_scans(trans, inj, init)
    gate = torch.sigmoid(
        (xv @ _t(w["output_gate.down.weight"]).T) @ _t(w["output_gate.up.weight"]).T
        + _t(w["output_gate.up.bias"])
    )
    state = gather_linear_state(prefix, suffix, alpha, bounds, cfg.bridge, s0)
    readout = qf @ state.transpose(-1, -2)
    normed = rms_norm(readout, w["norm.weight"], 1e-6)
    out = normed.permute(0, 2, 1, 3).reshape(rows_total, heads * dim) * gate
    if return_parts:
        parts = dict(q=qf, k=kf, v=vf, beta=beta, A=a, B=b, alpha=alpha, text_state=s0,
                     prefix=prefix, suffix=suffix, state=state, gate=gate, readout=readout)
        return out, parts
    return out


# ---------------------------------------------------------------------------------------
# Projections (projection.py:259-268, fp8.py:84-266) and the config-2 INT8 scheme
# ---------------------------------------------------------------------------------------

def _int8_rows_np(x32: np.ndarray) -> tuple[torch.Tensor, torch.Tensor]:
    """IEEE fp32 arithmetic throughout: scale = max(amax / 127, 1e-12); q = rne(x / scale)."""
    amax = np.abs(x32).max(axis=1)
    scale = np.maximum(amax / np.float32(127.0), np.float32(1e-12)).astype(np.float32)
    q = np.clip(np.rint(x32 / scale[:, None]), -127, 127).astype(np.int8)
    return torch.from_numpy(q), torch.from_numpy(scale)


def int8_quantize_weight(w) -> tuple[torch.Tensor, torch.Tensor]:
    """Symmetric per-output-channel int8 (config 2): one fp32 scale per row of W [N, K]."""
    return _int8_rows_np(_t(w).to(torch.float32).numpy())


def int8_quantize_rows(x) -> tuple[torch.Tensor, torch.Tensor]:
    """Dynamic per-token int8 (config 2), the same rule as the weights: one scale per row."""
    return _int8_rows_np(_t(x).to(torch.float32).numpy())


CONVROT_GROUP = 256  # projection.py:44 (INT8_CONVROT_GROUP)


def convrot_rotate(x, group: int = CONVROT_GROUP) -> np.ndarray:
    """ConvRot's group-wise rotation of the rows of ``x`` [rows, K], in IEEE fp32.

    The reference hands the rotation to comfy-kitchen (``QuantizedTensor.from_float(...,
    convrot=True, convrot_groupsize=256)`` and ``ck.int8_linear(..., convrot=True)``,
    projection.py:74-97 and :243-256); comfy-kitchen is not in the reference tree, so this
    restates the published ConvRot method (a block-diagonal regular Hadamard rotation over
    groups of ``group`` channels) with one fixed construction: each group is multiplied by
    R / sqrt(group), R the Kronecker power of the order-4 regular Hadamard matrix J - 2I.
    Parity against comfy-kitchen is unpinned (its matrix ordering is not visible here).

    Evaluation order (the CUDA quantiser follows it exactly): the group index is written in
    base 4, digits d0 (least significant) to dn; for each digit in that order every quadruple
    of elements that differ only in that digit becomes y = S - 2 x with
    S = (x[d=0] + x[d=1]) + (x[d=2] + x[d=3]); the result is scaled by 1 / sqrt(group).
    """
    x32 = np.ascontiguousarray(_t(x).to(torch.float32).numpy())
    rows, K = x32.shape
    digits = int(round(math.log(group, 4)))
    if 4 ** digits != group or K % group:
        raise ValueError("ConvRot needs a group that is a power of 4 dividing K")
    v = x32.reshape(rows, K // group, *([4] * digits))  # last axis = d0
    for axis in range(v.ndim - 1, 1, -1):
        a = [np.take(v, t, axis=axis) for t in range(4)]
        s = np.expand_dims((a[0] + a[1]) + (a[2] + a[3]), axis)
        v = s - np.float32(2.0) * v
    v = v * np.float32(1.0 / math.sqrt(group))
    return v.reshape(rows, K).astype(np.float32)


def int8_quantize_rows_convrot(x, group: int = CONVROT_GROUP) -> tuple[torch.Tensor, torch.Tensor]:
    """ConvRot int8 rows: the fp32 rotation above of the bf16 rows, then the per-row int8 rule
    of ``_int8_rows_np`` (weights: per output channel, the reference quantises their bf16
    copy, projection.py:84; activations: per token)."""
    xb = _t(x).to(torch.bfloat16).to(torch.float32)
    return _int8_rows_np(convrot_rotate(xb, group))


def project_int8_convrot(rows, w, group: int = CONVROT_GROUP):
    """``rows @ W^T`` through ConvRot int8 (projection.py:243-256): both operands rotated per
    group, quantised per row, exact integer accumulate, dequantised by the two scales."""
    qa, sa = int8_quantize_rows_convrot(rows, group)
    qw, sw = int8_quantize_rows_convrot(w, group)
    acc = int8_accumulate(qa, qw).to(_COMPUTE[0])
    return acc * sa.to(_COMPUTE[0])[:, None] * sw.to(_COMPUTE[0])[None, :]


def int8_accumulate(qa: torch.Tensor, qw: torch.Tensor) -> torch.Tensor:
    """Exact int32 accumulator of int8 operands, computed in int64 then checked to fit."""
    acc = qa.to(torch.int64) @ qw.to(torch.int64).T
    if acc.abs().max() >= 2**31:
        raise OverflowError("int8 accumulator exceeds int32")
    return acc.to(torch.int32)


def fp8_quantize_tensor(x) -> tuple[torch.Tensor, float]:
    """Per-tensor e4m3: scale = max(amax/448, 1e-12) in fp32; q = rn(clamp(x/scale))
    (fp8.py:88-105 with per_tensor=True)."""
    x32 = _t(x).to(torch.float32).numpy()
    scale = np.maximum(np.float32(np.abs(x32).max()) / np.float32(FP8_MAX), np.float32(1e-12)).astype(np.float32)
    q = np.clip(x32 / scale, -FP8_MAX, FP8_MAX).astype(np.float32)
    return torch.from_numpy(q).to(torch.float8_e4m3fn), float(scale)


def project(rows, w, precision="bf16"):
    """``rows @ W^T`` under the chosen precision; float64 result (projection.py:259-268)."""
    if precision == "bf16" and _MATMUL[0] is not None:
        md = _MATMUL[0]

        def operand(t):  # straight to the matmul dtype (no copy when the tensor already is)
            return (torch.from_numpy(t) if isinstance(t, np.ndarray) else t).detach().to("cpu", md)

        return (operand(rows) @ operand(w).T).to(_COMPUTE[0])
    if precision == "bf16" or precision == "fp64":
        return _t(rows) @ _t(w).T
    if precision == "int8":
        qa, sa = int8_quantize_rows(rows)
        qw, sw = int8_quantize_weight(w)
        acc = int8_accumulate(qa, qw).to(_COMPUTE[0])
        return acc * sa.to(_COMPUTE[0])[:, None] * sw.to(_COMPUTE[0])[None, :]
    if precision == "fp8":
        qa, sa = fp8_quantize_tensor(rows)
        qw, sw = fp8_quantize_tensor(w)
        return (qa.to(_COMPUTE[0]) @ qw.to(_COMPUTE[0]).T) * (sa * sw)
    raise ValueError(f"unknown precision {precision!r}")


# ---------------------------------------------------------------------------------------
# Whole block (hybrid.py:409-579)
# ---------------------------------------------------------------------------------------

@dataclass
class BlockWeights:
    """One H3 attention block plus its VDN branch weights (spec.py:471-486)."""

    qkv: torch.Tensor  # [3*H*D, hidden]
    q_norm: torch.Tensor  # [D]
    k_norm: torch.Tensor  # [D]
    out: torch.Tensor  # [hidden, H*D]
    branch: dict = field(default_factory=dict)


def block_forward(x, bw: BlockWeights, lay: Layout, heads, dim, cfg: BranchConfig,
                  *, enable_softmax_gate=True, linear_enabled=True, precision="bf16",
                  return_parts=False, rope_freqs=None, to_out_convrot=False, to_out_precision=None,
                  attention="dense", rows=None):
    """VDN hybrid block forward: QKV, branch on raw video q/k/v, q/k RMSNorm, window
    softmax, per-token head gate, out_proj, delta add on video rows (hybrid.py:409-579).

    ``precision`` selects the projection arithmetic of qkv/out_proj/to_out_linear
    (``bf16`` = exact float64 here; ``int8``/``fp8`` = the config-2 quantised schemes).
    ``to_out_convrot`` (int8 only): ``to_out_linear`` through ConvRot int8 instead, the
    reference's INT8 projection (projection.py:243-256).  ``to_out_precision`` (default:
    ``precision``) is the arithmetic of ``to_out_linear`` alone: the reference projects it in
    the representation its map stores (projection.py:259-268), e.g. bf16 for the edge blocks
    an fp8 model keeps (fp8.py:198).
    ``attention``: ``dense`` (masked square, ``window_attention``) or ``grouped`` (the
    reference's gathered-key spelling, ``window_attention_grouped``; same result, a fraction
    of the work at video sizes).  ``rows``: output only these rows ([len(rows), hidden]):
    the projections of x and the branch statistics still cover every row (keys and frame
    states need them), the attention, gate and output projections only the requested ones.
    """
    to_out_precision = precision if to_out_precision is None else to_out_precision
    x = _t(x)
    seq = x.shape[0]
    inner = heads * dim
    qkv = project(x, bw.qkv, precision)
    q_raw = qkv[:, :inner].reshape(seq, heads, dim)
    k_raw = qkv[:, inner:2 * inner].reshape(seq, heads, dim)
    v = qkv[:, 2 * inner:].reshape(seq, heads, dim)
    w = bw.branch
    linear_active = linear_enabled and not lay.full_cover
    delta = None
    parts = {}
    if linear_active:
        va, vb = lay.video_start, lay.video_end
        ta, tb = lay.text_start, lay.text_start + lay.text_len
        text = cfg.enable_text_state and lay.text_len > 0
        readout = branch_readout(
            w, x[va:vb], q_raw[va:vb], k_raw[va:vb], v[va:vb], lay.num_frames,
            lay.tokens_per_frame, list(lay.bounds), lay.frame_size, heads, dim, cfg,
            text_x=x[ta:tb] if text else None, text_k=k_raw[ta:tb] if text else None,
            text_v=v[ta:tb] if text else None, skip_ends=(lay.anchor_frames == "both"),
        )
        parts["readout"] = readout
    sel = torch.arange(seq) if rows is None else torch.as_tensor(rows, dtype=torch.long)
    if linear_active:
        va, vb = lay.video_start, lay.video_end
        in_video = (sel >= va) & (sel < vb)
        r_read = readout if rows is None else readout[sel[in_video] - va]
        if to_out_convrot and to_out_precision == "int8":
            d = project_int8_convrot(r_read, w["to_out_linear.weight"])
        else:
            d = project(r_read, w["to_out_linear.weight"], to_out_precision)
        if rows is None:
            delta = d
        else:
            delta = torch.zeros(len(sel), d.shape[1], dtype=d.dtype)
            delta[in_video] = d
    qn = rms_norm(q_raw, bw.q_norm, 1e-6)
    kn = rms_norm(k_raw, bw.k_norm, 1e-6)
    if rope_freqs is not None:  # after the norm, softmax path only (the branch read q_raw)
        qn, kn = rope_split_half(qn, rope_freqs), rope_split_half(kn, rope_freqs)
    scale = dim ** -0.5
    attend = window_attention_grouped if attention == "grouped" else window_attention
    if lay.full_cover:
        soft = attend(qn, kn, v, 0, seq, 1, seq, [(0, 0)], scale, "none", rows=rows)
    else:
        soft = attend(qn, kn, v, lay.video_start, lay.video_end, lay.num_frames, lay.tokens_per_frame,
                      list(lay.bounds), scale, lay.anchor_frames, rows=rows)
    parts["softmax"] = soft
    xs = x[sel]
    if enable_softmax_gate:
        g = torch.sigmoid(xs @ _t(w["softmax_gate.up.weight"]).T + _t(w["softmax_gate.up.bias"]))
        flat = (soft * g.reshape(len(sel), heads, 1)).reshape(len(sel), inner)
        parts["gate"] = g
    else:
        flat = soft.reshape(len(sel), inner)
    out = project(flat, bw.out, precision)
    if delta is not None:
        if rows is None:
            out[lay.video_start:lay.video_end] += delta
        else:
            out += delta
        parts["delta"] = delta
    return (out, parts) if return_parts else out


# ---------------------------------------------------------------------------------------
# Seeded synthetic inputs (the benchmark configs' shapes and value distributions)
# ---------------------------------------------------------------------------------------

def make_branch_weights(gen, hidden, heads, dim, *, std=0.02, kernel=5, gate=True,
                        short_conv=("k", "v")) -> dict:
    ch = heads * dim

    def n(*shape, s=std, mean=0.0):
        return torch.randn(*shape, generator=gen, dtype=torch.float32) * s + mean

    w = {
        "to_out_linear.weight": n(hidden, ch),
        "beta_proj.weight": n(heads, hidden),
        "norm.weight": 1.0 + n(dim, s=0.1),
        "alpha.A_log": n(heads, s=0.3),
        "alpha.dt_bias": n(ch, s=0.5, mean=-2.0),
        "alpha.down.weight": n(dim, hidden),
        "alpha.up.weight": n(ch, dim, s=0.1),
        "output_gate.down.weight": n(dim, hidden),
        "output_gate.up.weight": n(ch, dim, s=0.1),
        "output_gate.up.bias": n(ch, s=0.1),
    }
    if gate:
        w["softmax_gate.up.weight"] = n(heads, hidden)
        w["softmax_gate.up.bias"] = n(heads, s=0.5)
    for t in short_conv:
        w[f"short_conv.{t}_sp.weight"] = n(ch, 1, kernel, kernel, s=0.2)
        w[f"short_conv.{t}_tm.weight"] = n(ch, 1, 5, s=0.45)
    return w


def make_block(seed, hidden, heads, dim, *, std=0.02) -> BlockWeights:
    gen = torch.Generator().manual_seed(seed)
    inner = heads * dim
    qkv = torch.randn(3 * inner, hidden, generator=gen) * std
    out = torch.randn(hidden, inner, generator=gen) * std
    qn = 1.0 + torch.randn(dim, generator=gen) * 0.1
    kn = 1.0 + torch.randn(dim, generator=gen) * 0.1
    branch = make_branch_weights(gen, hidden, heads, dim, std=std)
    return BlockWeights(qkv=qkv, q_norm=qn, k_norm=kn, out=out, branch=branch)


def make_x(seed, seq, hidden) -> torch.Tensor:
    gen = torch.Generator().manual_seed(seed + 7919)
    return torch.randn(seq, hidden, generator=gen)


def make_kernel_inputs(seed, lay: Layout, heads, dim):
    """Config-0 kernel-level inputs: q,k,v ~ N(0,1) with k L2-normalised per head,
    beta = sigmoid(N(0,1)) [F,H,tpf], alpha = sigmoid(N(2,1)) [F,H,D],
    gate = sigmoid(N(0,1)) [S,H,1]."""
    gen = torch.Generator().manual_seed(seed)
    s = lay.seq_len
    q = torch.randn(s, heads, dim, generator=gen)
    k = torch.randn(s, heads, dim, generator=gen)
    k = k / k.norm(dim=-1, keepdim=True)
    v = torch.randn(s, heads, dim, generator=gen)
    beta = torch.sigmoid(torch.randn(lay.num_frames, heads, lay.tokens_per_frame, generator=gen))
    alpha = torch.sigmoid(torch.randn(lay.num_frames, heads, dim, generator=gen) + 2.0)
    gate = torch.sigmoid(torch.randn(s, heads, 1, generator=gen))
    return dict(q=q, k=k, v=v, beta=beta, alpha=alpha, gate=gate)


CONFIG0 = dict(text=32, frames=15, grid=(4, 4), heads=4, dim=64, hidden=256)
CONFIG1 = dict(text=512, frames=31, grid=(38, 22), heads=40, dim=128, hidden=5120)
CONFIG3 = dict(text=512, frames=31, grid=(80, 48), heads=40, dim=128, hidden=5120)


def config_layout(cfg: dict, **kw) -> Layout:
    return make_layout(cfg["text"], cfg["frames"], cfg["grid"], **kw)


def attention_pairs(lay: Layout) -> int:
    """Allowed (query, key) pairs per head (used for the algorithmic FLOP count)."""
    return int(key_count_per_row(lay.seq_len, lay.video_start, lay.video_end, lay.num_frames,
                                 lay.tokens_per_frame, list(lay.bounds), lay.anchor_frames).sum())


def block_flops(lay: Layout, heads, dim, hidden, *, branch=True) -> dict:
    """Algorithmic FLOPs of one block forward (allowed attention pairs only)."""
    s = lay.seq_len
    inner = heads * dim
    fl = {}
    fl["attention"] = 4.0 * attention_pairs(lay) * dim * heads
    fl["qkv"] = 2.0 * s * hidden * 3 * inner
    fl["out_proj"] = 2.0 * s * inner * hidden
    fl["gates"] = 2.0 * s * hidden * heads
    if branch and not lay.full_cover:
        fb = lay.num_frames - 2 if lay.anchor_frames == "both" else lay.num_frames
        rows = fb * lay.tokens_per_frame
        tpf = lay.tokens_per_frame
        fl["to_out_linear"] = 2.0 * rows * inner * hidden
        fl["branch_gates"] = 2.0 * rows * hidden * (heads + 2 * dim) + 2.0 * rows * dim * inner
        fl["frame_stats"] = 2.0 * 2 * fb * heads * tpf * dim * dim
        fl["factor"] = (fb + 1) * heads * (dim ** 3) * 3.0
        fl["scan"] = 2.0 * 2 * fb * heads * dim ** 3
        fl["readout"] = 2.0 * rows * heads * dim * dim
    fl["total"] = sum(fl.values())
    return fl


# ---------------------------------------------------------------------------------------
# DiT block around the hybrid attention (block_kernels.py:85-240)
# ---------------------------------------------------------------------------------------

MOD_NAMES = ("shift_msa", "scale_msa", "gate_msa", "shift_mlp", "scale_mlp", "gate_mlp")


@dataclass
class DiTWeights:
    """One MiniMax-H3 DiT block: its attention block plus norm1/norm2 and the MLP."""

    attn: BlockWeights
    norm1: torch.Tensor  # [hidden]
    norm2: torch.Tensor  # [hidden]
    fc1: torch.Tensor  # [2F, hidden] (SwiGLU: gate rows then up rows) or [F, hidden] (GELU)
    fc1_b: torch.Tensor | None
    fc2: torch.Tensor  # [hidden, F]
    fc2_b: torch.Tensor | None
    eps: float = 1e-6


def segment_rows(segments, rows) -> torch.Tensor:
    """Modulation row index of every token (block_kernels.py:34-60, int segments)."""
    ids = torch.empty(rows, dtype=torch.long)
    covered = 0
    for start, stop, row in segments:
        if start != covered or stop < start or stop > rows:
            raise ValueError("MiniMax-H3 modulation segments must cover the sequence contiguously")
        ids[start:stop] = int(row)
        covered = stop
    if covered != rows:
        raise ValueError(f"MiniMax-H3 modulation segments cover {covered}/{rows} rows")
    return ids


def dit_pre(x, weight, eps, scale, shift, idx):
    """RMSNorm(x) * weight * (1 + scale[idx]) + shift[idx] (block_kernels.py:85-89)."""
    return rms_norm(_t(x), weight, eps) * (1.0 + _t(scale)[idx]) + _t(shift)[idx]


def dit_post(residual, gate, idx, branch_out):
    """residual + gate[idx] * branch_out (block_kernels.py:92-93)."""
    return _t(residual) + _t(gate)[idx] * _t(branch_out)


def dit_mlp(h, dw: DiTWeights, activation="swiglu", precision="bf16"):
    """fc2(act(fc1(h))): SwiGLU silu(gate) * up over fc1's two row halves
    (block_kernels.py:113-146), or GELU (erf) over one fc1."""
    a = project(h, dw.fc1, precision)
    if dw.fc1_b is not None:
        a = a + _t(dw.fc1_b)
    if activation == "swiglu":
        gate, up = a.chunk(2, dim=-1)
        a = F.silu(gate) * up
    elif activation == "gelu":
        a = F.gelu(a)
    else:
        raise ValueError(f"unknown MLP activation {activation!r}")
    out = project(a, dw.fc2, precision)
    if dw.fc2_b is not None:
        out = out + _t(dw.fc2_b)
    return out


def dit_block_forward(x, dw: DiTWeights, mods, idx, lay: Layout, heads, dim, cfg: BranchConfig, *,
                      activation="swiglu", precision="bf16", mlp_precision=None, rope_freqs=None):
    """The fused DiT block forward of block_kernels.py:149-240: pre-norm + AdaLN, hybrid
    attention, gated residual, pre-norm + AdaLN, MLP, gated residual.  ``mods`` are the six
    adaln_proj outputs [rows of modulation, hidden] in MOD_NAMES order."""
    shift_msa, scale_msa, gate_msa, shift_mlp, scale_mlp, gate_mlp = mods
    x = _t(x)
    h = dit_pre(x, dw.norm1, dw.eps, scale_msa, shift_msa, idx)
    attn_out = block_forward(h, dw.attn, lay, heads, dim, cfg, precision=precision, rope_freqs=rope_freqs)
    x = dit_post(x, gate_msa, idx, attn_out)
    h = dit_pre(x, dw.norm2, dw.eps, scale_mlp, shift_mlp, idx)
    return dit_post(x, gate_mlp, idx, dit_mlp(h, dw, activation, mlp_precision or precision))


def make_dit(seed, hidden, heads, dim, ffn, *, activation="swiglu", std=0.02, bias=True) -> DiTWeights:
    gen = torch.Generator().manual_seed(seed + 104729)
    rows1 = 2 * ffn if activation == "swiglu" else ffn
    return DiTWeights(
        attn=make_block(seed, hidden, heads, dim, std=std),
        norm1=1.0 + 0.1 * torch.randn(hidden, generator=gen),
        norm2=1.0 + 0.1 * torch.randn(hidden, generator=gen),
        fc1=torch.randn(rows1, hidden, generator=gen) * std,
        fc1_b=torch.randn(rows1, generator=gen) * 0.02 if bias else None,
        fc2=torch.randn(hidden, ffn, generator=gen) * std,
        fc2_b=torch.randn(hidden, generator=gen) * 0.02 if bias else None,
    )


def make_mods(seed, groups, hidden) -> list[torch.Tensor]:
    """Six adaln tables [groups, hidden]: shifts and scales ~ N(0, 0.1), gates ~ N(1, 0.1)."""
    gen = torch.Generator().manual_seed(seed + 15485863)
    out = []
    for name in MOD_NAMES:
        t = torch.randn(groups, hidden, generator=gen) * 0.1
        if name.startswith("gate"):
            t = t + 1.0
        out.append(t)
    return out


def dit_flops(lay: Layout, heads, dim, hidden, ffn, activation="swiglu") -> dict:
    """Algorithmic FLOPs of one DiT block forward: the hybrid attention block plus the MLP."""
    fl = dict(block_flops(lay, heads, dim, hidden))
    s = lay.seq_len
    rows1 = 2 * ffn if activation == "swiglu" else ffn
    fl["mlp"] = 2.0 * s * hidden * rows1 + 2.0 * s * ffn * hidden
    fl["total"] = fl["total"] + fl["mlp"]
    return fl
