"""Packed-sequence geometry for the VDN-H3 hot path (mirrors vdn_h3/layout.py and the
geometry helpers of vdn_h3/window.py).

The layout is request-local: ``publish_layout`` sets it in a ``ContextVar`` for one
diffusion forward and every patched block reads it with ``current_layout``
(layout.py:44-69), so concurrent or nested requests never see each other's geometry.
"""

from __future__ import annotations

from contextlib import contextmanager
from contextvars import ContextVar
from dataclasses import dataclass, replace
from typing import Iterator

ANCHOR_FRAME_MODES = ("none", "columns", "rows", "both")


def window_bounds(num_frames: int, radius: int, chunk: int = 0) -> list[tuple[int, int]]:
    """Inclusive visible key-frame range per frame (window.py:141-153)."""
    if isinstance(num_frames, bool) or not isinstance(num_frames, int) or num_frames < 0:
        raise ValueError("num_frames must be a non-negative integer")
    if isinstance(radius, bool) or not isinstance(radius, int) or radius < 0:
        raise ValueError("radius must be a non-negative integer")
    if isinstance(chunk, bool) or not isinstance(chunk, int):
        raise ValueError("chunk must be an integer")
    if chunk <= 0:
        return [(f - radius, f + radius) for f in range(num_frames)]
    return [((f // chunk - radius) * chunk, (f // chunk + radius + 1) * chunk - 1) for f in range(num_frames)]


def full_coverage(bounds, num_frames) -> bool:
    """window.py:156-159."""
    if len(bounds) != num_frames:
        raise ValueError("bounds must contain exactly one entry per frame")
    return all(lo <= 0 and hi >= num_frames - 1 for lo, hi in bounds)


def validate_layout(sequence_length, video_start, video_end, num_frames, tokens_per_frame, bounds,
                    anchor_frames) -> None:
    """Same checks and messages as window.py:162-178."""
    if anchor_frames not in ANCHOR_FRAME_MODES:
        raise ValueError(f"anchor_frames={anchor_frames!r}; expected one of {ANCHOR_FRAME_MODES}")
    if num_frames <= 0 or tokens_per_frame <= 0:
        raise ValueError("num_frames and tokens_per_frame must be positive")
    if not 0 <= video_start <= video_end <= sequence_length:
        raise ValueError("video range is outside the packed sequence")
    if video_end - video_start != num_frames * tokens_per_frame:
        raise ValueError("video range does not equal num_frames * tokens_per_frame")
    if len(bounds) != num_frames:
        raise ValueError("bounds must contain exactly one entry per frame")
    for frame, pair in enumerate(bounds):
        if len(pair) != 2:
            raise ValueError(f"bounds[{frame}] must be a (lo, hi) pair")
        lo, hi = pair
        if lo > frame or hi < frame or lo > hi:
            raise ValueError(f"bounds[{frame}]={pair!r} does not contain its query frame")


@dataclass(frozen=True, slots=True)
class VDNLayout:
    """Geometry needed by both branches of Video Delta Attention (layout.py:19-41)."""

    seq_len: int
    video_start: int
    video_end: int
    num_frames: int
    tokens_per_frame: int
    frame_size: tuple[int, int]
    text_start: int
    text_len: int
    bounds: tuple[tuple[int, int], ...] = ()
    full_cover: bool = False
    anchor_frames: str = "both"

    @property
    def frame_height(self) -> int:
        return self.frame_size[0]

    @property
    def frame_width(self) -> int:
        return self.frame_size[1]


CURRENT_LAYOUT: ContextVar[VDNLayout | None] = ContextVar("vdn_b200_layout", default=None)


def current_layout(*, required: bool = True) -> VDNLayout | None:
    layout = CURRENT_LAYOUT.get()
    if required and layout is None:
        raise RuntimeError(
            "VDN-H3 attention ran without a packed layout. Apply the model through "
            "the VDN-H3 node and do not invoke a patched attention block directly."
        )
    return layout


@contextmanager
def publish_layout(layout: VDNLayout) -> Iterator[VDNLayout]:
    if not isinstance(layout, VDNLayout):
        raise TypeError(f"expected VDNLayout, got {type(layout).__name__}")
    token = CURRENT_LAYOUT.set(layout)
    try:
        yield layout
    finally:
        CURRENT_LAYOUT.reset(token)


def make_layout(text_len: int, num_frames: int, grid: tuple[int, int], *, radius: int = 1, chunk: int = 5,
                anchor_frames: str = "both", text_first: bool = True) -> VDNLayout:
    """Layout of a packed [text | video] (or [video | text]) sequence."""
    gh, gw = grid
    tpf = gh * gw
    video = num_frames * tpf
    ts, vs = (0, text_len) if text_first else (video, 0)
    bounds = tuple((int(a), int(b)) for a, b in window_bounds(num_frames, radius, chunk))
    return VDNLayout(seq_len=text_len + video, video_start=vs, video_end=vs + video, num_frames=num_frames,
                     tokens_per_frame=tpf, frame_size=(gh, gw), text_start=ts, text_len=text_len, bounds=bounds,
                     full_cover=full_coverage(bounds, num_frames), anchor_frames=anchor_frames)


def with_window(layout: VDNLayout, *, radius: int, chunk: int) -> VDNLayout:
    bounds = tuple((int(a), int(b)) for a, b in window_bounds(layout.num_frames, radius, chunk))
    return replace(layout, bounds=bounds, full_cover=full_coverage(bounds, layout.num_frames))


# ---------------------------------------------------------------- ComfyUI PackedLayout adapter

def _single_segment(segments, kind: str) -> tuple[int, int]:
    """[start, stop) of the one ``kind`` segment of a PackedLayout (layout.py:72-86)."""
    found = []
    for seg in segments:
        if not isinstance(seg, (tuple, list)) or len(seg) < 3:
            raise TypeError(f"invalid PackedLayout segment {seg!r}")
        if seg[2] == kind:
            found.append((int(seg[0]), int(seg[1])))
    if len(found) != 1:
        raise ValueError(f"expected exactly one {kind!r} segment, got {len(found)}")
    start, stop = found[0]
    if start < 0 or stop <= start:
        raise ValueError(f"invalid {kind!r} segment [{start}, {stop})")
    return start, stop


def _non_negative_int(value, what: str) -> int:
    if isinstance(value, bool) or not isinstance(value, int) or value < 0:
        raise ValueError(f"window {what} must be a non-negative integer, got {value!r}")
    return value


def from_comfy_packed_layout(packed, *, radius: int = 1, chunk: int = 5, anchor_frames: str = "both") -> VDNLayout:
    """VDNLayout of ComfyUI's MiniMax-H3 ``PackedLayout`` (layout.py:106-158): exactly one text
    and one video segment; every other segment (audio, reference frames, keyframes) is a
    global row block that sees and is seen by every row.  ``signature`` = (text_len,
    latent_t, latent_h, latent_w, audio_t) with the latent grid patchified 2x2 (odd sizes
    padded up)."""
    _non_negative_int(radius, "radius")
    _non_negative_int(chunk, "chunk")
    if anchor_frames not in ANCHOR_FRAME_MODES:
        raise ValueError(f"anchor_frames must be one of {sorted(ANCHOR_FRAME_MODES)}, got {anchor_frames!r}")
    try:
        signature = tuple(int(v) for v in packed.signature)
        segments = tuple(packed.segments)
        seq_len = int(packed.seq_len)
    except (AttributeError, TypeError, ValueError) as exc:
        raise TypeError("not a compatible ComfyUI MiniMax-H3 PackedLayout") from exc
    if len(signature) != 5:
        raise ValueError("PackedLayout.signature must be (text_len, latent_t, latent_h, latent_w, audio_t), "
                         f"got {signature!r}")
    text_len, latent_t, latent_h, latent_w, _audio_t = signature
    if min(seq_len, text_len, latent_t, latent_h, latent_w) <= 0:
        raise ValueError(f"invalid PackedLayout signature/length: {signature!r}, seq={seq_len}")
    text_start, text_end = _single_segment(segments, "text")
    video_start, video_end = _single_segment(segments, "video")
    if text_end - text_start != text_len:
        raise ValueError(f"text segment length disagrees with PackedLayout.signature: {text_end - text_start} != "
                         f"{text_len}")
    if video_end > seq_len or text_end > seq_len:
        raise ValueError("a PackedLayout segment extends past the packed sequence")
    rows = video_end - video_start
    if rows % latent_t:
        raise ValueError(f"{rows} video rows are not divisible by {latent_t} latent frames")
    tpf = rows // latent_t
    grid = ((latent_h + 1) // 2, (latent_w + 1) // 2)
    if grid[0] * grid[1] != tpf:
        raise ValueError(f"patched grid {grid[0]}x{grid[1]} does not match {tpf} video tokens per frame")
    bounds = tuple((int(a), int(b)) for a, b in window_bounds(latent_t, radius, chunk))
    return VDNLayout(seq_len=seq_len, video_start=video_start, video_end=video_end, num_frames=latent_t,
                     tokens_per_frame=tpf, frame_size=grid, text_start=text_start, text_len=text_len, bounds=bounds,
                     full_cover=full_coverage(bounds, latent_t), anchor_frames=anchor_frames)


def layout_from_payload(payload, x, context, config) -> VDNLayout:
    """The layout of the PackedLayout native H3 consumes for this input (layout.py:161-196):
    the payload's own layout when its signature matches x = (video [B,C,T,H,W], audio
    [..., T]) and context [B, text, hidden], else one rebuilt with ComfyUI's PackedLayout."""
    payload = payload or {}
    packed = payload.get("layout")
    try:
        video, audio = x[0], x[1]
        text_len = int(context.shape[1])
        latent_t, latent_h, latent_w = (int(v) for v in video.shape[2:5])
        audio_t = int(audio.shape[-1])
    except (IndexError, AttributeError, TypeError, ValueError) as exc:
        raise TypeError("VDN-H3 expected x=(video[B,C,T,H,W], audio[...,T]) and context[B,text,hidden]") from exc
    signature = (text_len, latent_t, (latent_h + 1) // 2 * 2, (latent_w + 1) // 2 * 2, audio_t)
    if packed is None or tuple(getattr(packed, "signature", ())) != signature:
        try:
            from comfy.ldm.minimax.model import PackedLayout
        except ImportError as exc:
            raise RuntimeError("minimax_payload has no layout matching this input and ComfyUI's MiniMax-H3 "
                               "PackedLayout is unavailable") from exc
        packed = PackedLayout(*signature, keyframes=payload.get("keyframes"), refs=payload.get("refs"))
    return from_comfy_packed_layout(packed, radius=int(config.get("radius", 1)), chunk=int(config.get("chunk", 5)),
                                    anchor_frames=str(config.get("anchor_frames", "both")))
