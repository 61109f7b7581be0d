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
