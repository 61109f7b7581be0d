"""CPU tests of the ComfyUI PackedLayout adapter (layout.py:72-196 semantics and messages):
extra global segments (audio, reference frames, keyframes) around the video, odd latent
grids padded before the 2x2 patchify, and every rejection the reference raises."""

from __future__ import annotations

import types

import pytest
import torch

from __graft_entry__ import load_package

pkg = load_package()


def _packed(text=32, t=5, h=8, w=10, audio=12, order=("text", "audio", "video", "ref"), ref_rows=None):
    gh, gw = (h + 1) // 2, (w + 1) // 2
    sizes = {"text": text, "audio": audio, "video": t * gh * gw, "ref": ref_rows if ref_rows is not None else gh * gw}
    segs, pos = [], 0
    for kind in order:
        segs.append((pos, pos + sizes[kind], kind))
        pos += sizes[kind]
    return types.SimpleNamespace(signature=(text, t, h, w, audio), segments=segs, seq_len=pos)


def test_packed_layout_with_global_segments_around_the_video():
    p = _packed()
    lay = pkg.from_comfy_packed_layout(p, radius=1, chunk=0, anchor_frames="rows")
    assert (lay.text_start, lay.text_len) == (0, 32)
    assert (lay.video_start, lay.video_end) == (44, 44 + 5 * 20)
    assert lay.seq_len == 44 + 100 + 20 and lay.frame_size == (4, 5) and lay.tokens_per_frame == 20
    assert lay.bounds == tuple(pkg.window_bounds(5, 1, 0)) and not lay.full_cover
    assert lay.anchor_frames == "rows"
    # video first, text last
    p2 = _packed(order=("video", "audio", "text"))
    lay2 = pkg.from_comfy_packed_layout(p2)
    assert lay2.video_start == 0 and lay2.text_start == 100 + 12


def test_odd_latent_grid_is_padded_before_patchify():
    lay = pkg.from_comfy_packed_layout(_packed(h=7, w=9))
    assert lay.frame_size == (4, 5)


@pytest.mark.parametrize("mutate,exc,msg", [
    (lambda p: setattr(p, "signature", (32, 5, 8, 10)), ValueError, "must be"),
    (lambda p: setattr(p, "segments", p.segments + [(0, 1, "text")]), ValueError, "exactly one 'text'"),
    (lambda p: setattr(p, "segments", [s for s in p.segments if s[2] != "video"]), ValueError, "exactly one 'video'"),
    (lambda p: setattr(p, "segments", p.segments + [(3,)]), TypeError, "invalid PackedLayout segment"),
    (lambda p: setattr(p, "seq_len", 50), ValueError, "extends past"),
    (lambda p: setattr(p, "signature", (31, 5, 8, 10, 12)), ValueError, "text segment length"),
    (lambda p: setattr(p, "signature", (32, 3, 8, 10, 12)), ValueError, "not divisible"),
    (lambda p: setattr(p, "signature", (32, 5, 8, 12, 12)), ValueError, "does not match"),
    (lambda p: setattr(p, "signature", (32, 0, 8, 10, 12)), ValueError, "invalid PackedLayout"),
])
def test_packed_layout_rejections(mutate, exc, msg):
    p = _packed()
    mutate(p)
    with pytest.raises(exc, match=msg):
        pkg.from_comfy_packed_layout(p)


def test_packed_layout_argument_checks():
    with pytest.raises(TypeError, match="compatible"):
        pkg.from_comfy_packed_layout(object())
    with pytest.raises(ValueError, match="radius"):
        pkg.from_comfy_packed_layout(_packed(), radius=-1)
    with pytest.raises(ValueError, match="chunk"):
        pkg.from_comfy_packed_layout(_packed(), chunk=True)
    with pytest.raises(ValueError, match="anchor_frames"):
        pkg.from_comfy_packed_layout(_packed(), anchor_frames="middle")


def test_layout_from_payload_uses_the_matching_payload_layout():
    p = _packed(t=5, h=8, w=10, audio=12)
    video = torch.zeros(1, 16, 5, 8, 10)
    audio = torch.zeros(1, 8, 12)
    context = torch.zeros(1, 32, 64)
    lay = pkg.layout_from_payload({"layout": p}, (video, audio), context, {"radius": 2, "chunk": 0})
    assert lay.bounds == tuple(pkg.window_bounds(5, 2, 0))
    # a payload layout whose signature disagrees must be rebuilt, which needs ComfyUI here
    with pytest.raises(RuntimeError, match="PackedLayout is unavailable"):
        pkg.layout_from_payload({"layout": p}, (torch.zeros(1, 16, 6, 8, 10), audio), context, {})
    with pytest.raises(TypeError, match="expected x="):
        pkg.layout_from_payload({}, (video,), context, {})


@pytest.mark.parametrize("rows", [1, 100, 127, 128, 129, 992, 26428, 119552])
@pytest.mark.parametrize("chunks", [1, 2, 4, 7])
def test_streamer_row_blocks_tile_rows_on_gemm_tiles(rows, chunks):
    from vdn_b200.host_io import row_blocks

    blocks = row_blocks(rows, chunks)
    assert blocks[0][0] == 0 and blocks[-1][1] == rows and len(blocks) <= chunks
    assert all(a1 == b0 for (_, a1), (b0, _) in zip(blocks, blocks[1:]))
    assert all(r0 % 128 == 0 and r1 > r0 for r0, r1 in blocks)
