"""CPU tests of the DiT block's host logic (no GPU): modulation segments -> row groups
(block_kernels.py:34-60 semantics and error messages), the index cache, the SwiGLU row
interleave that lets one GEMM tile hold a gate block and its up block, and the oracle's
block restatement on its own terms (the MLP with zero gates leaves the stream untouched)."""

from __future__ import annotations

import pytest
import torch

from __graft_entry__ import load_package
from oracle import vdn_oracle as vo

pkg = load_package()
from vdn_b200 import dit as bdit  # noqa: E402


def test_segment_indices_follow_the_reference_rules():
    segs = [(0, 3, 0), (3, 7, torch.tensor(2)), (7, 10, torch.tensor([1, 1, 0]))]
    got = bdit.segment_indices(segs, 10, "cpu")
    assert got.dtype == torch.int32
    assert got.tolist() == [0, 0, 0, 2, 2, 2, 2, 1, 1, 0]
    assert torch.equal(vo.segment_rows([(0, 3, 0), (3, 10, 1)], 10), torch.tensor([0] * 3 + [1] * 7))
    with pytest.raises(ValueError, match="contiguously"):
        bdit.segment_indices([(0, 3, 0), (4, 10, 1)], 10, "cpu")
    with pytest.raises(ValueError, match="cover 7/10"):
        bdit.segment_indices([(0, 7, 0)], 10, "cpu")
    with pytest.raises(ValueError, match="expected 3"):
        bdit.segment_indices([(0, 7, 0), (7, 10, torch.tensor([1, 2]))], 10, "cpu")


def test_segment_cache_reuses_int_segments_only():
    cache = bdit.SegmentIndexCache(limit=2)
    a = cache.indices([(0, 5, 0), (5, 9, 1)], 9, "cpu")
    assert cache.indices([(0, 5, 0), (5, 9, 1)], 9, "cpu") is a
    t = cache.indices([(0, 9, torch.tensor(1))], 9, "cpu")
    assert t.tolist() == [1] * 9 and len(cache._ids) == 1
    cache.indices([(0, 9, 0)], 9, "cpu")
    cache.indices([(0, 9, 1)], 9, "cpu")
    assert len(cache._ids) == 2  # LRU limit


def test_swiglu_interleave_pairs_gate_and_up_blocks():
    F, K = 384, 3
    w = torch.arange(2 * F * K, dtype=torch.float32).reshape(2 * F, K)
    wi = bdit.interleave_swiglu_rows(w)
    for b in range(F // 128):
        assert torch.equal(wi[256 * b:256 * b + 128], w[128 * b:128 * b + 128])
        assert torch.equal(wi[256 * b + 128:256 * b + 256], w[F + 128 * b:F + 128 * b + 128])
    bias = torch.arange(2 * F, dtype=torch.float32)
    assert torch.equal(bdit.interleave_swiglu_rows(bias).view(-1, 2, 128)[:, 1] - F,
                       bdit.interleave_swiglu_rows(bias).view(-1, 2, 128)[:, 0])
    with pytest.raises(ValueError):
        bdit.interleave_swiglu_rows(torch.zeros(200, 4))


def test_oracle_dit_block_with_zero_gates_is_identity():
    c = vo.CONFIG0
    lay = vo.config_layout(c)
    dw = vo.make_dit(1, c["hidden"], c["heads"], c["dim"], 256, activation="gelu")
    mods = vo.make_mods(1, 2, c["hidden"])
    mods[2] = torch.zeros_like(mods[2])
    mods[5] = torch.zeros_like(mods[5])
    idx = vo.segment_rows([(0, lay.video_start, 0), (lay.video_start, lay.seq_len, 1)], lay.seq_len)
    x = vo.make_x(1, lay.seq_len, c["hidden"])
    y = vo.dit_block_forward(x, dw, mods, idx, lay, c["heads"], c["dim"], vo.BranchConfig(), activation="gelu")
    assert torch.equal(y, x.double())


def test_dit_block_rejects_unsupported_settings():
    fake_attn = type("A", (), {"geo": type("G", (), {"hidden": 8})()})()
    w = torch.zeros(8)
    with pytest.raises(ValueError, match="activation"):
        pkg.B200DiTBlock(fake_attn, w, 1e-6, w, 1e-6, torch.zeros(16, 8), None, torch.zeros(8, 16), None, "cpu",
                         activation="relu")
    with pytest.raises(ValueError, match="bf16 or int8"):
        pkg.B200DiTBlock(fake_attn, w, 1e-6, w, 1e-6, torch.zeros(16, 8), None, torch.zeros(8, 16), None, "cpu",
                         precision="fp8")
    with pytest.raises(ValueError, match="fc1 has"):
        pkg.B200DiTBlock(fake_attn, w, 1e-6, w, 1e-6, torch.zeros(16, 8), None, torch.zeros(8, 16), None, "cpu",
                         activation="swiglu")
