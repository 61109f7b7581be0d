"""Pin the float64 oracle against golden vectors produced by the reference itself.

The fixture ``tests/golden/config0.npz`` holds outputs of the reference's own torch
path (window.py, branch.py, runtime.py, hybrid.py of hyukudan/ComfyUI-Kirei-VDN-H3)
on seeded config-0 inputs; ``tests/golden/make_golden.py`` made it.  Inputs are
rebuilt here from the same seeds and checked by digest first, so a drift of the
torch RNG shows up as a clear failure rather than as a numerical mismatch.
"""

from __future__ import annotations

import os

import numpy as np
import pytest
import torch

from oracle import vdn_oracle as vo

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "config0.npz")


@pytest.fixture(scope="module")
def golden():
    return dict(np.load(GOLDEN))


@pytest.fixture(scope="module")
def setup():
    c = vo.CONFIG0
    lay = vo.config_layout(c)
    ki = vo.make_kernel_inputs(0, lay, c["heads"], c["dim"])
    return c, lay, ki


def _close(got, want, rtol, atol):
    got = got.detach().cpu().numpy() if isinstance(got, torch.Tensor) else got
    np.testing.assert_allclose(got, want, rtol=rtol, atol=atol)


def test_inputs_are_the_golden_inputs(golden, setup):
    from tests.golden.make_golden import tensor_digest

    _, _, ki = setup
    assert str(golden["input_digest"]) == tensor_digest(ki["q"], ki["k"], ki["v"], ki["beta"], ki["alpha"])


@pytest.mark.parametrize("mode", vo.ANCHOR_MODES)
def test_window_attention_matches_reference(golden, setup, mode):
    c, lay, ki = setup
    got = vo.window_attention(ki["q"], ki["k"], ki["v"], lay.video_start, lay.video_end,
                              lay.num_frames, lay.tokens_per_frame, list(lay.bounds),
                              c["dim"] ** -0.5, mode)
    if mode != "both":
        got = got[::4]
    _close(got, golden[f"window_{mode}"], 2e-5, 2e-6)


def test_window_sliding_geometry_matches_reference(golden):
    lay2 = vo.Layout(seq_len=24 + 9 * 16 + 8, video_start=24, video_end=24 + 9 * 16,
                     num_frames=9, tokens_per_frame=16, frame_size=(4, 4), text_start=0,
                     text_len=24, bounds=tuple(vo.window_bounds(9, 2, 0)), anchor_frames="columns")
    ki2 = vo.make_kernel_inputs(5, lay2, 2, 64)
    got = vo.window_attention(ki2["q"], ki2["k"], ki2["v"], lay2.video_start, lay2.video_end,
                              9, 16, list(lay2.bounds), 64 ** -0.5, "columns")
    _close(got, golden["window_sliding_columns"], 2e-5, 2e-6)


def _branch_inputs(setup):
    c, lay, ki = setup
    heads, dim = c["heads"], c["dim"]
    fb, tpf = lay.num_frames - 2, lay.tokens_per_frame
    inner = slice(lay.video_start + tpf, lay.video_end - tpf)
    kf = ki["k"][inner].reshape(fb, tpf, heads, dim).permute(0, 2, 1, 3)
    vf = ki["v"][inner].reshape(fb, tpf, heads, dim).permute(0, 2, 1, 3)
    text = torch.randn(heads, dim, dim, generator=torch.Generator().manual_seed(11)) * 0.1
    bounds_b = [(lo - 1, hi - 1) for lo, hi in lay.bounds[1:-1]]
    return kf, vf, ki["beta"][1:-1], ki["alpha"][1:-1], text, bounds_b


def test_statistics_factor_scan_gather_match_reference(golden, setup):
    kf, vf, beta, alpha, text, bounds_b = _branch_inputs(setup)
    a, b = vo.frame_statistics(kf, vf, beta)
    _close(a[:4, 1], golden["stats_A_f03_h1"], 1e-5, 1e-5)
    _close(b[:4, 1], golden["stats_B_f03_h1"], 1e-5, 1e-5)
    trans, inj = vo.factor_apply(alpha, a, b)
    _close(trans[0], golden["inverse_T_f0"], 1e-4, 2e-6)
    _close(inj[0], golden["inj_f0"], 1e-4, 2e-6)
    prefix, suffix = vo.run_scans(trans, inj, vo._t(text))
    _close(prefix[-1], golden["prefix_last"], 1e-4, 1e-5)
    _close(suffix[0], golden["suffix_first"], 1e-4, 1e-5)
    state = vo.gather_linear_state(prefix, suffix, vo._t(alpha), bounds_b, "alpha", vo._t(text))
    # the reference gathers in fp32; its output moves by ~1.5e-5 with the CPU thread count
    _close(state[::2, 0], golden["state_h0"], 1e-4, 3e-5)
    state_nt = vo.gather_linear_state(prefix, suffix, vo._t(alpha), bounds_b, "alpha", None)
    _close(state_nt[1::3, 1], golden["state_notext_h1"], 1e-4, 1e-5)


def test_sana_factor_and_scans_match_reference(golden, setup):
    """delta_rule="sana_scaled": T = diag(alpha) (I - A/L), Inj = B/sqrt(L) (branch.py:163-177)."""
    c, lay, _ = setup
    kf, vf, beta, alpha, text, _ = _branch_inputs(setup)
    a, b = vo.frame_statistics(kf, vf, beta)
    trans, inj = vo.sana_factor_apply(alpha, a, b, lay.tokens_per_frame)
    _close(trans[0], golden["sana_T_f0"], 1e-5, 1e-6)
    _close(inj[0], golden["sana_inj_f0"], 1e-5, 1e-6)
    prefix, suffix = vo.run_scans(trans, inj, vo._t(text))
    _close(prefix[-1], golden["sana_prefix_last"], 1e-4, 1e-5)
    _close(suffix[0], golden["sana_suffix_first"], 1e-4, 1e-5)


def test_sana_block_forward_matches_reference(golden, setup):
    c, lay, _ = setup
    bw = vo.make_block(0, c["hidden"], c["heads"], c["dim"])
    x = vo.make_x(0, lay.seq_len, c["hidden"])
    out = vo.block_forward(x, bw, lay, c["heads"], c["dim"], vo.BranchConfig(delta_rule="sana_scaled"))
    _close(out, golden["sana_block_out"], 1e-4, 2e-6)
    # the two rules really differ on this input
    assert np.abs(golden["sana_block_out"] - golden["block_out"]).max() > 1e-3


def test_conv_features_match_reference(golden, setup):
    c, lay, ki = setup
    bw = vo.make_block(0, c["hidden"], c["heads"], c["dim"])
    w = bw.branch
    got = vo.conv_features(ki["k"][lay.video_start:lay.video_end], w["short_conv.k_sp.weight"],
                           w["short_conv.k_tm.weight"], lay.num_frames, lay.frame_size, True)
    _close(got[3], golden["conv_k_f3"], 1e-5, 1e-6)


def test_block_forward_matches_reference(golden, setup):
    c, lay, _ = setup
    bw = vo.make_block(0, c["hidden"], c["heads"], c["dim"])
    x = vo.make_x(0, lay.seq_len, c["hidden"])
    out, parts = vo.block_forward(x, bw, lay, c["heads"], c["dim"], vo.BranchConfig(), return_parts=True)
    _close(out, golden["block_out"], 1e-4, 2e-6)
    delta = torch.zeros(lay.video_end - lay.video_start, c["hidden"], dtype=torch.float64)
    delta[:] = parts["delta"]
    _close(delta, golden["branch_delta"], 1e-4, 2e-6)
    # skip_ends: the anchor frames get no branch contribution (runtime.py:603-607).
    tpf = lay.tokens_per_frame
    assert float(parts["delta"][:tpf].abs().max()) == 0.0
    assert float(parts["delta"][-tpf:].abs().max()) == 0.0


def test_window_geometry_known_answers():
    # Known answers of the reference's own geometry tests (tests/test_window.py:193-202).
    assert vo.window_bounds(4, 1) == [(-1, 1), (0, 2), (1, 3), (2, 4)]
    assert vo.window_bounds(6, 1, 5)[0] == (-5, 9)
    assert vo.window_bounds(6, 1, 5)[5] == (0, 14)
    assert vo.full_coverage(vo.window_bounds(6, 1, 5), 6)
    assert not vo.full_coverage(vo.window_bounds(16, 1, 5), 16)


def test_int8_scheme_is_exact_integer_arithmetic():
    gen = torch.Generator().manual_seed(3)
    x = torch.randn(37, 256, generator=gen).to(torch.bfloat16).float()
    w = torch.randn(48, 256, generator=gen) * 0.02
    qa, sa = vo.int8_quantize_rows(x)
    qw, sw = vo.int8_quantize_weight(w)
    assert qa.dtype == torch.int8 and int(qa.abs().max()) <= 127
    acc = vo.int8_accumulate(qa, qw)
    want = (qa.double() @ qw.double().T)
    assert torch.equal(acc.double(), want)
    # The dequantised product approximates the float product within int8 resolution.
    approx = acc.double() * sa.double()[:, None] * sw.double()[None, :]
    exact = x.double() @ w.double().T
    rel = (approx - exact).norm() / exact.norm()
    assert rel < 2e-2


def test_convrot_rotation_is_the_regular_hadamard_group_rotation():
    """ConvRot (projection.py:74-97, :243-256; comfy-kitchen, unpinned): the staged fp32
    rotation equals the explicit block-diagonal R/16, R = (J - 2I)^(x4), which is symmetric
    and orthogonal, so rotating both operands leaves x W^T unchanged."""
    r4 = np.ones((4, 4)) - 2 * np.eye(4)
    r = r4
    for _ in range(3):
        r = np.kron(r, r4)
    h = r / 16
    assert np.allclose(h, h.T) and np.allclose(h @ h, np.eye(256))
    assert np.allclose(h.sum(axis=1), h[0].sum())  # regular: equal row sums
    gen = torch.Generator().manual_seed(5)
    x = torch.randn(9, 768, generator=gen)
    w = torch.randn(11, 768, generator=gen)
    xr = vo.convrot_rotate(x)
    blocks = [x.double().numpy()[:, g * 256:(g + 1) * 256] @ h for g in range(3)]
    np.testing.assert_allclose(xr, np.concatenate(blocks, 1), rtol=0, atol=2e-6)
    wr = vo.convrot_rotate(w)
    np.testing.assert_allclose(xr.astype(np.float64) @ wr.astype(np.float64).T,
                               x.double().numpy() @ w.double().numpy().T, rtol=0, atol=2e-4)
    with pytest.raises(ValueError):
        vo.convrot_rotate(torch.zeros(2, 320))


def test_convrot_int8_is_exact_integer_arithmetic_and_beats_plain_on_outliers():
    gen = torch.Generator().manual_seed(6)
    x = torch.randn(64, 1024, generator=gen)
    x[:, 3] *= 200
    x = x.to(torch.bfloat16).float()
    w = torch.randn(48, 1024, generator=gen) * 0.02
    qa, sa = vo.int8_quantize_rows_convrot(x)
    qw, sw = vo.int8_quantize_rows_convrot(w)
    assert qa.dtype == torch.int8 and int(qa.abs().max()) == 127
    assert torch.equal(vo.int8_accumulate(qa, qw).double(), qa.double() @ qw.double().T)
    exact = x.double() @ w.double().T
    e_rot = float((vo.project_int8_convrot(x, w) - exact).norm() / exact.norm())
    e_plain = float((vo.project(x, w, "int8") - exact).norm() / exact.norm())
    assert e_rot < 0.5 * e_plain


def test_block_composition_mirrors_the_reference_hybrid_tests():
    """tests/test_hybrid.py:107-189: with a zero softmax gate (sigmoid(0) = 1/2) the block is half
    the ungated block, and the branch delta changes the video rows only."""
    c = vo.CONFIG0
    lay = vo.config_layout(c)
    H, D, hidden = c["heads"], c["dim"], c["hidden"]
    bw = vo.make_block(0, hidden, H, D)
    x = vo.make_x(0, lay.seq_len, hidden)
    cfg = vo.BranchConfig()
    zero_gate = dict(bw.branch, **{"softmax_gate.up.weight": torch.zeros(H, hidden),
                                   "softmax_gate.up.bias": torch.zeros(H)})
    bw0 = vo.BlockWeights(bw.qkv, bw.q_norm, bw.k_norm, bw.out, zero_gate)
    gated = vo.block_forward(x, bw0, lay, H, D, cfg, enable_softmax_gate=True, linear_enabled=False)
    plain = vo.block_forward(x, bw0, lay, H, D, cfg, enable_softmax_gate=False, linear_enabled=False)
    torch.testing.assert_close(gated, 0.5 * plain, rtol=1e-12, atol=1e-12)
    on = vo.block_forward(x, bw, lay, H, D, cfg)
    off = vo.block_forward(x, bw, lay, H, D, cfg, linear_enabled=False)
    vs, ve = lay.video_start, lay.video_end
    assert torch.equal(on[:vs], off[:vs]) and torch.equal(on[ve:], off[ve:])
    changed = (on[vs:ve] - off[vs:ve]).abs().amax(dim=1) > 0
    tpf = lay.tokens_per_frame
    # skip_ends (anchors "both"): frames 0 and F-1 carry no delta (runtime.py:576-585)
    assert not changed[:tpf].any() and not changed[-tpf:].any()
    assert changed[tpf:-tpf].all()


def test_short_conv_k_features_have_unit_norm():
    """tests/test_branch.py:130-146: after the spatial + temporal conv and SiLU, every k feature
    vector is L2-normalised per head (v features are not)."""
    c = vo.CONFIG0
    lay = vo.config_layout(c)
    H, D = c["heads"], c["dim"]
    w = vo.make_branch_weights(torch.Generator().manual_seed(1), c["hidden"], H, D)
    rows = lay.num_frames * lay.tokens_per_frame
    tok = torch.randn(rows, H, D, generator=torch.Generator().manual_seed(2))
    k = vo.conv_features(tok, w["short_conv.k_sp.weight"], w["short_conv.k_tm.weight"], lay.num_frames,
                         lay.frame_size, True)
    assert k.shape == (lay.num_frames, H, lay.tokens_per_frame, D)
    torch.testing.assert_close(k.norm(dim=-1), torch.ones(k.shape[:-1], dtype=k.dtype), rtol=0, atol=1e-9)
    v = vo.conv_features(tok, w["short_conv.v_sp.weight"], w["short_conv.v_tm.weight"], lay.num_frames,
                         lay.frame_size, False)
    assert not torch.allclose(v.norm(dim=-1), torch.ones(v.shape[:-1], dtype=v.dtype))


def test_branch_with_skip_ends_zeroes_the_end_frames_and_stays_finite():
    """tests/test_branch.py:163-194: with skip_ends the rows of frames 0 and F-1 are zero and the
    rest finite."""
    c = vo.CONFIG0
    lay = vo.config_layout(c)
    H, D, hidden = c["heads"], c["dim"], c["hidden"]
    bw = vo.make_block(0, hidden, H, D)
    x = vo.make_x(0, lay.seq_len, hidden)
    ki = vo.make_kernel_inputs(0, lay, H, D)
    vs, ve, tpf = lay.video_start, lay.video_end, lay.tokens_per_frame
    out = vo.branch_readout(bw.branch, x[vs:ve], ki["q"][vs:ve], ki["k"][vs:ve], ki["v"][vs:ve], lay.num_frames, tpf,
                            list(lay.bounds), lay.frame_size, H, D, vo.BranchConfig(), skip_ends=True)
    assert out.shape == (ve - vs, H * D)
    assert torch.count_nonzero(out[:tpf]) == 0 and torch.count_nonzero(out[-tpf:]) == 0
    assert torch.isfinite(out).all()
    # an interior frame reads the states before and after its window; a window that spans the
    # whole clip (frames 1 .. F-2 after skip_ends) leaves none, so without text state it is zero
    F = lay.num_frames
    for f in range(1, F - 1):
        lo, hi = lay.bounds[f]
        rows = out[f * tpf:(f + 1) * tpf]
        if lo <= 1 and hi >= F - 2:
            assert torch.count_nonzero(rows) == 0, f
        else:
            assert (rows.abs().amax(dim=1) > 0).all(), f


@pytest.mark.parametrize("anchors", ["none", "columns", "rows", "both"])
def test_grouped_attention_and_row_subsets_equal_the_dense_oracle(anchors):
    """The gathered-key spelling of the window softmax (the reference's grouped backend,
    window.py:277-313) and a row-restricted block equal the dense masked oracle."""
    c = vo.CONFIG0
    lay = vo.config_layout(c, anchor_frames=anchors)
    bw = vo.make_block(0, c["hidden"], c["heads"], c["dim"])
    x = vo.make_x(0, lay.seq_len, c["hidden"])
    dense = vo.block_forward(x, bw, lay, c["heads"], c["dim"], vo.BranchConfig())
    grouped = vo.block_forward(x, bw, lay, c["heads"], c["dim"], vo.BranchConfig(), attention="grouped")
    assert float((dense - grouped).abs().max()) < 1e-12
    rows = torch.tensor([271, 0, 5, 31, 32, 40, 100, 200])  # text, anchors, interior; unsorted
    sub = vo.block_forward(x, bw, lay, c["heads"], c["dim"], vo.BranchConfig(), attention="grouped", rows=rows)
    assert float((dense[rows] - sub).abs().max()) < 1e-12
