"""CPU tests of the host side: the block-sparse window plan, layout mirrors, the C-ABI
library exports and the deferred Cholesky scope.  No GPU compute is called."""

from __future__ import annotations

import os
import re

import numpy as np
import pytest
import torch

from __graft_entry__ import ROOT, load_package
from oracle import vdn_oracle as vo

pkg = load_package()
from vdn_b200 import window as bw  # noqa: E402
from vdn_b200 import branch as bbr  # noqa: E402


def _expand_plan(plan, S):
    """Emulate the kernel's key-tile walk and mask formula: returns a bool [S, S] matrix
    and asserts that no (row, key) pair is visited twice."""
    vs, ve, F, tpf = plan.video_start, plan.video_end, plan.num_frames, plan.tokens_per_frame
    allowed = np.zeros((S, S), dtype=bool)
    rows_seen = np.zeros(S, dtype=np.int32)
    for qt in range(plan.n_qtiles):
        halves = plan.q_halves(qt)
        assert 1 <= len(halves) <= 2 and all(1 <= n <= bw.BQ // 2 and r0 + n <= S for r0, n in halves)
        rows = np.concatenate([np.arange(r0, r0 + n) for r0, n in halves])
        rows_seen[rows] += 1
        dense = (rows < vs) | (rows >= ve)
        f = np.clip((rows - vs) // tpf, 0, F - 1)
        if plan.anchor_rows:
            dense |= (~dense) & ((f == 0) | (f == F - 1))
        wlo = vs + plan.frame_lo[f] * tpf
        whi = vs + (plan.frame_hi[f] + 1) * tpf
        acol_lo = vs + tpf if plan.anchor_cols else vs
        acol_hi = ve - tpf if plan.anchor_cols else ve
        seen = np.zeros((len(rows), S), dtype=np.int32)
        for t in range(plan.tile_off[qt], plan.tile_off[qt + 1]):
            code = int(plan.ktile[t])
            k0, masked, valid = code >> 9, (code >> 8) & 1, (code & 0xFF) + 1
            keys = np.arange(k0, k0 + valid)
            assert keys.max() < S
            if masked:
                ok = (dense[:, None] | (keys[None] < vs) | (keys[None] >= ve)
                      | ((keys[None] >= wlo[:, None]) & (keys[None] < whi[:, None]))
                      | (keys[None] < acol_lo) | (keys[None] >= acol_hi))
            else:
                ok = np.ones((len(rows), len(keys)), dtype=bool)
            seen[:, keys] += 1
            allowed[rows[:, None], keys[None, :]] |= ok
        assert seen.max() <= 1, "a key tile overlaps another one"
    assert np.all(rows_seen == 1), "query tiles must tile the sequence"
    return allowed


GEOMS = [
    # (text_before, frames, tpf, text_after, radius, chunk)
    (32, 15, 16, 0, 1, 5),
    (4, 11, 3, 2, 1, 3),
    (4, 11, 3, 2, 2, 4),
    (4, 11, 3, 2, 2, 0),
    (24, 9, 16, 8, 2, 0),
    (0, 7, 40, 0, 1, 2),
    (130, 6, 200, 70, 0, 1),
    (512, 31, 836, 0, 1, 5),
]


@pytest.mark.parametrize("geom", GEOMS)
@pytest.mark.parametrize("anchors", vo.ANCHOR_MODES)
@pytest.mark.parametrize("cutting", ["class", "dense"])
def test_window_plan_covers_exactly_the_reference_mask(geom, anchors, cutting):
    before, F, tpf, after, radius, chunk = geom
    vs, ve = before, before + F * tpf
    S = ve + after
    if S > 8192 and anchors != "both":
        pytest.skip("large geometry checked in the released anchor mode only")
    bounds = vo.window_bounds(F, radius, chunk)
    plan = bw.build_window_plan(S, vs, ve, F, tpf, bounds, anchors, cutting=cutting)
    if cutting == "class":
        assert plan.masked_tiles == 0  # every tile's rows share one visible-key set
    if S > 8192:
        # spot-check rows instead of the full [S, S] mask
        got = _expand_plan(plan, S)
        rows = np.unique(np.linspace(0, S - 1, 97).astype(int))
        want = vo.allowed_mask(S, vs, ve, F, tpf, bounds, anchors)[torch.as_tensor(rows)].numpy()
        np.testing.assert_array_equal(got[rows], want)
        return
    got = _expand_plan(plan, S)
    want = vo.allowed_mask(S, vs, ve, F, tpf, bounds, anchors).numpy()
    np.testing.assert_array_equal(got, want)


@pytest.mark.parametrize("long_factor", [None, 1.5, 1.0])
def test_plan_items_sorted_by_cost_and_cover_all_heads(long_factor):
    lay = vo.config_layout(vo.CONFIG0)
    plan = bw.build_window_plan(lay.seq_len, lay.video_start, lay.video_end, lay.num_frames,
                                lay.tokens_per_frame, list(lay.bounds), lay.anchor_frames)
    items = plan.items(4, long_factor)
    assert len(items) == 4 * plan.n_qtiles
    heads = items >> 20
    qts = items & 0xFFFFF
    costs = plan.tiles_per_q[qts]
    assert sorted(zip(heads.tolist(), qts.tolist())) == [(h, q) for h in range(4) for q in range(plan.n_qtiles)]
    # the long items first, head by head; then head-major, longest first per head
    if long_factor is None:
        long_q = np.zeros(plan.n_qtiles, dtype=bool)
    else:
        long_q = plan.tiles_per_q >= long_factor * max(float(np.median(plan.tiles_per_q)), 1.0)
    n_long = 4 * int(long_q.sum())
    assert np.all(long_q[qts[:n_long]]) and not np.any(long_q[qts[n_long:]])
    for lo, hi in ((0, n_long), (n_long, len(items))):
        hh = heads[lo:hi]
        assert np.all(np.diff(hh) >= 0)
        for h in range(4):
            assert np.all(np.diff(costs[lo:hi][hh == h]) <= 0)


def test_plan_at_config1_cuts_query_tiles_at_dense_rows():
    lay = vo.config_layout(vo.CONFIG1)
    plan = bw.build_window_plan(lay.seq_len, lay.video_start, lay.video_end, lay.num_frames,
                                lay.tokens_per_frame, list(lay.bounds), lay.anchor_frames)
    w0, w1 = lay.video_start + lay.tokens_per_frame, lay.video_end - lay.tokens_per_frame
    full = (lay.seq_len + bw.BKV - 1) // bw.BKV
    paired = 0
    for qt in range(plan.n_qtiles):
        halves = plan.q_halves(qt)
        dense = [r0 + n <= w0 or r0 >= w1 for r0, n in halves]
        # no tile mixes rows that see every key with windowed rows
        for (r0, n), d in zip(halves, dense):
            assert d or (w0 <= r0 and r0 + n <= w1), (r0, n)
        assert len(set(dense)) == 1
        if dense[0]:
            assert plan.tiles_per_q[qt] == full
            assert not any((int(c) >> 8) & 1 for c in plan.ktile[plan.tile_off[qt]:plan.tile_off[qt + 1]])
        if len(halves) == 2 and halves[1][0] != halves[0][0] + halves[0][1]:
            paired += 1
    # the 68-row remainders of the front and back every-key segments share one item
    assert paired == 1
    items = plan.items(5, 1.5)
    costs = plan.tiles_per_q[items & 0xFFFFF]
    n_dense = 5 * int((plan.tiles_per_q == full).sum())
    # with a long factor, the text rows and anchor frames (every key visible) lead the queue
    assert np.all(costs[:n_dense] == full) and np.all(costs[n_dense:] < full)


def test_plan_at_config1_is_block_sparse():
    lay = vo.config_layout(vo.CONFIG1)
    plan = bw.build_window_plan(lay.seq_len, lay.video_start, lay.video_end, lay.num_frames,
                                lay.tokens_per_frame, list(lay.bounds), lay.anchor_frames)
    dense_tiles = plan.n_qtiles * ((lay.seq_len + 127) // 128)
    visited = int(plan.tiles_per_q.sum())
    pairs = vo.attention_pairs(lay)
    # visited key tiles carry at most ~12 % more work than the allowed pairs, and far less than dense
    assert visited * bw.BQ * bw.BKV < 1.08 * pairs
    assert visited < 0.6 * dense_tiles
    assert plan.masked_tiles < 0.25 * visited


def test_layout_mirrors_reference_geometry():
    assert pkg.window_bounds(4, 1) == [(-1, 1), (0, 2), (1, 3), (2, 4)]
    assert pkg.window_bounds(6, 1, 5)[0] == (-5, 9)
    assert pkg.full_coverage(pkg.window_bounds(6, 1, 5), 6)
    lay = pkg.make_layout(512, 31, (38, 22))
    assert lay.seq_len == 26428 and lay.video_start == 512 and lay.tokens_per_frame == 836
    with pytest.raises(ValueError):
        pkg.window_bounds(3, -1)
    with pytest.raises(RuntimeError):
        pkg.current_layout()
    with pkg.publish_layout(lay):
        assert pkg.current_layout() is lay
    assert pkg.current_layout(required=False) is None


def test_library_exports_every_declared_symbol():
    header = open(os.path.join(ROOT, "include", "vdn_b200.h")).read()
    declared = set(re.findall(r"^int (vdn_\w+)\(", header, flags=re.M))
    assert declared, "no declarations found"
    lib_path = os.path.join(ROOT, "comfyui-kirei-vdn-h3_b200", "libvdn_b200.so")
    if not os.path.exists(lib_path):
        import __graft_entry__

        __graft_entry__.build()
    lib = pkg._lib.library()
    for name in sorted(declared):
        assert hasattr(lib, name), name
    assert declared == set(pkg._lib.SIGNATURES), "ctypes table and header disagree"
    assert re.search(r"^long long vdn_launch_count\(void\);", header, flags=re.M)
    assert pkg._lib.launch_count() == 0  # nothing launched without a GPU


def test_missing_library_fails_loudly(monkeypatch):
    monkeypatch.setattr(pkg._lib, "_lib", None)
    monkeypatch.setattr(pkg._lib, "LIB_PATH", "/nonexistent/libvdn_b200.so")
    with pytest.raises(RuntimeError, match="no CPU or library fallback"):
        pkg._lib.library()


def test_cpu_tensors_are_rejected():
    q = torch.zeros(16, 2, 64, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="CUDA"):
        pkg.window_softmax_b200(q, q, q, 0, 16, 1, 16, [(0, 0)], 0.125)


def test_deferred_cholesky_scope_reports_factor_and_batch():
    good = torch.zeros(3, 2, dtype=torch.int32)
    bad = torch.zeros(3, 2, dtype=torch.int32)
    bad.view(-1)[3] = 7
    with pytest.raises(torch.linalg.LinAlgError, match="factor 1, batch 3: leading minor of order 7"):
        with bbr.cholesky_runtime_scope() as checks:
            bbr.record_factor_status([good])
            bbr.record_factor_status([bad])
            assert checks.factor_calls == 2
    with bbr.cholesky_runtime_scope() as checks:
        bbr.record_factor_status([good])
    # outside a scope the check is immediate
    with pytest.raises(torch.linalg.LinAlgError):
        bbr.record_factor_status([bad])


def test_factor_status_slots_are_per_call_and_survive_later_blocks():
    """Blocks sharing one workspace each get their own status slot, so a failure in an early
    block is still reported at the scope's exit with its own factor index (the reference's
    fresh cholesky_ex info per call, branch.py:62-71); each call records its text factor before
    its clip factor (branch.py:795-799)."""
    ring = bbr.InfoRing(3, 2, "cpu")  # 2 clip frames + the text frame, 2 heads
    with pytest.raises(torch.linalg.LinAlgError, match="factor 1, batch 3: leading minor of order 5"):
        with bbr.cholesky_runtime_scope() as checks:
            slots = []
            for block in range(3):
                slot = bbr.claim_factor_status(ring)
                slot.zero_()  # the kernel writes every entry of its slot
                if block == 0:
                    slot[1, 1] = 5  # clip frame 1, head 1: batch 1 * 2 + 1 of block 0's clip factor
                bbr.record_factor_status([slot[2:3], slot[:2]], ring, slot)
                slots.append(slot)
            assert len({s.data_ptr() for s in slots}) == 3 and checks.factor_calls == 6
    assert len(ring.free) == ring.CHUNK  # released at the scope's exit
    # a slot recorded outside a scope is validated at once and handed back
    slot = bbr.claim_factor_status(ring)
    slot.zero_()
    bbr.record_factor_status([slot[2:3], slot[:2]], ring, slot)
    assert len(ring.free) == ring.CHUNK


def test_delta_rules_mirror_the_reference_and_unknown_rules_raise():
    assert bbr.DELTA_RULES == ("vdn_solve", "sana_scaled")  # branch.py:180
    w = vo.make_branch_weights(torch.Generator().manual_seed(0), 32, 2, 64)
    assert pkg.B200LinearBranch(w, 2, 64, delta_rule="sana_scaled").delta_rule == "sana_scaled"
    with pytest.raises(ValueError, match="delta rule"):
        pkg.B200LinearBranch(w, 2, 64, delta_rule="gated_delta")
    with pytest.raises(ValueError, match="delta rule"):
        bbr.run_branch(None, None, q_raw=None, k_raw=None, v_raw=None, aux=None, beta_col0=0, ogd_col0=0,
                       ad_col0=0, Fb=1, tpf=1, frame_size=(1, 1), bounds=[(0, 0)], bridge="alpha", out=None,
                       out_row0=0, status=None, delta_rule="gated_delta")


def test_rope_table_accepts_comfy_shapes_and_rejects_others():
    S, D = 10, 64
    f = vo.make_rope_freqs(S, 32)
    t = pkg.rope_table(f.reshape(1, S, 1, 16, 2, 2), S, D, "cpu")
    assert t.rot == 32 and t.ld == 64 and t.freqs.shape == (S, 64) and t.freqs.dtype == torch.float32
    assert torch.equal(t.freqs.reshape(S, 16, 2, 2), f)
    shared = pkg.rope_table(f[:1].reshape(1, 1, 16, 2, 2), S, D, "cpu")
    assert shared.ld == 0 and shared.freqs.shape == (1, 64)
    assert pkg.rope_table(None, S, D, "cpu") is None
    with pytest.raises(ValueError, match="2, 2"):
        pkg.rope_table(torch.zeros(S, 16, 4), S, D, "cpu")
    with pytest.raises(ValueError, match="rot_dim"):
        pkg.rope_table(vo.make_rope_freqs(S, 128), S, D, "cpu")
    with pytest.raises(ValueError, match="one per row"):
        pkg.rope_table(torch.zeros(1, S, 3, 16, 2, 2), S, D, "cpu")  # per-head tables


def test_oracle_rope_is_comfy_rotation_on_split_halves():
    """Split-half RoPE equals ComfyUI's interleaved rotation applied to the features
    reordered (j, j + rot/2) -> (2j, 2j + 1), keeps pair norms and leaves features past rot."""
    S, H, D, rot = 6, 2, 16, 12
    g = torch.Generator().manual_seed(3)
    x = torch.randn(S, H, D, generator=g, dtype=torch.float64)
    f = vo.make_rope_freqs(S, rot, offset=3).double()
    got = vo.rope_split_half(x, f)
    half = rot // 2
    inter = torch.stack([x[..., :half], x[..., half:rot]], -1)  # [S, H, half, 2]
    rotated = (f[:, None] * inter[..., None, :]).sum(-1)  # out_a = sum_b f[a, b] pair_b
    assert torch.allclose(got[..., :half], rotated[..., 0]) and torch.allclose(got[..., half:rot], rotated[..., 1])
    assert torch.equal(got[..., rot:], x[..., rot:])
    assert torch.allclose(got[..., :half] ** 2 + got[..., half:rot] ** 2, x[..., :half] ** 2 + x[..., half:rot] ** 2)


def test_frame_tiles_cover_the_clip_with_halo_sized_buffers():
    assert bbr.frame_tiles(7, None) == [(0, 7)] and bbr.frame_tiles(7, 7) == [(0, 7)]
    assert bbr.frame_tiles(7, 3) == [(0, 3), (3, 6), (6, 7)]
    assert bbr.frame_tiles(5, 1) == [(i, i + 1) for i in range(5)]
    assert bbr.feature_frames(29, None) == 29 and bbr.feature_frames(29, 4) == 8 and bbr.feature_frames(5, 4) == 5
    with pytest.raises(ValueError):
        bbr.frame_tiles(7, 0)
    w = vo.make_branch_weights(torch.Generator().manual_seed(0), 32, 2, 64)
    assert pkg.B200LinearBranch(w, 2, 64, tile_frames=4).tile_frames == 4
    for bad in (-1, 2.5, True):
        with pytest.raises(ValueError, match="tile_frames"):
            pkg.B200LinearBranch(w, 2, 64, tile_frames=bad)


def test_status_codes_map_to_reference_exceptions():
    with pytest.raises(ValueError):
        pkg._lib.check(-1, "x")
    with pytest.raises(ValueError):
        pkg._lib.check(-2, "x")
    with pytest.raises(RuntimeError):
        pkg._lib.check(-3, "x")
    pkg._lib.check(0, "x")


def test_convrot_is_an_int8_option_only():
    with pytest.raises(ValueError, match="int8"):
        pkg.prepare_projection_maps([{"to_out_linear.weight": torch.zeros(8, 256)}], "cpu", "fp8", convrot=True)


@pytest.mark.parametrize("convrot", [False, True])
def test_stored_int8_master_dequantises_to_the_weight(convrot):
    """A stored int8 to_out_linear master (plain or ConvRot codes, per-channel scales) turns back
    into the weight within int8 resolution; the ConvRot rotation is its own inverse."""
    gen = torch.Generator().manual_seed(9)
    w = torch.randn(48, 512, generator=gen) * 0.02
    q, s = vo.int8_quantize_rows_convrot(w) if convrot else vo.int8_quantize_weight(w)
    deq = pkg.projection.dequantize_projection_weight(q, s, 256 if convrot else None)
    assert deq.shape == w.shape and deq.dtype == torch.float32
    assert float((deq - w).norm() / w.norm()) < 1.5e-2
    h = pkg.projection.convrot_matrix(256)
    assert torch.allclose(h, h.T) and torch.allclose(h @ h, torch.eye(256, dtype=torch.float64))
    assert torch.allclose(h, torch.from_numpy(vo.convrot_rotate(torch.eye(256))).double(), atol=1e-7)


def test_stored_fp8_master_scales_per_tensor_or_per_channel():
    q = torch.ones(4, 16).to(torch.float8_e4m3fn)
    assert torch.equal(pkg.projection.dequantize_projection_weight(q, torch.tensor([[0.5]])), torch.full((4, 16), 0.5))
    per_ch = pkg.projection.dequantize_projection_weight(q, torch.tensor([[1.0, 2.0, 3.0, 4.0]]))
    assert torch.equal(per_ch[:, 0], torch.tensor([1.0, 2.0, 3.0, 4.0]))
    with pytest.raises(ValueError):
        pkg.projection.dequantize_projection_weight(q, torch.ones(3))



def test_mask_known_answers_with_hand_written_bounds():
    """The reference's mask cases (tests/test_window.py:378-389): video rows [4, 34), 3 frames of
    10 tokens, frames 0-1 see frames 0-2 and frame 2 sees frame 0 only.  The mask function takes
    such bounds; a layout does not (window.py:172-178): the plan builder rejects them with the
    reference's message."""
    S, vs, ve, F, tpf = 40, 4, 34, 3, 10
    bounds = [(0, 2), (0, 2), (0, 0)]
    none = vo.allowed_mask(S, vs, ve, F, tpf, bounds, "none").numpy()
    assert not none[30, 18]  # frame 1 is outside frame 2's window
    assert none[30, 8]  # frame 0 inside
    assert none[30, 36]  # a global key
    assert none[1, 18]  # a global query
    both = vo.allowed_mask(S, vs, ve, F, tpf, bounds, "both").numpy()
    assert both[30, 18]  # frame 2 is the last frame: an anchor row
    with pytest.raises(ValueError, match=r"bounds\[2\]=\(0, 0\) does not contain its query frame"):
        bw.build_window_plan(S, vs, ve, F, tpf, bounds, "none")
    # the same answers from a valid layout whose last frame sees frames 1-2 only
    ok = [(0, 2), (0, 2), (1, 2)]
    for anchors in ("none", "both"):
        want = vo.allowed_mask(S, vs, ve, F, tpf, ok, anchors).numpy()
        assert want[30, 18]
        assert want[30, 8] == (anchors == "both")  # frame 0 only through the anchor rows
        plan = bw.build_window_plan(S, vs, ve, F, tpf, ok, anchors)
        np.testing.assert_array_equal(_expand_plan(plan, S), want)


def test_alpha_parameters_keep_fp32_precision():
    """The reference keeps alpha.A_log and alpha.dt_bias in fp32 when the other branch weights go
    to bf16 (tests/test_optimized_runtime.py:97-105); the device weight map does too."""
    from vdn_b200.branch import BranchDeviceWeights

    c = vo.CONFIG0
    H, D, hidden = c["heads"], c["dim"], c["hidden"]
    w = vo.make_branch_weights(torch.Generator().manual_seed(0), hidden, H, D)
    w["alpha.A_log"] = torch.full((H,), 1.0 + 2.0 ** -20)  # not representable in bf16
    w["alpha.dt_bias"] = torch.full((H * D,), -3.0 + 2.0 ** -19)
    bdw = BranchDeviceWeights.from_dict(w, H, D, "cpu")
    assert bdw.a_log.dtype == torch.float32 and bdw.dt_bias.dtype == torch.float32
    assert torch.equal(bdw.a_log, w["alpha.A_log"]) and torch.equal(bdw.dt_bias, w["alpha.dt_bias"])
    assert bdw.beta_w.dtype == torch.bfloat16  # the projections themselves run in bf16


# ------------------------------------------------------------------ branch settings at the operator
def _fused_block_for(config, branch, maps=None, **state_kw):
    """The FusedBlock a B200State builds for block 0 (on the CPU: construction moves weights
    only, no kernel runs)."""
    from __graft_entry__ import _Attn

    bw_ = vo.make_block(0, 64, 2, 64)
    branches = [branch if branch is not None else bw_.branch]
    state = pkg.B200State("t", config, branches, 2, 64, weight_maps=maps, **state_kw)
    return state.fused_block(_Attn(bw_, 2, 64), 0, "cpu")


def test_node_config_without_branch_keys_resolves_like_the_reference():
    """A config without the keys builds what nodes.py:98-116 builds (short_conv=(),
    bridge alpha, vdn_solve) and no text state (hybrid.py:449-451 default False)."""
    fb = _fused_block_for({}, None)
    assert fb.short_conv == () and fb.enable_text_state is False
    assert fb.bridge == "alpha" and fb.delta_rule == "vdn_solve" and fb.tile_frames == 0
    assert fb.bw.conv == {}  # no conv weights loaded for an empty short_conv


def test_node_config_keys_set_the_branch_structure():
    cfg = vo.BranchConfig(delta_rule="sana_scaled", bridge="none").node_config()
    fb = _fused_block_for(cfg, None, tile_frames=5)
    assert fb.short_conv == ("k", "v") and fb.enable_text_state is True
    assert fb.bridge == "none" and fb.delta_rule == "sana_scaled" and fb.tile_frames == 5


def test_branch_object_settings_win_over_the_config():
    """The operator reads the branch object first (hybrid.py:449-451; the branch's own
    bridge / short_conv / delta_rule / tile_frames drive its readout, runtime.py:545-607)."""
    w = vo.make_block(0, 64, 2, 64).branch
    br = pkg.B200LinearBranch(w, 2, 64, delta_rule="sana_scaled", bridge="none", short_conv=("v",),
                              enable_text_state=False, tile_frames=3)
    cfg = vo.BranchConfig().node_config()  # says k,v conv, text state on, alpha, vdn_solve
    fb = _fused_block_for(cfg, br, tile_frames=7)
    assert fb.short_conv == ("v",) and fb.enable_text_state is False
    assert fb.bridge == "none" and fb.delta_rule == "sana_scaled" and fb.tile_frames == 3


def test_to_out_follows_the_stored_representation():
    """to_out_linear runs in the representation its map stores (projection.py:259-268): a
    bf16 master (an fp8 model's edge block, fp8.py:198) stays bf16 in a quantised block, so
    the block cannot fuse both projections into one K-concat GEMM; a bf16 block with a bf16
    master can."""
    w = vo.make_block(0, 64, 2, 64).branch
    assert "to_out_linear.weight" in w
    fb = _fused_block_for({}, None, maps=[w])
    assert fb.to_out_kind == "bf16" and fb.concat_out
    fb8 = _fused_block_for({}, None, maps=[w], projection_precision="bf16")
    assert fb8.w_to_b16 is None  # folded into the K-concat weight


@pytest.mark.parametrize("n_chunks", [1, 3, 4, 9])
def test_chunk_items_finish_every_row_before_its_chunk_ends(n_chunks):
    """The head-sharded block launches the attention chunk by chunk of rows and queues each
    chunk's exchange behind it: every item runs exactly once, and after the launches of
    chunks 0..c every row before chunk c's end has been computed by them."""
    lay = vo.config_layout(vo.CONFIG1)
    plan = bw.build_window_plan(lay.seq_len, lay.video_start, lay.video_end, lay.num_frames,
                                lay.tokens_per_frame, list(lay.bounds), lay.anchor_frames)
    S, heads = lay.seq_len, 3
    step = -(-S // n_chunks)
    ends = [min(S, (c + 1) * step) for c in range(n_chunks)]
    chunks = plan.chunk_items(heads, ends)
    flat = np.concatenate(chunks)
    assert sorted(flat.tolist()) == sorted(plan.items(heads).tolist())
    done = np.zeros(S, dtype=bool)
    for c, its in enumerate(chunks):
        for code in its.tolist():
            for r0, n in plan.q_halves(code & 0xFFFFF):
                done[r0:r0 + n] = True
        assert done[:ends[c]].all()


@pytest.mark.parametrize("n_chunks,launches", [(4, 1), (4, 2), (4, 3), (4, 4), (8, 3), (3, 5)])
def test_chunk_groups_cover_the_chunks_in_order(n_chunks, launches):
    """Chunks merged into fewer attention launches: the runs are consecutive, cover every
    chunk once, and each run's items are its chunks' items in chunk order."""
    lay = vo.config_layout(vo.CONFIG1)
    plan = bw.build_window_plan(lay.seq_len, lay.video_start, lay.video_end, lay.num_frames,
                                lay.tokens_per_frame, list(lay.bounds), lay.anchor_frames)
    S, heads = lay.seq_len, 2
    step = -(-S // n_chunks)
    ends = [min(S, (c + 1) * step) for c in range(n_chunks)]
    per = plan.chunk_items(heads, ends)
    groups = plan.chunk_groups(heads, ends, launches)
    assert len(groups) == min(launches, n_chunks)
    covered = [c for _, r in groups for c in r]
    assert covered == list(range(n_chunks))
    for items, r in groups:
        want = np.concatenate([per[c] for c in r]) if len(r) else np.zeros(0, np.int32)
        assert np.array_equal(items, want)
