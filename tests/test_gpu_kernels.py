"""GPU parity of the individual sm_100a kernels against the float64 oracle / fp32 torch.

Tolerances: bf16 outputs within 2e-2 relative L2 (most checks are far tighter), int8
quantisation codes and int32 accumulators bit-exact."""

from __future__ import annotations

import os

import numpy as np
import pytest
import torch

from __graft_entry__ import load_package
from oracle import vdn_oracle as vo

pytestmark = pytest.mark.gpu

pkg = load_package()
DEV = torch.device("cuda:0") if torch.cuda.is_available() else None


def rel_l2(got, want):
    got = got.double().cpu()
    want = want.double().cpu()
    return float((got - want).norm() / want.norm().clamp_min(1e-30))


def _randn(*shape, seed=0, scale=1.0):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(*shape, generator=g) * scale


# --------------------------------------------------------------------------- GEMM
@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (257, 520, 192), (1000, 768, 1024), (3000, 1024, 5120),
                                   (200, 130, 96), (77, 40, 48)])
def test_gemm_bf16_matches_fp32(M, N, K):
    a = _randn(M, K, seed=1).to(torch.bfloat16)
    b = _randn(N, K, seed=2, scale=0.05).to(torch.bfloat16)
    got = pkg.gemm(a.to(DEV), b.to(DEV), out_dtype=torch.float32)
    want = a.float() @ b.float().T
    assert rel_l2(got, want) < 1e-5


def test_gemm_k_concat_equals_single_operand():
    M, K1, K2, N = 300, 256, 512, 256
    a1 = _randn(M, K1, seed=3).to(torch.bfloat16)
    a2 = _randn(M, K2, seed=4).to(torch.bfloat16)
    b = _randn(N, K1 + K2, seed=5, scale=0.05).to(torch.bfloat16)
    got = pkg.gemm(a1.to(DEV), b.to(DEV), a2=a2.to(DEV), k_split=K1, out_dtype=torch.float32)
    want = torch.cat([a1, a2], 1).float() @ b.float().T
    assert rel_l2(got, want) < 1e-5


def test_gemm_epilogue_scale_bias_sigmoid_addend():
    M, N, K = 200, 512, 128
    a = _randn(M, K, seed=6).to(torch.bfloat16)
    b = _randn(N, K, seed=7, scale=0.05).to(torch.bfloat16)
    rs = torch.rand(M) + 0.5
    cs = torch.rand(N) + 0.5
    bias = _randn(N, seed=8)
    add = _randn(M, N, seed=9).to(torch.bfloat16)
    got = pkg.gemm(a.to(DEV), b.to(DEV), alpha=0.7, row_scale=rs.to(DEV), col_scale=cs.to(DEV),
                   col_bias=bias.to(DEV), sigmoid=True, addend=add.to(DEV), out_dtype=torch.float32)
    want = torch.sigmoid((a.float() @ b.float().T) * 0.7 * rs[:, None] * cs[None] + bias) + add.float()
    assert rel_l2(got, want) < 1e-5


def test_int8_quantisation_and_accumulator_bit_exact():
    M, N, K = 333, 512, 1024
    x = _randn(M, K, seed=10).to(torch.bfloat16)
    w = _randn(N, K, seed=11, scale=0.02)
    qa = pkg.quantize_rows_int8(x.to(DEV))
    qw = pkg.quantize_rows_int8(w.to(DEV))
    oa, sa = vo.int8_quantize_rows(x.float())
    ow, sw = vo.int8_quantize_weight(w)
    assert torch.equal(qa.data.cpu(), oa) and torch.equal(qa.scale.cpu(), sa)
    assert torch.equal(qw.data.cpu(), ow) and torch.equal(qw.scale.cpu(), sw)
    acc = pkg.gemm(qa.data, qw.data, kind=2, out_dtype=torch.int32)
    assert torch.equal(acc.cpu(), vo.int8_accumulate(oa, ow))
    deq = pkg.gemm(qa.data, qw.data, kind=2, row_scale=qa.scale, col_scale=qw.scale, out_dtype=torch.float32)
    want = acc.cpu().double() * sa.double()[:, None] * sw.double()[None]
    assert rel_l2(deq, want) < 1e-6


@pytest.mark.parametrize("K", [8, 1000, 1004, 5120, 20480, 20488])
def test_int8_row_quantiser_is_bit_exact_at_every_width(K):
    """Both quantiser kernels (16-byte register-resident rows for bf16 with K % 8 == 0, the
    scalar one otherwise) give the oracle's codes and scales bit for bit."""
    x = (_randn(37, K, seed=K) * 3).to(torch.bfloat16)
    x[5] = 0  # an all-zero row: scale 1e-12, codes 0
    q = pkg.quantize_rows_int8(x.to(DEV))
    oa, sa = vo.int8_quantize_rows(x.float())
    assert torch.equal(q.scale.cpu(), sa)
    assert torch.equal(q.data.cpu(), oa)


def test_fp8_gemm_matches_oracle():
    M, N, K = 500, 768, 2048
    x = _randn(M, K, seed=12).to(torch.bfloat16)
    w = _randn(N, K, seed=13, scale=0.02)
    qa = pkg.quantize_tensor_fp8(x.to(DEV))
    qw = pkg.quantize_tensor_fp8(w.to(DEV))
    oa, sa = vo.fp8_quantize_tensor(x.float())
    ow, sw = vo.fp8_quantize_tensor(w)
    assert abs(float(qa.scale) - sa) <= 1e-7 * sa and abs(float(qw.scale) - sw) <= 1e-7 * sw
    assert torch.equal(qa.data.cpu().view(torch.uint8), oa.view(torch.uint8))
    got = pkg.gemm(qa.data, qw.data, kind=1, dev_scale0=qa.scale, dev_scale1=qw.scale, out_dtype=torch.float32)
    want = vo.project(x.float(), w, "fp8")
    assert rel_l2(got, want) < 1e-5
    # and the fp8 product stays within 2e-2 of the exact product
    assert rel_l2(got, x.double() @ w.double().T) < 5e-2


def test_qkv_gemm_epilogue():
    S, hidden, H, D = 300, 256, 2, 128
    inner = H * D
    n_aux = 256
    x = _randn(S, hidden, seed=14).to(torch.bfloat16)
    w = _randn(3 * inner + n_aux, hidden, seed=15, scale=0.05).to(torch.bfloat16)
    nw = (1 + 0.1 * _randn(2 * D, seed=16)).float()
    qkv = torch.empty(S, 3 * inner, device=DEV, dtype=torch.bfloat16)
    qkn = torch.empty(S, 2 * inner, device=DEV, dtype=torch.bfloat16)
    aux = torch.empty(S, n_aux, device=DEV, dtype=torch.float32)
    # branch q features of rows [r0, r0 + Fq * tq), frame-head-token-dim
    r0, Fq, tq = 17, 5, 40
    qf = torch.empty(Fq, H, tq, D, device=DEV, dtype=torch.bfloat16)
    st = pkg._lib.DeviceStatus(DEV)
    xd, wd, nwd = x.to(DEV), w.to(DEV), nw.to(DEV)
    pkg._lib.call("vdn_qkv_gemm", 0, xd.data_ptr(), hidden, wd.data_ptr(), hidden, S, hidden, inner, n_aux, D,
                  nwd.data_ptr(), 1e-6, 1.0, None, None, None, None, qkv.data_ptr(), 3 * inner,
                  qkn.data_ptr(), 2 * inner, aux.data_ptr(), n_aux, qf.data_ptr(), r0, Fq * tq, tq, st.err_ptr,
                  pkg._lib.stream_handle(DEV))
    torch.cuda.synchronize()
    st.raise_if_failed()
    full = x.float() @ w.float().T
    assert rel_l2(qkv, full[:, :3 * inner]) < 5e-3
    assert rel_l2(aux, full[:, 3 * inner:]) < 1e-5
    raw = full[:, :2 * inner].to(torch.bfloat16).float().reshape(S, 2, H, D)
    normed = raw * torch.rsqrt(raw.square().mean(-1, keepdim=True) + 1e-6) * nw.reshape(2, 1, D)
    assert rel_l2(qkn, normed.reshape(S, 2 * inner)) < 5e-3
    qraw = full[r0:r0 + Fq * tq, :inner].to(torch.bfloat16).double().reshape(Fq * tq, H, D)
    want_qf = vo.to_fhsd(vo.activate(qraw, True), Fq)
    assert rel_l2(qf, want_qf) < 5e-3


# --------------------------------------------------------------------------- window attention
def _attention_case(lay, heads, dim, seed, gate=True):
    ki = vo.make_kernel_inputs(seed, lay, heads, dim)
    q, k, v = (ki[n].to(torch.bfloat16) for n in ("q", "k", "v"))
    logits = _randn(lay.seq_len, heads, seed=seed + 1)
    bias = _randn(heads, seed=seed + 2) * 0.5
    return q, k, v, logits, bias


@pytest.mark.parametrize("mode", vo.ANCHOR_MODES)
def test_window_attention_config0(mode):
    lay = vo.config_layout(vo.CONFIG0)
    H, D = 4, 64
    q, k, v, logits, bias = _attention_case(lay, H, D, 20)
    got = pkg.window_softmax_b200(q.to(DEV), k.to(DEV), v.to(DEV), lay.video_start, lay.video_end, lay.num_frames,
                                  lay.tokens_per_frame, list(lay.bounds), D ** -0.5, mode,
                                  gate=(logits.to(DEV), bias.to(DEV)))
    want = vo.window_attention(q.float(), k.float(), v.float(), lay.video_start, lay.video_end, lay.num_frames,
                               lay.tokens_per_frame, list(lay.bounds), D ** -0.5, mode)
    want = want * torch.sigmoid(logits.double() + bias.double())[:, :, None]
    assert rel_l2(got, want) < 1e-2


def test_window_attention_golden_vector():
    g = dict(np.load(os.path.join(os.path.dirname(__file__), "golden", "config0.npz")))
    lay = vo.config_layout(vo.CONFIG0)
    ki = vo.make_kernel_inputs(0, lay, 4, 64)
    got = pkg.window_softmax_b200(*(ki[n].to(DEV, torch.bfloat16) for n in ("q", "k", "v")), lay.video_start,
                                  lay.video_end, lay.num_frames, lay.tokens_per_frame, list(lay.bounds), 64 ** -0.5,
                                  "both")
    assert rel_l2(got, torch.from_numpy(g["window_both"])) < 1e-2


@pytest.mark.parametrize("geom", [(24, 9, (4, 4), 8, 2, 0, "columns", 2, 64),
                                  (512, 7, (38, 22), 0, 1, 5, "both", 2, 128),
                                  (100, 5, (20, 13), 37, 1, 2, "rows", 3, 128)])
@pytest.mark.parametrize("cutting", ["class", "dense"])
def test_window_attention_ragged_tiles(geom, cutting):
    before, F, grid, after, radius, chunk, mode, H, D = geom
    tpf = grid[0] * grid[1]
    vs, ve = before, before + F * tpf
    S = ve + after
    lay = vo.Layout(seq_len=S, video_start=vs, video_end=ve, num_frames=F, tokens_per_frame=tpf, frame_size=grid,
                    text_start=0, text_len=before, bounds=tuple(vo.window_bounds(F, radius, chunk)),
                    anchor_frames=mode)
    q, k, v, logits, bias = _attention_case(lay, H, D, 30)
    plan = pkg.window.build_window_plan(S, vs, ve, F, tpf, list(lay.bounds), mode, cutting=cutting)
    got = torch.empty(S, H, D, device=DEV, dtype=torch.bfloat16)
    st = pkg.DeviceStatus(DEV)
    pkg.window.launch_window_attention(q.to(DEV), k.to(DEV), v.to(DEV), got, plan, H, D, D ** -0.5, st)
    torch.cuda.synchronize()
    st.raise_if_failed()
    rows = torch.unique(torch.cat([torch.arange(0, S, 37), torch.arange(max(0, vs - 3), min(S, vs + 130)),
                                   torch.tensor([S - 1])]))
    want = vo.window_attention(q.float(), k.float(), v.float(), vs, ve, F, tpf, list(lay.bounds), D ** -0.5, mode,
                               rows=rows)
    assert rel_l2(got[rows], want) < 1e-2


@pytest.mark.parametrize("D", [64, 128])
def test_window_attention_moving_reference_is_exact(D):
    """Scores far from the N(0, 1) range exercise every branch of the online softmax: rows
    whose reference maximum moves by more than 2^8 within and across key tiles (large q), rows
    whose first tile lies entirely below 2^-32 of the speculative reference (q opposite to
    every key), and ordinary rows."""
    lay = vo.make_layout(40, 9, (6, 8), anchor_frames="both")
    S, H = lay.seq_len, 2
    g = torch.Generator().manual_seed(50)
    u = torch.nn.functional.normalize(torch.randn(H, D, generator=g), dim=-1)
    k = torch.nn.functional.normalize(u + 0.3 * torch.randn(S, H, D, generator=g), dim=-1)
    q = torch.randn(S, H, D, generator=g)
    q[0::3] *= 30
    q[1::3] = -300.0 * u
    v = torch.randn(S, H, D, generator=g)
    q, k, v = (t.to(torch.bfloat16) for t in (q, k, v))
    got = pkg.window_softmax_b200(q.to(DEV), k.to(DEV), v.to(DEV), lay.video_start, lay.video_end, lay.num_frames,
                                  lay.tokens_per_frame, list(lay.bounds), D ** -0.5, "both")
    want = vo.window_attention(q.double(), k.double(), v.double(), lay.video_start, lay.video_end, lay.num_frames,
                               lay.tokens_per_frame, list(lay.bounds), D ** -0.5, "both")
    assert torch.isfinite(got.float()).all()
    for name, rows in (("moving", slice(0, S, 3)), ("below", slice(1, S, 3)), ("plain", slice(2, S, 3))):
        assert rel_l2(got[rows], want[rows]) < 1e-2, name


# --------------------------------------------------------------------------- branch kernels
def _branch_setup(seed=40, Fb=6, grid=(4, 5), H=2, D=64, text=9):
    tpf = grid[0] * grid[1]
    rows = Fb * tpf
    g = torch.Generator().manual_seed(seed)
    w = vo.make_branch_weights(g, 96, H, D)
    q = torch.randn(rows, H * D, generator=g).to(torch.bfloat16)
    k = torch.randn(rows, H * D, generator=g).to(torch.bfloat16)
    v = torch.randn(rows, H * D, generator=g).to(torch.bfloat16)
    return w, q, k, v, tpf, rows


def test_conv_features_match_oracle():
    w, q, k, v, tpf, rows = _branch_setup()
    Fb, H, D, grid = 6, 2, 64, (4, 5)
    bwt = pkg.branch.BranchDeviceWeights.from_dict(w, H, D, DEV)
    ws = pkg.branch.BranchWorkspace(DEV, Fb, tpf, H, D, 0)
    kd = k.to(DEV)
    sp, kh, kw, tm, taps = bwt.conv["k"]
    s = pkg._lib.stream_handle(DEV)
    pkg._lib.call("vdn_spatial_conv", kd.data_ptr(), kd.stride(0), sp.data_ptr(), kh, kw, Fb, grid[0], grid[1],
                  H * D, ws.conv_buffer().data_ptr(), ws.conv_buffer().stride(0), s)
    pkg._lib.call("vdn_temporal_act", ws.conv_buffer().data_ptr(), ws.conv_buffer().stride(0), tm.data_ptr(), taps, Fb, tpf, H,
                  D, 1, ws.kf.data_ptr(), s)
    qd = q.to(DEV)
    pkg._lib.call("vdn_temporal_act", qd.data_ptr(), qd.stride(0), None, 0, Fb, tpf, H, D, 1, ws.qf.data_ptr(), s)
    torch.cuda.synchronize()
    want_k = vo.conv_features(k.float().reshape(rows, H, D), w["short_conv.k_sp.weight"], w["short_conv.k_tm.weight"],
                              Fb, grid, True)
    want_q = vo.to_fhsd(vo.activate(q.float().reshape(rows, H, D), True), Fb)
    assert rel_l2(ws.kf, want_k) < 1e-2
    assert rel_l2(ws.qf, want_q) < 5e-3


@pytest.mark.parametrize("F,gh,gw,C,pitch_mult", [
    (3, 22, 38, 192, 3),   # config-1 frame grid, three 64-channel slabs, strided rows (double-buffered tiles)
    (2, 9, 97, 128, 1),    # wide rows: one shared-memory buffer
    (2, 7, 11, 96, 2),     # C not a multiple of 64: the untiled paired kernel
    (1, 3, 4, 64, 1),      # frame smaller than the 5x5 window
])
def test_spatial_conv_matches_torch_conv2d(F, gh, gw, C, pitch_mult):
    g = torch.Generator().manual_seed(F * 1000 + gw)
    rows = F * gh * gw
    base = torch.randn(rows, C * pitch_mult, generator=g).to(torch.bfloat16)
    x = base[:, :C]
    w = torch.randn(C, 1, 5, 5, generator=g) * 0.2
    xd, wd = base.to(DEV), w.reshape(C, 25).contiguous().to(DEV)
    out = torch.empty(rows, C, device=DEV, dtype=torch.bfloat16)
    pkg._lib.call("vdn_spatial_conv", xd.data_ptr(), xd.stride(0), wd.data_ptr(), 5, 5, F, gh, gw, C, out.data_ptr(),
                  out.stride(0), pkg._lib.stream_handle(DEV))
    torch.cuda.synchronize()
    img = x.double().reshape(F, gh, gw, C).permute(0, 3, 1, 2)
    want = torch.nn.functional.conv2d(img, w.double(), padding=2, groups=C).permute(0, 2, 3, 1).reshape(rows, C)
    # one bf16 rounding of the output: ~2^-9 relative per element
    assert rel_l2(out, want) < 3e-3
    assert float((out.double().cpu() - want).abs().max()) < 2e-2 * float(want.abs().max())


def test_statistics_factor_scan_match_oracle_and_report_non_spd():
    Fb, H, T, D = 5, 3, 70, 128
    g = torch.Generator().manual_seed(50)
    kf = torch.nn.functional.normalize(torch.randn(Fb, H, T, D, generator=g), dim=-1).to(torch.bfloat16)
    vf = torch.randn(Fb, H, T, D, generator=g).to(torch.bfloat16)
    logits = torch.randn(Fb * T, 8, generator=g)
    alpha = torch.sigmoid(torch.randn(Fb, H, D, generator=g) + 2)
    A = torch.empty(Fb, H, D, D, device=DEV)
    B = torch.empty_like(A)
    s = pkg._lib.stream_handle(DEV)
    ld, kd, vd = logits.to(DEV), kf.to(DEV), vf.to(DEV)  # device copies must outlive the async launch
    pkg._lib.call("vdn_frame_stats", kd.data_ptr(), vd.data_ptr(), Fb, H, T, D, ld.data_ptr(), 8, 2,
                  A.data_ptr(), B.data_ptr(), s)
    beta = torch.sigmoid(logits[:, 2:2 + H]).reshape(Fb, T, H).permute(0, 2, 1)
    wa, wb = vo.frame_statistics(kf.float(), vf.float(), beta)
    torch.cuda.synchronize()
    assert rel_l2(A, wa) < 1e-5 and rel_l2(B, wb) < 1e-5
    # the tensor-core statistics (bf16 products of beta-weighted features) agree too
    A_tc, B_tc = torch.empty_like(A), torch.empty_like(A)
    st = pkg._lib.DeviceStatus(DEV)
    pkg._lib.call("vdn_frame_stats_tc", kd.data_ptr(), vd.data_ptr(), Fb, H, T, ld.data_ptr(), 8, 2,
                  A_tc.data_ptr(), B_tc.data_ptr(), st.err_ptr, s)
    torch.cuda.synchronize()
    st.raise_if_failed()
    assert rel_l2(A_tc, wa) < 5e-3 and rel_l2(B_tc, wb) < 5e-3
    inv = torch.empty_like(A)
    info = torch.zeros(Fb, H, device=DEV, dtype=torch.int32)
    split = torch.empty(2, Fb, H, D, D, device=DEV, dtype=torch.bfloat16)
    pkg._lib.call("vdn_delta_factor", A.data_ptr(), B.data_ptr(), Fb, H, D, inv.data_ptr(), info.data_ptr(), -1, 0.0,
                  None, split.data_ptr(), s)
    eye = torch.eye(D, dtype=torch.float64)
    want_inv = torch.linalg.inv(eye + wa)
    torch.cuda.synchronize()
    assert int(info.abs().sum()) == 0
    assert rel_l2(inv, want_inv) < 1e-5
    prefix = torch.empty_like(A)
    suffix = torch.empty_like(A)
    s0 = (torch.randn(H, D, D, generator=g) * 0.1)
    ad, s0d = alpha.to(DEV), s0.to(DEV)
    pkg._lib.call("vdn_bidir_scan", inv.data_ptr(), B.data_ptr(), ad.data_ptr(), s0d.data_ptr(), Fb, H, D, 0.0,
                  prefix.data_ptr(), suffix.data_ptr(), s)
    trans, inj = vo.factor_apply(alpha, wa, wb)
    wp, wsf = vo.run_scans(trans, inj, s0.double())
    torch.cuda.synchronize()
    assert rel_l2(prefix, wp) < 1e-4 and rel_l2(suffix, wsf) < 1e-4
    # hi + lo halves reproduce the inverse to ~2^-16, and the tensor-core scan matches
    assert rel_l2(split[0].float() + split[1].float(), want_inv) < 2e-5
    p_tc, s_tc = torch.empty_like(A), torch.empty_like(A)
    pkg._lib.call("vdn_bidir_scan_tc", split.data_ptr(), B.data_ptr(), ad.data_ptr(), s0d.data_ptr(), Fb, Fb, H, 0.0,
                  p_tc.data_ptr(), s_tc.data_ptr(), st.err_ptr, s)
    torch.cuda.synchronize()
    st.raise_if_failed()
    assert rel_l2(p_tc, wp) < 1e-4 and rel_l2(s_tc, wsf) < 1e-4
    # a matrix that is not SPD reports the order of its first bad leading minor
    bad = wa.clone().float()
    bad[2, 1] = -3.0 * torch.eye(D)
    bd = bad.to(DEV)
    pkg._lib.call("vdn_delta_factor", bd.data_ptr(), B.data_ptr(), Fb, H, D, inv.data_ptr(), info.data_ptr(), -1, 0.0,
                  None, None, s)
    torch.cuda.synchronize()
    want_info = vo.cholesky_info(bad.double())
    assert torch.equal(info.cpu(), want_info)
    assert int(info[2, 1]) == 1


@pytest.mark.parametrize("D,rot,shared", [(128, 128, False), (128, 64, True), (64, 48, False), (64, 12, False)])
def test_rope_split_half_matches_oracle(D, rot, shared):
    """In-place RoPE on q and k heads (16-byte path for rot % 16 == 0, with a lane's matrices
    fixed per row when rot/16 divides 32; scalar path otherwise; one table per row or one for
    all rows): within one bf16 rounding of the float64 oracle."""
    S, H = 300, 3
    g = torch.Generator().manual_seed(52)
    qk = torch.randn(S, 2 * H * D + 16, generator=g).to(torch.bfloat16)  # padded pitch
    freqs = vo.make_rope_freqs(1 if shared else S, rot, offset=7)
    dev_qk = qk.to(DEV)
    fd = freqs.to(DEV).reshape(freqs.shape[0], -1).contiguous()
    pkg._lib.call("vdn_rope_split_half", dev_qk.data_ptr(), dev_qk.stride(0), S, 2 * H, D, rot, fd.data_ptr(),
                  0 if shared else fd.stride(0), pkg._lib.stream_handle(DEV))
    heads = qk[:, :2 * H * D].double().reshape(S, 2 * H, D)
    want = vo.rope_split_half(heads, freqs.expand(S, -1, -1, -1) if shared else freqs)
    torch.cuda.synchronize()
    got = dev_qk.cpu()
    assert torch.equal(got[:, 2 * H * D:], qk[:, 2 * H * D:])  # the pitch padding is untouched
    got = got[:, :2 * H * D].double().reshape(S, 2 * H, D)
    assert torch.equal(got[..., rot:], heads[..., rot:])  # features past rot_dim pass through
    err = (got - want).abs()
    assert float((err - 2 ** -8 * want.abs()).max()) <= 1e-6  # one bf16 rounding (half an ulp, with slack)


@pytest.mark.parametrize("D", [64, 128])
def test_sana_factor_and_scans_match_oracle(D):
    """delta_rule="sana_scaled" (branch.py:163-177): M = I - A/L, s_t = s_{t-1} diag(alpha) M + B/sqrt(L),
    through the SIMT scan and, at head_dim 128, the tensor-core scan; text state 0.5 B/sqrt(L_text)."""
    Fb, H, T, L_text = 6, 3, 70, 11
    g = torch.Generator().manual_seed(51)
    kf = torch.nn.functional.normalize(torch.randn(Fb + 1, H, T, D, generator=g), dim=-1)
    vf = torch.randn(Fb + 1, H, T, D, generator=g)
    beta = torch.sigmoid(torch.randn(Fb + 1, H, T, generator=g))
    alpha = torch.sigmoid(torch.randn(Fb, H, D, generator=g) + 2)
    wa, wb = vo.frame_statistics(kf, vf, beta)  # the last frame stands in for the text frame
    A, B = wa.float().to(DEV).contiguous(), wb.float().to(DEV).contiguous()
    s = pkg._lib.stream_handle(DEV)
    M = torch.empty_like(A)
    split = torch.empty(2, Fb + 1, H, D, D, device=DEV, dtype=torch.bfloat16) if D == 128 else None
    s0 = torch.empty(H, D, D, device=DEV)
    pkg._lib.call("vdn_sana_factor", A.data_ptr(), B.data_ptr(), Fb + 1, H, D, 1.0 / T, M.data_ptr(),
                  None if split is None else split.data_ptr(), Fb, (1.0 / L_text) ** 0.5, 0.5, s0.data_ptr(), s)
    trans, inj = vo.sana_factor_apply(alpha, wa[:Fb], wb[:Fb], T)
    _, t_inj = vo.sana_factor_apply(torch.ones(1, H, D), wa[Fb:], wb[Fb:], L_text)
    want_s0 = 0.5 * t_inj[0]
    eye = torch.eye(D, dtype=torch.float64)
    torch.cuda.synchronize()
    assert rel_l2(M[:Fb], eye - wa[:Fb] / T) < 1e-6
    assert rel_l2(s0, want_s0) < 1e-6
    wp, wsf = vo.run_scans(trans, inj, want_s0)
    ad = alpha.to(DEV)
    prefix, suffix = torch.empty(Fb, H, D, D, device=DEV), torch.empty(Fb, H, D, D, device=DEV)
    pkg._lib.call("vdn_bidir_scan", M.data_ptr(), B.data_ptr(), ad.data_ptr(), s0.data_ptr(), Fb, H, D,
                  (1.0 / T) ** 0.5, prefix.data_ptr(), suffix.data_ptr(), s)
    torch.cuda.synchronize()
    assert rel_l2(prefix, wp) < 1e-5 and rel_l2(suffix, wsf) < 1e-5
    # the vdn_solve folding gives a different answer on the same buffers
    assert rel_l2(prefix, vo.run_scans(*vo.factor_apply(alpha, wa[:Fb], wb[:Fb]), want_s0)[0]) > 1e-2
    if D == 128:
        # the split holds M^T: element [n][k] = M[k][n], hi + lo to ~2^-16
        mt = (eye - wa / T).transpose(-1, -2)
        assert rel_l2(split[0].float() + split[1].float(), mt) < 2e-5
        st = pkg._lib.DeviceStatus(DEV)
        p_tc, s_tc = torch.empty_like(prefix), torch.empty_like(prefix)
        pkg._lib.call("vdn_bidir_scan_tc", split.data_ptr(), B.data_ptr(), ad.data_ptr(), s0.data_ptr(), Fb, Fb + 1,
                      H, (1.0 / T) ** 0.5, p_tc.data_ptr(), s_tc.data_ptr(), st.err_ptr, s)
        torch.cuda.synchronize()
        st.raise_if_failed()
        assert rel_l2(p_tc, wp) < 1e-4 and rel_l2(s_tc, wsf) < 1e-4


@pytest.mark.parametrize("D,grid,tile", [(64, (4, 5), 1), (64, (4, 5), 4), (128, (10, 15), 3), (128, (10, 15), 2)])
def test_frame_tiled_branch_equals_untiled(D, grid, tile):
    """The low-memory frame-tiled spelling (runtime.py:421-543; the reference's own test holds
    it to 3e-5 of the untiled branch, tests/test_domestic_runtime.py:42-109) gives the same
    bits here: every kernel computes a frame from the same inputs in the same order."""
    H, hidden, F = 2, 96, 9
    tpf = grid[0] * grid[1]
    rows = F * tpf
    g = torch.Generator().manual_seed(61)
    w = vo.make_branch_weights(g, hidden, H, D)
    w["to_out_linear.weight"] = torch.randn(hidden, H * D, generator=g) * 0.02
    xv = torch.randn(rows, hidden, generator=g).to(torch.bfloat16).to(DEV)
    q, k, v = (torch.randn(rows, H, D, generator=g).to(torch.bfloat16).to(DEV) for _ in range(3))
    tx = torch.randn(11, hidden, generator=g).to(torch.bfloat16).to(DEV)
    tk, tv = (torch.randn(11, H, D, generator=g).to(torch.bfloat16).to(DEV) for _ in range(2))
    bounds = vo.window_bounds(F, 1, 2)
    for rule in ("vdn_solve", "sana_scaled"):
        br = pkg.B200LinearBranch(w, H, D, delta_rule=rule)
        args = (w, xv, q, k, v, F, tpf, bounds)
        kw = dict(frame_size=grid, text_x=tx, text_k_raw=tk, text_v_raw=tv, skip_ends=True)
        whole = br.readout(*args, **kw).clone()
        tiled = br.readout(*args, **kw, tile_frames=tile)
        torch.cuda.synchronize()
        assert torch.equal(tiled, whole), f"{rule}: tiled readout differs"
        assert br.workspace(DEV, F - 2, tpf, 11, tile).feature_frames == min(F - 2, tile + 4)
        # projected_delta tiles only in inference, as runtime.py:584-590 does
        p_tiled = br.projected_delta(*args, **kw, inference=True, tile_frames=tile)
        p_whole = br.projected_delta(*args, **kw, inference=False, tile_frames=tile)
        torch.cuda.synchronize()
        assert torch.equal(p_tiled, p_whole)


@pytest.mark.parametrize("delta_rule", ["vdn_solve", "sana_scaled"])
@pytest.mark.parametrize("D,grid", [(64, (4, 5)), (128, (10, 15))])
def test_branch_readout_matches_oracle_with_and_without_text(D, grid, delta_rule):
    H, hidden = 2, 96
    F = 8
    tpf = grid[0] * grid[1]
    rows = F * tpf
    g = torch.Generator().manual_seed(60)
    w = vo.make_branch_weights(g, hidden, H, D)
    xv = torch.randn(rows, hidden, generator=g).to(torch.bfloat16)
    q, k, v = (torch.randn(rows, H, D, generator=g).to(torch.bfloat16) for _ in range(3))
    tx = torch.randn(11, hidden, generator=g).to(torch.bfloat16)
    tk, tv = (torch.randn(11, H, D, generator=g).to(torch.bfloat16) for _ in range(2))
    bounds = vo.window_bounds(F, 1, 2)
    br = pkg.B200LinearBranch(w, H, D, delta_rule=delta_rule)
    for text in (True, False):
        got = br.readout(w, xv.to(DEV), q.to(DEV), k.to(DEV), v.to(DEV), F, tpf, bounds, frame_size=grid,
                         text_x=tx.to(DEV) if text else None, text_k_raw=tk.to(DEV), text_v_raw=tv.to(DEV),
                         skip_ends=True)
        want, parts = vo.branch_readout(w, xv.float(), q.float(), k.float(), v.float(), F, tpf, bounds, grid, H, D,
                                        vo.BranchConfig(delta_rule=delta_rule), text_x=tx.float() if text else None,
                                        text_k=tk.float(),
                                        text_v=tv.float(), skip_ends=True, return_parts=True)
        ws = br.workspace(DEV, F - 2, tpf, 11 if text else 0)
        stages = {name: rel_l2(getattr(ws, attr), parts[name]) for name, attr in
                  (("q", "qf"), ("k", "kf"), ("v", "vf"), ("alpha", "alpha"), ("prefix", "prefix"),
                   ("suffix", "suffix"))}
        stages["A"] = rel_l2(ws.A[:F - 2], parts["A"])
        stages["B"] = rel_l2(ws.B[:F - 2], parts["B"])
        if text:
            stages["text_state"] = rel_l2(ws.s0, parts["text_state"])
        msg = "; ".join(f"{k}={v:.3e}" for k, v in stages.items())
        assert rel_l2(got, want) < 2e-2, f"text={text} out={rel_l2(got, want):.3e} stages: {msg}"
        assert float(got[:tpf].abs().max()) == 0.0 and float(got[-tpf:].abs().max()) == 0.0


@pytest.mark.parametrize("F,grid,H,D,l2,pitch_mult", [
    (29, (38, 22), 2, 128, True, 3),   # config-1 frame grid (one column block), k features
    (7, (38, 22), 2, 128, False, 1),   # v features (no L2)
    (5, (9, 48), 1, 128, True, 1),     # config-3 width: three column blocks
    (3, (5, 7), 4, 64, True, 2),       # head_dim 64, bands and blocks smaller than a unit
    (1, (3, 4), 2, 128, True, 1),      # a single frame: both temporal neighbours are padding
])
def test_fused_conv_features_equal_the_two_kernel_path(F, grid, H, D, l2, pitch_mult):
    """vdn_conv_features (spatial 5x5 + temporal 5-tap + SiLU + L2 in one pass) against
    vdn_spatial_conv followed by vdn_temporal_act on the same rows: the same arithmetic, but
    the two kernels add a spatial output's 25 products in different orders, so a spatial
    output now and then rounds to the neighbouring bf16 value, and the features it feeds
    differ by about that much."""
    g = torch.Generator().manual_seed(F * 100 + D)
    gh, gw = grid
    tpf = gh * gw
    rows, C = F * tpf, H * D
    base = (torch.randn(rows, C * pitch_mult, generator=g) * 2).to(torch.bfloat16).to(DEV)
    x = base[:, :C]
    w_sp = (torch.randn(C, 25, generator=g) * 0.2).to(DEV)
    w_tm = (torch.randn(C, 5, generator=g) * 0.45).to(DEV)
    s = pkg._lib.stream_handle(DEV)
    tmp = torch.empty(rows, C, device=DEV, dtype=torch.bfloat16)
    two = torch.empty(F, H, tpf, D, device=DEV, dtype=torch.bfloat16)
    one = torch.full((F, H, tpf, D), 7.0, device=DEV, dtype=torch.bfloat16)
    pkg._lib.call("vdn_spatial_conv", x.data_ptr(), x.stride(0), w_sp.data_ptr(), 5, 5, F, gh, gw, C, tmp.data_ptr(),
                  C, s)
    pkg._lib.call("vdn_temporal_act", tmp.data_ptr(), C, w_tm.data_ptr(), 5, F, tpf, H, D, int(l2), two.data_ptr(), s)
    pkg._lib.call("vdn_conv_features", x.data_ptr(), x.stride(0), w_sp.data_ptr(), 5, 5, w_tm.data_ptr(), 5, F, gh, gw,
                  H, D, int(l2), one.data_ptr(), s)
    torch.cuda.synchronize()
    assert torch.isfinite(one.float()).all()
    diff = (one.float() - two.float()).abs()
    # nearly all elements equal; the rest differ by the rounding of a spatial output
    assert rel_l2(one, two.float()) < 1e-3
    assert float(diff.max()) <= 2 ** -6 * float(two.float().abs().max())
    assert float((diff > 0).float().mean()) < 1e-2
    want = vo.conv_features(x.float().cpu().reshape(rows, H, D), w_sp.cpu().reshape(C, 1, 5, 5),
                            w_tm.cpu().reshape(C, 1, 5), F, grid, l2)
    assert rel_l2(one, want) < 1e-2
