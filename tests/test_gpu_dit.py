"""GPU parity of the DiT block around the hybrid attention (block_kernels.py:85-240):
the AdaLN RMSNorm row kernel, the fused GEMM epilogues (GELU, paired SwiGLU, gated
residual), the whole block against the float64 oracle (bf16 and INT8, SwiGLU and GELU),
the drop-in ``make_fast_block_forward`` and a two-rank head-sharded block emulated on one
GPU (exchange replayed by copies, the MLP token-parallel on each rank's rows)."""

from __future__ import annotations

import types

import numpy as np
import pytest
import torch

from __graft_entry__ import _Attn, load_package
from oracle import vdn_oracle as vo

pytestmark = pytest.mark.gpu

pkg = load_package()
from vdn_b200 import dit as bdit  # noqa: E402
from vdn_b200 import shard as sh  # noqa: E402
from vdn_b200.hybrid import GatedResidual, gemm_block  # noqa: E402

DEV = torch.device("cuda:0") if torch.cuda.is_available() else None
CFG = dict(vo.CONFIG0)
FFN = 512


def rel_l2(got, want):
    got = got.double().cpu()
    want = want.double().cpu()
    return float((got - want).norm() / want.norm())


def _b16(t):
    return t.to(DEV, torch.bfloat16).contiguous()


def _segments(lay):
    # text rows use modulation row 0, video rows row 1 (two groups, like H3's text / video)
    return [(0, lay.video_start, 0), (lay.video_start, lay.seq_len, 1)]


@pytest.mark.parametrize("H", [256, 5120, 12288, 40960])
def test_adaln_rmsnorm_matches_oracle_and_int8_codes_are_exact(H):
    """Every kernel width class: CTA-per-row with 2 or 4 vectors per thread of 256 / 1024
    threads, and the warp-per-row streaming kernel for the widest rows."""
    gen = torch.Generator().manual_seed(1)
    S = 777 if H <= 12288 else 97
    x = torch.randn(S, H, generator=gen).to(torch.bfloat16)
    w = 1 + 0.1 * torch.randn(H, generator=gen)
    scale = (torch.randn(3, H, generator=gen) * 0.1).to(torch.bfloat16)
    shift = (torch.randn(3, H, generator=gen) * 0.1).to(torch.bfloat16)
    group = torch.randint(0, 3, (S,), generator=gen, dtype=torch.int32)
    out = torch.empty(S, H, device=DEV, dtype=torch.bfloat16)
    q = torch.empty(S, H, device=DEV, dtype=torch.int8)
    qs = torch.empty(S, device=DEV, dtype=torch.float32)
    # device copies bound to names: they must outlive the launch
    xd, wd, sd, hd, gd = _b16(x), w.to(DEV), _b16(scale), _b16(shift), group.to(DEV)
    pkg._lib.call("vdn_adaln_rmsnorm", xd.data_ptr(), H, S, H, wd.data_ptr(), 1e-6, sd.data_ptr(), hd.data_ptr(), H,
                  gd.data_ptr(), out.data_ptr(), H, q.data_ptr(), H, qs.data_ptr(), pkg._lib.stream_handle(DEV))
    torch.cuda.synchronize()
    want = vo.dit_pre(x.double(), w.double(), 1e-6, scale.double(), shift.double(), group.long())
    assert rel_l2(out, want) < 4e-3
    # the int8 codes are the config-2 quantiser applied to the bf16 row the kernel wrote
    y = out.float().cpu().numpy()
    amax = np.abs(y).max(axis=1).astype(np.float32)
    s = np.maximum(amax / np.float32(127.0), np.float32(1e-12)).astype(np.float32)
    codes = np.clip(np.rint(y / s[:, None]), -127, 127).astype(np.int8)
    np.testing.assert_array_equal(qs.cpu().numpy(), s)
    np.testing.assert_array_equal(q.cpu().numpy(), codes)


@pytest.mark.parametrize("kind", ["bf16", "int8"])
def test_gemm_block_epilogues_match_torch(kind):
    gen = torch.Generator().manual_seed(2)
    M, K, F, N = 300, 512, 768, 640
    a = torch.randn(M, K, generator=gen)
    w1 = torch.randn(2 * F, K, generator=gen) * 0.05
    b1 = torch.randn(2 * F, generator=gen) * 0.1
    w2 = torch.randn(N, F, generator=gen) * 0.05
    res = torch.randn(M, N, generator=gen).to(torch.bfloat16)
    gate = (1 + 0.1 * torch.randn(2, N, generator=gen)).to(torch.bfloat16)
    group = torch.randint(0, 2, (M,), generator=gen, dtype=torch.int32)
    st = pkg.DeviceStatus(DEV)
    stream = pkg._lib.stream_handle(DEV)
    kc = 0 if kind == "bf16" else 2

    def prep(x, w):
        if kind == "bf16":
            return _b16(x), _b16(w), None, None, x.to(torch.bfloat16).double(), w.to(torch.bfloat16).double()
        qa, sa = vo.int8_quantize_rows(x)
        qw, sw = vo.int8_quantize_weight(w)
        deq_a = qa.double() * sa.double()[:, None]
        deq_w = qw.double() * sw.double()[:, None]
        return qa.to(DEV), qw.to(DEV), sa.to(DEV), sw.to(DEV), deq_a, deq_w

    # SwiGLU over interleaved fc1 rows, bias included
    A, W, rs, cs, da, dw = prep(a, bdit.interleave_swiglu_rows(w1))
    act = torch.empty(M, F, device=DEV, dtype=torch.bfloat16)
    gemm_block(kc, A, W, act, row_scale=rs, col_scale=cs, col_bias=bdit.interleave_swiglu_rows(b1).to(DEV),
               act=3, status=st, stream=stream, rows=M)
    z = da @ dw.T + bdit.interleave_swiglu_rows(b1).double()
    zg = z.view(M, F // 128, 2, 128)
    want = torch.nn.functional.silu(zg[:, :, 0]) * zg[:, :, 1]
    torch.cuda.synchronize()
    assert rel_l2(act, want.reshape(M, F)) < 1e-2
    # GELU
    A, W, rs, cs, da, dw = prep(a, w1[:F])
    g_out = torch.empty(M, F, device=DEV, dtype=torch.bfloat16)
    gemm_block(kc, A, W, g_out, row_scale=rs, col_scale=cs, col_bias=b1[:F].to(DEV), act=2, status=st,
               stream=stream, rows=M)
    want = torch.nn.functional.gelu(da @ dw.T + b1[:F].double())
    torch.cuda.synchronize()
    assert rel_l2(g_out, want) < 1e-2
    # gated residual: out = res + gate[group] * (act w2^T)
    A, W, rs, cs, da, dw = prep(act.float().cpu(), w2)
    out = torch.empty(M, N, device=DEV, dtype=torch.bfloat16)
    gemm_block(kc, A, W, out, row_scale=rs, col_scale=cs,
               residual=GatedResidual(_b16(res), _b16(gate), group.to(DEV)), status=st, stream=stream, rows=M)
    want = res.double() + gate.double()[group.long()] * (da @ dw.T)
    torch.cuda.synchronize()
    st.raise_if_failed()
    assert rel_l2(out, want) < 1e-2


@pytest.mark.parametrize("act", [0, 2, 3])
def test_row_amax_epilogue_gives_the_quantiser_its_exact_scales(act):
    """fc1 with row_amax + the streaming quantiser == the two-pass row quantiser, bit for bit."""
    gen = torch.Generator().manual_seed(5)
    M, K, F = 333, 512, 1024
    a = torch.randn(M, K, generator=gen)
    w = torch.randn(2 * F if act == 3 else F, K, generator=gen) * 0.05
    qa, sa = vo.int8_quantize_rows(a)
    qw, sw = vo.int8_quantize_weight(w)
    A, W, rs, cs = qa.to(DEV), qw.to(DEV), sa.to(DEV), sw.to(DEV)
    out = torch.empty(M, F, device=DEV, dtype=torch.bfloat16)
    amax = torch.zeros(M, device=DEV)
    st = pkg.DeviceStatus(DEV)
    stream = pkg._lib.stream_handle(DEV)
    gemm_block(2, A, W, out, row_scale=rs, col_scale=cs, act=act, row_amax=amax, status=st, stream=stream, rows=M)
    q = torch.empty(M, F, device=DEV, dtype=torch.int8)
    qs = torch.empty(M, device=DEV)
    pkg._lib.call("vdn_quant_int8_rows_amax", out.data_ptr(), out.stride(0), M, F, amax.data_ptr(), q.data_ptr(),
                  q.stride(0), qs.data_ptr(), stream)
    torch.cuda.synchronize()
    st.raise_if_failed()
    assert torch.equal(amax.cpu(), out.float().abs().amax(1).cpu())
    ref = pkg.quantize_rows_int8(out)
    assert torch.equal(q, ref.data) and torch.equal(qs, ref.scale)


def _dit(seed, activation):
    H, D, hidden = CFG["heads"], CFG["dim"], CFG["hidden"]
    return vo.make_dit(seed, hidden, H, D, FFN, activation=activation)


def _device_block(dw, precision, activation, shard=None):
    H, D = CFG["heads"], CFG["dim"]
    bw = dw.attn
    branch = bw.branch
    if precision != "bf16":
        # to_out_linear runs in its stored representation: store it quantised too
        branch = pkg.prepare_projection_maps([branch], DEV, precision, skip_end_blocks=0)[0][0]
    fb = pkg.FusedBlock(bw.qkv, bw.q_norm, bw.k_norm, bw.out, branch, H, D, DEV, precision=precision, shard=shard)
    return pkg.B200DiTBlock(fb, dw.norm1, dw.eps, dw.norm2, dw.eps, dw.fc1, dw.fc1_b, dw.fc2, dw.fc2_b, DEV,
                            activation=activation, precision=precision)


@pytest.mark.parametrize("precision", ["bf16", "int8"])
@pytest.mark.parametrize("activation", ["swiglu", "gelu"])
def test_dit_block_matches_oracle(precision, activation):
    H, D, hidden = CFG["heads"], CFG["dim"], CFG["hidden"]
    lay_o = vo.config_layout(CFG)
    lay = pkg.make_layout(CFG["text"], CFG["frames"], CFG["grid"])
    dw = _dit(7, activation)
    mods = vo.make_mods(7, 2, hidden)
    idx = vo.segment_rows(_segments(lay_o), lay_o.seq_len)
    x = vo.make_x(7, lay_o.seq_len, hidden).to(torch.bfloat16)
    blk = _device_block(dw, precision, activation)
    status = pkg.DeviceStatus(DEV)
    with pkg.cholesky_runtime_scope():
        got = blk.forward(x.to(DEV), [_b16(m) for m in mods], idx.to(DEV, torch.int32), lay, pkg.WindowPlanCache(),
                          status)
    torch.cuda.synchronize()
    status.raise_if_failed()
    want = vo.dit_block_forward(x.double(), dw, [m.to(torch.bfloat16).double() for m in mods], idx, lay_o, H, D,
                                vo.BranchConfig(), activation=activation, precision=precision)
    # the block output is x plus two gated branches: compare the branch increments too
    inc_want = want - x.double()
    inc_got = got.double().cpu() - x.double()
    assert rel_l2(got, want) < 2e-2
    assert rel_l2(inc_got, inc_want) < (3e-2 if precision == "bf16" else 6e-2)


class _Linear:
    def __init__(self, w, b):
        self.weight, self.bias = w, b


def _comfy_block(dw, mods):
    """Stand-in of a ComfyUI MiniMax-H3 DiTBlock carrying the weights the patch reads."""
    H, D = CFG["heads"], CFG["dim"]
    blk = types.SimpleNamespace()
    blk.attn = _Attn(dw.attn, H, D)
    blk.norm1 = types.SimpleNamespace(weight=dw.norm1, eps=dw.eps)
    blk.norm2 = types.SimpleNamespace(weight=dw.norm2, eps=dw.eps)
    blk.mlp = types.SimpleNamespace(fc1=_Linear(dw.fc1, dw.fc1_b), fc2=_Linear(dw.fc2, dw.fc2_b))
    blk.adaln_proj = lambda t_emb: tuple(m * t_emb for m in mods)  # a modulation that depends on t_emb
    blk.calls = []

    def original(x, t_emb, mod_segments, rope_freqs, transformer_options=None, attention=None):
        blk.calls.append(attention)
        return x

    blk.forward = original
    return blk


def test_fast_block_forward_is_a_drop_in():
    H, D, hidden = CFG["heads"], CFG["dim"], CFG["hidden"]
    lay_o = vo.config_layout(CFG)
    lay = pkg.make_layout(CFG["text"], CFG["frames"], CFG["grid"])
    dw = _dit(11, "swiglu")
    mods = [m.to(torch.bfloat16) for m in vo.make_mods(11, 2, hidden)]
    blk = _comfy_block(dw, [_b16(m) for m in mods])
    state = pkg.B200State("dit", vo.BranchConfig().node_config(), [dw.attn.branch], H, D)
    fwd = pkg.make_fast_block_forward(blk, state, 0)
    x = vo.make_x(11, lay_o.seq_len, hidden).to(torch.bfloat16)
    t_emb = torch.tensor(1.0, device=DEV, dtype=torch.bfloat16)
    segs = _segments(lay_o)
    freqs = vo.make_rope_freqs(lay_o.seq_len, D)  # RoPE on the attention's q / k (parity unpinned)
    with pkg.publish_layout(lay):
        got = pkg.run_forward_checked(state, fwd, x.to(DEV), t_emb, segs, freqs.to(DEV))
        # an attention override runs the block's own forward, as in the reference
        fwd(x.to(DEV), t_emb, segs, None, attention="native")
    assert blk.calls == ["native"]
    with pytest.raises(TypeError):
        with pkg.publish_layout(lay):
            fwd(x.to(DEV), t_emb, segs, object())
    idx = vo.segment_rows(segs, lay_o.seq_len)
    want = vo.dit_block_forward(x.double(), dw, [m.double() for m in mods], idx, lay_o, H, D, vo.BranchConfig(),
                                rope_freqs=freqs)
    assert rel_l2(got, want) < 2e-2


@pytest.mark.parametrize("precision", ["bf16", "int8"])
def test_dit_block_sharded_rows_emulated_on_one_gpu(precision, monkeypatch):
    """Two ranks' heads, the chunked all-to-all replayed by copies, each rank's output
    projection with the gated residual and its MLP on its own rows (the token-parallel path
    of the sharded block) must reproduce the unsharded block."""
    monkeypatch.setattr(pkg.hybrid, "EXCHANGE_MIN_ROWS", 1)
    H, D, hidden = CFG["heads"], CFG["dim"], CFG["hidden"]
    lay_o = vo.config_layout(CFG)
    lay = pkg.make_layout(CFG["text"], CFG["frames"], CFG["grid"])
    dw = _dit(13, "swiglu")
    mods = [_b16(m) for m in vo.make_mods(13, 2, hidden)]
    group = vo.segment_rows(_segments(lay_o), lay_o.seq_len).to(DEV, torch.int32)
    x = _b16(vo.make_x(13, lay_o.seq_len, hidden))
    status = pkg.DeviceStatus(DEV)
    stream = pkg._lib.stream_handle(DEV)
    with pkg.cholesky_runtime_scope():
        ref = _device_block(dw, precision, "swiglu").forward(x, mods, group, lay, pkg.WindowPlanCache(), status).clone()
        world = 2
        blocks = [_device_block(dw, precision, "swiglu", sh.HeadShard(r, world, H)) for r in range(world)]
        plans = pkg.WindowPlanCache()
        parts = []
        for b in blocks:
            h = b.workspace(lay_o.seq_len)["h"][:lay_o.seq_len]
            b._adaln(x, b.norm1, b.eps1, mods[1], mods[0], group, out=h, stream=stream)
            parts.append(b.attn.forward_heads(h, lay, plans, status))
        xr0 = parts[0][0]["xchg"]
        cs = xr0.cs
        out = torch.zeros(world * xr0.chunks * cs, hidden, device=DEV, dtype=torch.bfloat16)
        residual = GatedResidual(x, mods[2], group)
        for r, b in enumerate(blocks):
            ws, la = parts[r]
            xr = ws["xchg"]
            for c in range(xr.chunks):
                r0, rows = xr.rows_of(c)
                for src in range(world):
                    xr.recv[c][src].copy_(parts[src][0]["xchg"].send[r0:r0 + cs])
                b.attn.project_rows(ws, la, xr.recv[c], rows, out[r0:r0 + cs], status, stream,
                                    residual=residual.rows(r0, rows))
                b.mlp_rows(out[r0:r0 + rows], group[r0:r0 + rows], mods, status, stream)
    torch.cuda.synchronize()
    status.raise_if_failed()
    got = out[:lay_o.seq_len]
    if precision == "int8":
        assert torch.equal(got, ref), "int8 sharded DiT block differs from the unsharded one"
    else:
        assert rel_l2(got, ref) < 2e-3
