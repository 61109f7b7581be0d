"""GPU parity of the ConvRot int8 projection (projection.py:74-97, :243-256) against the oracle.

ConvRot's rotation lives in comfy-kitchen, outside the reference tree, so parity with the
reference is unpinned; these tests pin the CUDA quantiser to the oracle's fp32 restatement
(``vdn_oracle.convrot_rotate``): codes and scales bit-exact, the int32 accumulator
bit-exact, the bf16 projection within 5e-3 relative L2 (one bf16 rounding of the output)."""

from __future__ import annotations

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


# K covers every kernel instance: 1/2/3/4 groups per warp at 8 warps, 2 and 4 at 32 warps
@pytest.mark.parametrize("K", [256, 2048, 3328, 5120, 8192, 12288, 20480])
def test_convrot_quantiser_is_bit_exact(K):
    x = _randn(37, K, seed=K).to(torch.bfloat16)
    x[:, 7] *= 40  # an outlier channel
    x[5] = 0  # an all-zero row: scale 1e-12, codes 0
    q = pkg.quantize_rows_int8_convrot(x.to(DEV))
    oa, sa = vo.int8_quantize_rows_convrot(x.float())
    assert torch.equal(q.scale.cpu(), sa)
    assert torch.equal(q.data.cpu(), oa)


def test_convrot_accumulator_bit_exact_and_projection_matches_oracle():
    M, N, K = 300, 640, 5120
    x = _randn(M, K, seed=21).to(torch.bfloat16)
    w = _randn(N, K, seed=22, scale=0.02)
    qa = pkg.quantize_rows_int8_convrot(x.to(DEV))
    qw = pkg.projection.quantize_weight(w, "int8", DEV, convrot=True)
    oa, sa = vo.int8_quantize_rows_convrot(x.float())
    ow, sw = vo.int8_quantize_rows_convrot(w)
    assert torch.equal(qw.data.cpu(), ow) and torch.equal(qw.scale.cpu(), sw)
    acc = pkg.gemm(qa.data, qw.data, kind=2, out_dtype=torch.int32)
    assert torch.equal(acc.cpu(), vo.int8_accumulate(oa, ow))
    maps, info = pkg.prepare_projection_maps([{"to_out_linear.weight": w}], DEV, "int8", convrot=True)
    assert info["convrot"] and int(maps[0][pkg.projection.CONVROT_KEY]) == 256
    got = pkg.project(x.to(DEV), maps[0])
    want = vo.project_int8_convrot(x.float(), w)
    assert rel_l2(got, want) < 5e-3
    # against the exact product the rotation only changes the quantisation error
    assert rel_l2(got, x.double() @ w.double().T) < 3e-2


def test_convrot_spreads_a_channel_outlier():
    """The point of ConvRot: one large channel no longer sets every code's step."""
    M, N, K = 256, 512, 2048
    x = _randn(M, K, seed=31)
    x[:, 100] *= 200
    x = x.to(torch.bfloat16)
    w = _randn(N, K, seed=32, scale=0.02)
    exact = x.double() @ w.double().T
    plain, _ = pkg.prepare_projection_maps([{"to_out_linear.weight": w}], DEV, "int8")
    rot, _ = pkg.prepare_projection_maps([{"to_out_linear.weight": w}], DEV, "int8", convrot=True)
    assert pkg.projection.CONVROT_KEY not in plain[0]
    e_plain = rel_l2(pkg.project(x.to(DEV), plain[0]), exact)
    e_rot = rel_l2(pkg.project(x.to(DEV), rot[0]), exact)
    assert e_rot < 0.5 * e_plain, (e_rot, e_plain)


def test_convrot_rejects_unsupported_widths():
    x = torch.zeros(4, 320, device=DEV, dtype=torch.bfloat16)  # 320 % 256 != 0
    with pytest.raises(ValueError):
        pkg.quantize_rows_int8_convrot(x)


# ------------------------------------------------------------------ the block with stored masters
def _block_case():
    c = dict(vo.CONFIG0, heads=2, dim=128)
    bw = vo.make_block(3, c["hidden"], c["heads"], c["dim"])
    lay_o = vo.config_layout(c)
    x = vo.make_x(3, lay_o.seq_len, c["hidden"]).to(torch.bfloat16).float()
    return c, bw, lay_o, x


def _run_block_maps(bw, maps, c, x, precision):
    from __graft_entry__ import _Attn

    state = pkg.B200State("t", vo.BranchConfig().node_config(), [bw.branch], c["heads"], c["dim"],
                          projection_precision=precision, weight_maps=maps)
    fwd = pkg.make_vdn_forward(_Attn(bw, c["heads"], c["dim"]), state, 0)
    with pkg.publish_layout(pkg.make_layout(c["text"], c["frames"], c["grid"])):
        out = pkg.run_forward_checked(state, fwd, x.to(DEV, torch.bfloat16))
    torch.cuda.synchronize()
    return out


def test_int8_block_runs_a_convrot_to_out_master_as_stored():
    """The reference's INT8 storage of to_out_linear (int8 codes + per-channel scales, ConvRot,
    projection.py:139-206) consumed by the int8 block: branch rows quantised with ConvRot."""
    c, bw, lay_o, x = _block_case()
    maps, _ = pkg.prepare_projection_maps([bw.branch], DEV, "int8", convrot=True)
    assert "to_out_linear.weight" not in maps[0]
    got = _run_block_maps(bw, maps, c, x, "int8")
    want = vo.block_forward(x, bw, lay_o, c["heads"], c["dim"], vo.BranchConfig(), precision="int8",
                            to_out_convrot=True)
    exact = vo.block_forward(x, bw, lay_o, c["heads"], c["dim"], vo.BranchConfig())
    assert rel_l2(got, want) < 2e-2
    assert rel_l2(got, exact) < 3e-2


@pytest.mark.parametrize("stored", ["int8", "int8_convrot", "fp8"])
def test_bf16_block_runs_a_stored_master_as_stored(stored):
    """A bf16 block given a quantised to_out_linear master projects the branch in that
    master's arithmetic, as the reference's project() dispatches on the stored weight
    (projection.py:259-268), while out_proj stays bf16 (the branch delta is as large as the
    output at this size, so a wrong or missing branch projection would show)."""
    c, bw, lay_o, x = _block_case()
    prec = "int8" if stored.startswith("int8") else "fp8"
    maps, _ = pkg.prepare_projection_maps([bw.branch], DEV, prec, skip_end_blocks=0,
                                          convrot=stored == "int8_convrot")
    got = _run_block_maps(bw, maps, c, x, "bf16")
    want = vo.block_forward(x, bw, lay_o, c["heads"], c["dim"], vo.BranchConfig(), precision="bf16",
                            to_out_precision=prec, to_out_convrot=stored == "int8_convrot")
    exact = vo.block_forward(x, bw, lay_o, c["heads"], c["dim"], vo.BranchConfig())
    assert rel_l2(got, want) < (2e-2 if prec == "int8" else 3e-2)
    assert rel_l2(got, exact) < (3e-2 if prec == "int8" else 8e-2)


def test_fp8_block_runs_a_per_tensor_master_as_stored():
    c, bw, lay_o, x = _block_case()
    maps, _ = pkg.prepare_projection_maps([bw.branch], DEV, "fp8", skip_end_blocks=0)
    got = _run_block_maps(bw, maps, c, x, "fp8")
    want = vo.block_forward(x, bw, lay_o, c["heads"], c["dim"], vo.BranchConfig(), precision="fp8")
    assert rel_l2(got, want) < 3e-2
