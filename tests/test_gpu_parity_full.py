"""Parity of the benchmarked block at full size: BASELINE configs 1 and 3.

* Config 1 (31 x 836 + 512 = 26,428 rows, H=40, D=128, hidden 5120): exactly the block
  ``bench.py`` times -- its seeded weights, its seed-1 input, its node config, through the
  drop-in operator -- compared on every output row with the float32 oracle run on the host
  cores (about half a minute on 16 cores).
* Config 3 (80 x 48 grid: 119,552 rows): the single-GPU block and the 8-rank head-sharded
  block (ranks emulated on one GPU, exchange replayed by copies) on a row sample -- every
  text row, rows of both anchor frames (which see every key), and rows at the start, middle
  and end of three interior frames -- against the oracle restricted to those rows (the
  oracle still projects and runs the branch statistics over the whole sequence).

North star's bar for bf16 outputs is 2e-2 relative L2 against the reference's torch path on
identical seeded inputs; the oracle is that path restated.
"""

from __future__ import annotations

import os

import pytest
import torch

import bench
from __graft_entry__ import _Attn, load_package
from oracle import vdn_oracle as vo

pytestmark = pytest.mark.gpu

pkg = load_package()
DEV = torch.device("cuda:0") if torch.cuda.is_available() else None
TOL = 2e-2


def rel_l2(got, want):
    got = got.double().cpu()
    want = want.double().cpu()
    return float((got - want).norm() / want.norm())


def _oracle_fp32(x, bw, lay_o, c, rows=None):
    torch.set_num_threads(os.cpu_count() or 1)
    prev = vo.set_compute_dtype(torch.float32)
    try:
        return vo.block_forward(x, bw, lay_o, c["heads"], c["dim"], vo.BranchConfig(), attention="grouped",
                                rows=rows)
    finally:
        vo.set_compute_dtype(prev)


def _bench_case(config: int):
    """bench.py's weights, input and node config for ``config``."""
    c = dict(bench.CONFIGS[config])
    qkv, qn, kn, out_w, branch = bench.make_weights(c, DEV)
    bw = vo.BlockWeights(qkv=qkv, q_norm=qn, k_norm=kn, out=out_w, branch=branch)
    lay = pkg.make_layout(c["text"], c["frames"], c["grid"])
    g = torch.Generator().manual_seed(1)
    x = torch.randn(lay.seq_len, c["hidden"], generator=g).to(torch.bfloat16)
    return c, bw, lay, x


def _operator_forward(c, bw, lay, x):
    state = pkg.B200State("parity", bench.node_config(), [bw.branch], c["heads"], c["dim"])
    fwd = pkg.make_vdn_forward(_Attn(bw, c["heads"], c["dim"]), state, 0)
    with pkg.publish_layout(lay):
        out = pkg.run_forward_checked(state, fwd, x.to(DEV))
    torch.cuda.synchronize()
    return out.cpu()


def test_config1_block_matches_oracle_on_every_row():
    c, bw, lay, x = _bench_case(1)
    got = _operator_forward(c, bw, lay, x)
    assert torch.isfinite(got.float()).all()
    want = _oracle_fp32(x.float(), bw, vo.config_layout(c), c)
    err = rel_l2(got, want)
    print(f"config 1: rel L2 {err:.3e} over {got.shape[0]} rows")
    assert err < TOL
    # and row class by row class (text rows, anchor frames, interior frames), so a large
    # error confined to a few rows cannot hide in the global norm
    vs, ve, tpf = lay.video_start, lay.video_end, lay.tokens_per_frame
    for name, sl in (("text", slice(0, vs)), ("anchor 0", slice(vs, vs + tpf)),
                     ("interior", slice(vs + tpf, ve - tpf)), ("anchor F-1", slice(ve - tpf, ve))):
        assert rel_l2(got[sl], want[sl]) < TOL, name


def _config3_rows(lay) -> torch.Tensor:
    vs, ve, tpf = lay.video_start, lay.video_end, lay.tokens_per_frame
    picks = [torch.arange(0, vs)]
    for f in (0, lay.num_frames - 1):  # anchor frames: every key visible
        base = vs + f * tpf
        picks += [torch.arange(base, base + 64), torch.arange(base + tpf - 64, base + tpf)]
    for f in (1, lay.num_frames // 2, lay.num_frames - 2):  # interior frames at chunk edges and middle
        base = vs + f * tpf
        picks += [torch.arange(base, base + 64), torch.arange(base + tpf // 2 - 32, base + tpf // 2 + 32),
                  torch.arange(base + tpf - 64, base + tpf)]
    return torch.cat(picks)


def _emulated_sharded_rows(c, bw, lay, x_dev, world, rows):
    """The head-sharded block of ``world`` ranks emulated on one GPU (each rank's phases 1-3,
    the all-to-all replayed by copies, each rank's row-split projection); returns ``rows``."""
    from vdn_b200 import shard as sh

    H, D = c["heads"], c["dim"]
    plans, status = pkg.WindowPlanCache(), pkg.DeviceStatus(DEV)
    stream = torch.cuda.current_stream().cuda_stream
    blocks = [pkg.FusedBlock(bw.qkv, bw.q_norm, bw.k_norm, bw.out, bw.branch, H, D, DEV,
                             shard=sh.HeadShard(r, world, H)) for r in range(world)]
    S = x_dev.shape[0]
    parts = []
    with pkg.cholesky_runtime_scope():
        for b in blocks:
            parts.append(b.forward_heads(x_dev, lay, plans, status))
    x0 = parts[0][0]["xchg"]
    out = torch.zeros(world * x0.chunks * x0.cs, bw.out.shape[0], device=DEV, dtype=torch.bfloat16)
    for r, b in enumerate(blocks):
        ws, linear_active = parts[r]
        xr = ws["xchg"]
        for ch in range(xr.chunks):
            r0, n = xr.rows_of(ch)
            for src in range(world):
                xr.recv[ch][src].copy_(parts[src][0]["xchg"].send[r0:r0 + xr.cs])
            b.project_rows(ws, linear_active, xr.recv[ch], n, out[r0:r0 + xr.cs], status, stream)
    torch.cuda.synchronize()
    status.raise_if_failed()
    return out[:S][rows.to(DEV)].cpu()


def test_config3_row_sample_single_gpu_and_sharded_match_oracle():
    c, bw, lay, x = _bench_case(3)
    rows = _config3_rows(lay)
    got = _operator_forward(c, bw, lay, x)[rows]
    sharded = _emulated_sharded_rows(c, bw, lay, x.to(DEV), 8, rows)
    want = _oracle_fp32(x.float(), bw, vo.config_layout(c), c, rows=rows)
    e1, e8 = rel_l2(got, want), rel_l2(sharded, want)
    print(f"config 3: rel L2 {e1:.3e} (1 GPU), {e8:.3e} (8 ranks emulated) over {len(rows)} rows")
    assert e1 < TOL and e8 < TOL
    # the sharded block sums the output projection's K in another order: close to 1 GPU's
    assert rel_l2(sharded, got) < 2e-3
