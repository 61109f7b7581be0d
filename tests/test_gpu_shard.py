"""GPU tests of the head-sharded block.

* On one GPU the ranks are emulated in one process: each rank's FusedBlock runs its heads
  (phases 1-3), the all-to-all is replayed by copies between the ranks' buffers, and each
  rank runs its row-split projection.  INT8 must reproduce the unsharded block bit for bit
  (every per-head value and every projected row is the same arithmetic); bf16 sums the
  output projection's K in rank-major order, so it is compared within 2e-3.
* With two or more GPUs, two NCCL ranks run the patched forward (B200State with
  shard_heads=True) and are compared with the unsharded block and the oracle.
"""

from __future__ import annotations

import os
import socket

import pytest
import torch

from __graft_entry__ import _Attn, load_package
from oracle import vdn_oracle as vo

pytestmark = pytest.mark.gpu

pkg = load_package()
from vdn_b200 import shard as sh  # noqa: E402

DEV = torch.device("cuda:0") if torch.cuda.is_available() else None


def rel_l2(got, want):
    got = got.double().cpu()
    want = want.double().cpu()
    return float((got - want).norm() / want.norm())


def _block(bw, heads, dim, precision, shard=None, exchange="rows"):
    return pkg.FusedBlock(bw.qkv, bw.q_norm, bw.k_norm, bw.out, bw.branch, heads, dim, DEV, precision=precision,
                          shard=shard, exchange=exchange)


def _emulated_sharded_forward(bw, lay, heads, dim, x, precision, world, exchange="rows"):
    """Every rank's phases 1-3, then the chunked exchange replayed by copies between the
    ranks' buffers and each rank's projection; returns rank 0's rows for "rows" (every rank
    writes its own row blocks into one output) or, for "heads", checks that all ranks project
    the same output and returns it."""
    plans = pkg.WindowPlanCache()
    status = pkg.DeviceStatus(DEV)
    stream = torch.cuda.current_stream().cuda_stream
    blocks = [_block(bw, heads, dim, precision, sh.HeadShard(r, world, heads), exchange) for r in range(world)]
    parts = [b.forward_heads(x, lay, plans, status) for b in blocks]
    S = x.shape[0]
    x0 = parts[0][0]["xchg"]
    cs = x0.cs
    rows_total = x0.send.shape[0]
    outs = [torch.zeros(rows_total, bw.out.shape[0], device=DEV, dtype=torch.bfloat16)
            for _ in range(world if exchange == "heads" else 1)]
    for r, b in enumerate(blocks):
        ws, linear_active = parts[r]
        xr = ws["xchg"]
        out = outs[r if exchange == "heads" else 0]
        for c in range(xr.chunks):
            r0, rows = xr.rows_of(c)
            for src in range(world):
                # "rows": rank r's block of chunk c from every rank; "heads": chunk c of every rank
                xr.recv[c][src].copy_(parts[src][0]["xchg"].send[r0:r0 + cs])
            b.project_rows(ws, linear_active, xr.recv[c], rows, out[r0:r0 + cs], status, stream)
    torch.cuda.synchronize()
    status.raise_if_failed()
    for other in outs[1:]:
        assert torch.equal(other[:S], outs[0][:S])
    return outs[0][:S]


GEOMETRIES = {
    "config0": (vo.CONFIG0, (2,)),
    "d128_ragged": (dict(text=64, frames=11, grid=(9, 14), heads=4, dim=128, hidden=512), (2, 4)),
}


@pytest.mark.parametrize("exchange", ["rows", "heads"])
@pytest.mark.parametrize("precision", ["bf16", "int8"])
@pytest.mark.parametrize("geom", sorted(GEOMETRIES))
def test_sharded_block_emulated_on_one_gpu(geom, precision, exchange, monkeypatch):
    monkeypatch.setattr(pkg.hybrid, "EXCHANGE_MIN_ROWS", 1)  # chunked exchange even at test sizes
    c, worlds = GEOMETRIES[geom]
    H, D, hidden = c["heads"], c["dim"], c["hidden"]
    bw = vo.make_block(5, hidden, H, D)
    lay = pkg.make_layout(c["text"], c["frames"], c["grid"])
    x = vo.make_x(5, lay.seq_len, hidden).to(DEV, torch.bfloat16)
    full = _block(bw, H, D, precision)
    ref = full.forward(x, lay, pkg.WindowPlanCache(), pkg.DeviceStatus(DEV)).clone()
    torch.cuda.synchronize()
    for world in worlds:
        got = _emulated_sharded_forward(bw, lay, H, D, x, precision, world, exchange)
        if precision == "int8":
            assert torch.equal(got, ref), f"world {world}: int8 sharded output differs from the unsharded block"
        else:
            assert rel_l2(got, ref) < 2e-3, world
    if precision == "bf16":
        want = vo.block_forward(x.float().cpu(), bw, vo.config_layout(c), H, D, vo.BranchConfig())
        assert rel_l2(got, want) < 2e-2


def test_grouped_k_gemm_matches_torch():
    gen = torch.Generator().manual_seed(11)
    G, Mp, Kg, N, M = 4, 300, 192, 520, 257
    a3 = (torch.randn(G, Mp, Kg, generator=gen) * 0.5).to(DEV, torch.bfloat16)
    b = (torch.randn(N, G * Kg, generator=gen) * 0.5).to(DEV, torch.bfloat16)
    got = pkg.projection.gemm_grouped_k(a3, b, rows=M, out_dtype=torch.float32)
    want = sh.concat_rows(a3.float(), M) @ b.float().T
    torch.testing.assert_close(got, want, rtol=1e-4, atol=1e-3)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _nccl_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import datetime

    import torch.distributed as dist

    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    try:
        pkg_r = load_package()
        c = dict(text=64, frames=11, grid=(9, 14), heads=4, dim=128, hidden=512)
        H, D, hidden = c["heads"], c["dim"], c["hidden"]
        bw = vo.make_block(6, hidden, H, D)
        lay = pkg_r.make_layout(c["text"], c["frames"], c["grid"])
        x = vo.make_x(6, lay.seq_len, hidden).to(f"cuda:{rank}", torch.bfloat16)
        res = {}
        for exchange, precision in [(e, p) for e in ("rows", "heads") for p in ("bf16", "int8", "fp8")]:
            state = pkg_r.B200State("t", vo.BranchConfig().node_config(), [bw.branch], H, D,
                                    projection_precision=precision, shard_heads=True, shard_exchange=exchange)
            fwd = pkg_r.make_vdn_forward(_Attn(bw, H, D), state, 0)
            with pkg_r.publish_layout(lay):
                got = pkg_r.run_forward_checked(state, fwd, x)
            single = pkg_r.B200State("t", vo.BranchConfig().node_config(), [bw.branch], H, D,
                                     projection_precision=precision)
            fwd1 = pkg_r.make_vdn_forward(_Attn(bw, H, D), single, 0)
            with pkg_r.publish_layout(lay):
                ref = pkg_r.run_forward_checked(single, fwd1, x)
            torch.cuda.synchronize()
            res[(exchange, precision)] = (bool(torch.equal(got, ref)), rel_l2(got, ref))
            if precision == "bf16":
                want = vo.block_forward(x.float().cpu(), bw, vo.config_layout(c), H, D, vo.BranchConfig())
                res[(exchange, "oracle")] = rel_l2(got, want)
        # the DiT block around it: MLP token-parallel on each rank's rows before the gather
        dw = vo.make_dit(8, hidden, H, D, 512, activation="swiglu")
        mods = [m.to(f"cuda:{rank}", torch.bfloat16) for m in vo.make_mods(8, 2, hidden)]
        group = torch.tensor([0] * lay.video_start + [1] * (lay.seq_len - lay.video_start), dtype=torch.int32,
                             device=f"cuda:{rank}")
        for precision in ("bf16", "int8"):
            outs = []
            for shard in (sh.default_shard(H), None):
                fb = pkg_r.FusedBlock(dw.attn.qkv, dw.attn.q_norm, dw.attn.k_norm, dw.attn.out, dw.attn.branch, H, D,
                                      f"cuda:{rank}", precision=precision, shard=shard)
                blk = pkg_r.B200DiTBlock(fb, dw.norm1, dw.eps, dw.norm2, dw.eps, dw.fc1, dw.fc1_b, dw.fc2, dw.fc2_b,
                                         f"cuda:{rank}", precision=precision)
                st = pkg_r.DeviceStatus(f"cuda:{rank}")
                with pkg_r.cholesky_runtime_scope():
                    outs.append(blk.forward(x, mods, group, lay, pkg_r.WindowPlanCache(), st).clone())
                torch.cuda.synchronize()
                st.raise_if_failed()
            res["dit_" + precision] = (bool(torch.equal(outs[0], outs[1])), rel_l2(outs[0], outs[1]))
        q.put((rank, res))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_sharded_block_on_two_gpus_over_nccl():
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_nccl_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=600) for _ in procs)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for rank, res in results.items():
        for exchange in ("rows", "heads"):
            assert res[(exchange, "int8")][0], (rank, exchange, res)
            # fp8: the row split's amax all-reduce restores the whole tensor's scale; the head
            # gather quantises every row on every rank
            assert res[(exchange, "fp8")][0], (rank, exchange, res)
            assert res[(exchange, "bf16")][1] < 2e-3, (rank, exchange, res)
            assert res[(exchange, "oracle")] < 2e-2, (rank, exchange, res)
        assert res["dit_int8"][0], (rank, res)
        assert res["dit_bf16"][1] < 2e-3, (rank, res)
