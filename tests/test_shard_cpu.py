"""CPU tests of head sharding (no GPU): the weight slicing, the rank-major order of the
output weight, the row blocks, and the all-to-all / all-gather exchange run as two and
four gloo ranks.  Each rank computes its heads' outputs with the float64 oracle from the
sliced weights; the exchanged, row-split projection must equal the unsharded oracle block."""

from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from __graft_entry__ import load_package
from oracle import vdn_oracle as vo

pkg = load_package()
from vdn_b200 import shard as sh  # noqa: E402


@pytest.mark.parametrize("S", [1, 7, 64, 26428, 120552])
@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_row_blocks_tile_the_sequence(S, world):
    s = sh.HeadShard(0, world, 40)
    covered = []
    for r in range(world):
        r0, n = s.rows_of(S, r)
        assert 0 <= n <= s.row_block(S)
        covered += list(range(r0, r0 + n))
    assert covered == list(range(S))


@pytest.mark.parametrize("S", [1, 7, 64, 26428])
@pytest.mark.parametrize("world,chunks", [(1, 1), (2, 1), (2, 4), (8, 4), (3, 2)])
def test_exchange_blocks_tile_the_sequence(S, world, chunks):
    sh_ = sh.HeadShard(0, world, 24)
    x = sh.RowExchange(sh_, S, 8, 4, "cpu", dtype=torch.float32, chunks=chunks)
    covered = []
    for c in range(chunks):
        for r in range(world):
            r0, n = x.rows_of(c, r)
            assert r0 == (c * world + r) * x.cs and 0 <= n <= x.cs
            covered += list(range(r0, r0 + n))
    assert covered == list(range(S))
    assert x.send.shape[0] == world * chunks * x.cs >= S


@pytest.mark.parametrize("S", [1, 7, 64, 26428])
@pytest.mark.parametrize("world,chunks", [(2, 1), (2, 4), (8, 3)])
def test_head_gather_chunks_tile_the_sequence(S, world, chunks):
    x = sh.HeadGather(sh.HeadShard(0, world, 24), S, 8, 4, "cpu", dtype=torch.float32, chunks=chunks)
    covered = []
    for c in range(chunks):
        r0, n = x.rows_of(c, 1)
        assert (r0, r0 + n) == (x.chunk_rows(c)[0], max(x.chunk_rows(c)))
        covered += list(range(r0, r0 + n))
    assert covered == list(range(S))
    assert x.recv.shape == (chunks, world, x.cs, 8)


def test_head_shard_rejects_uneven_split():
    with pytest.raises(ValueError):
        sh.HeadShard(0, 3, 40)
    with pytest.raises(ValueError):
        sh.HeadShard(2, 2, 40)


def test_qkv_rows_select_the_local_heads():
    H, D = 4, 3
    idx = sh.qkv_row_index(H, D, slice(2, 4))
    inner = H * D
    want = list(range(6, 12)) + list(range(inner + 6, inner + 12)) + list(range(2 * inner + 6, 2 * inner + 12))
    assert idx.tolist() == want


def test_rank_major_weight_matches_concat_rows():
    gen = torch.Generator().manual_seed(3)
    H, D, hidden, world, S = 8, 4, 16, 4, 13
    inner, hl = H * D, H // world
    out_w = torch.randn(hidden, inner, generator=gen, dtype=torch.float64)
    to_out = torch.randn(hidden, inner, generator=gen, dtype=torch.float64)
    flat = torch.randn(S, inner, generator=gen, dtype=torch.float64)
    branch = torch.randn(S, inner, generator=gen, dtype=torch.float64)
    want = flat @ out_w.T + branch @ to_out.T
    w_rm = sh.rank_major_out_weight(out_w, to_out, H, D, world)
    # what rank r sends: its heads' [flat | branch] columns; the receive buffer is [world, rows, 2*hl*D]
    recv = torch.stack([torch.cat([flat[:, r * hl * D:(r + 1) * hl * D], branch[:, r * hl * D:(r + 1) * hl * D]], 1)
                        for r in range(world)])
    got = sh.concat_rows(recv, S) @ w_rm.T
    torch.testing.assert_close(got, want)
    f2, b2 = sh.split_heads_outputs(sh.concat_rows(recv, S), world, hl * D)
    torch.testing.assert_close(f2, flat)
    torch.testing.assert_close(b2, branch)


def test_slice_branch_weights_shapes():
    cfg = vo.CONFIG0
    H, D, hidden = cfg["heads"], cfg["dim"], cfg["hidden"]
    w = vo.make_branch_weights(torch.Generator().manual_seed(0), hidden, H, D)
    w["to_out_linear.weight_fp8"] = torch.zeros(1)
    loc = sh.slice_branch_weights(w, H, D, slice(2, 4))
    assert "to_out_linear.weight_fp8" not in loc
    assert loc["beta_proj.weight"].shape == (2, hidden)
    assert loc["alpha.A_log"].shape == (2,)
    assert loc["alpha.up.weight"].shape == (2 * D, D)
    assert loc["short_conv.k_sp.weight"].shape[0] == 2 * D
    assert loc["to_out_linear.weight"].shape == (hidden, 2 * D)
    assert loc["norm.weight"] is w["norm.weight"]
    torch.testing.assert_close(loc["output_gate.up.bias"], w["output_gate.up.bias"][2 * D:4 * D])


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _heads_outputs(x, bw: vo.BlockWeights, lay, heads, dim, shard: sh.HeadShard, cfg):
    """[S, 2*H/g*D] = [gated softmax | branch readout] of this rank's heads (oracle)."""
    hs = shard.head_slice
    hl = shard.heads_local
    local = vo.BlockWeights(qkv=bw.qkv[sh.qkv_row_index(heads, dim, hs)], q_norm=bw.q_norm, k_norm=bw.k_norm,
                            out=bw.out[:, hs.start * dim:hs.stop * dim],
                            branch=sh.slice_branch_weights(bw.branch, heads, dim, hs))
    _, parts = vo.block_forward(x, local, lay, hl, dim, cfg, return_parts=True)
    S = x.shape[0]
    flat = (parts["softmax"] * parts["gate"].reshape(S, hl, 1)).reshape(S, hl * dim)
    branch = torch.zeros(S, hl * dim, dtype=flat.dtype)
    if "readout" in parts:
        branch[lay.video_start:lay.video_end] = parts["readout"]
    return torch.cat([flat, branch], 1)


def _worker(rank, world, port, anchors, chunks, q, kind="rows"):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        cfg = vo.CONFIG0
        H, D, hidden = cfg["heads"], cfg["dim"], cfg["hidden"]
        lay = vo.config_layout(cfg, anchor_frames=anchors)
        bw = vo.make_block(0, hidden, H, D)
        x = vo.make_x(0, lay.seq_len, hidden).double()
        bcfg = vo.BranchConfig()
        shard = sh.default_shard(H)
        assert shard.rank == rank and shard.world == world
        xchg = sh.EXCHANGES[kind](shard, lay.seq_len, 2 * shard.heads_local * D, hidden, "cpu",
                                  dtype=torch.float64, chunks=chunks)
        xchg.send[:lay.seq_len] = _heads_outputs(x, bw, lay, H, D, shard, bcfg)
        xchg.exchange()
        w_rm = sh.rank_major_out_weight(bw.out.double(), bw.branch["to_out_linear.weight"].double(), H, D, world)

        def project(recv, rows, out_rows, row0):
            if rows:
                out_rows[:rows] = sh.concat_rows(recv, rows) @ w_rm.T

        got = xchg.project_and_gather(project)
        want = vo.block_forward(x, bw, lay, H, D, bcfg)
        err = float((got - want).norm() / want.norm())
        q.put((rank, err, tuple(got.shape)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,anchors,chunks,kind", [(2, "both", 3, "rows"), (4, "none", 1, "rows"),
                                                       (2, "both", 2, "heads"), (4, "none", 3, "heads")])
def test_sharded_block_matches_unsharded_oracle_on_gloo_ranks(world, anchors, chunks, kind):
    """Both exchanges: all-to-all by row block + row-split projection + all-gather of the rows,
    and all-gather of the per-head outputs + the whole projection on every rank."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, anchors, chunks, q, kind)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    seq = vo.config_layout(vo.CONFIG0).seq_len
    for rank, err, shape in results:
        assert shape == (seq, vo.CONFIG0["hidden"])
        assert err < 1e-12, (rank, err)



def _leaving_worker(rank, world, port, q):
    """Rank 1 stops on the host before the exchange (between steps, none of its collectives in
    flight) and leaves; rank 0 goes on to the exchange, which must end with an error, bounded
    by the process group's timeout, instead of waiting for good."""
    import datetime

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    shard = sh.default_shard(4)
    xchg = sh.RowExchange(shard, 64, 2 * shard.heads_local * 8, 32, "cpu", dtype=torch.float64)
    if rank == 1:
        result = "left"
    else:
        xchg.send.normal_()
        try:
            xchg.exchange()
            xchg.project_and_gather(lambda recv, rows, out_rows, row0: None)
            result = "completed"
        except Exception as exc:  # noqa: BLE001 - the backend's error is the expected outcome
            result = f"error: {type(exc).__name__}: {exc}"
    q.put((rank, result))
    q.close()
    q.join_thread()  # flush the message before the hard exit
    os._exit(0)  # no teardown: the group is broken, its destructor would wait on the peer


def test_exchange_ends_with_an_error_when_a_rank_leaves():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_leaving_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    try:
        results = dict(q.get(timeout=120) for _ in procs)
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    assert results[1] == "left"
    assert results[0].startswith("error"), results[0]
