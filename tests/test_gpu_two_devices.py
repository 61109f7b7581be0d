"""One process driving two GPUs: every kernel that opts into more than 48 KB of dynamic shared
memory does so per device, so a launch on the second device after the first succeeds and
gives the same bits (run where two GPUs are visible)."""

from __future__ import annotations

import pytest
import torch

from __graft_entry__ import load_package
from oracle import vdn_oracle as vo

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                                 reason="needs two GPUs in one process")]

pkg = load_package()


def test_attention_and_gemm_run_on_two_devices_in_one_process():
    c = dict(text=64, frames=9, grid=(8, 12), heads=2, dim=128)
    lay = pkg.make_layout(c["text"], c["frames"], c["grid"])
    S, H, D = lay.seq_len, c["heads"], c["dim"]
    g = torch.Generator().manual_seed(3)
    q, k, v = ((torch.randn(S, H, D, generator=g) * 0.5).to(torch.bfloat16) for _ in range(3))
    a = torch.randn(300, 512, generator=g).to(torch.bfloat16)
    b = (torch.randn(256, 512, generator=g) * 0.02).to(torch.bfloat16)
    outs = []
    for dev in (torch.device("cuda:0"), torch.device("cuda:1")):
        with torch.cuda.device(dev):
            att = pkg.window_softmax_b200(q.to(dev), k.to(dev), v.to(dev), lay.video_start, lay.video_end,
                                          lay.num_frames, lay.tokens_per_frame, lay.bounds, D ** -0.5,
                                          lay.anchor_frames, cache=pkg.WindowPlanCache())
            mm = pkg.gemm(a.to(dev), b.to(dev))
            torch.cuda.synchronize(dev)
            outs.append((att.cpu(), mm.cpu()))
    assert torch.equal(outs[0][0], outs[1][0]) and torch.equal(outs[0][1], outs[1][1])
    want = vo.window_attention(q.double(), k.double(), v.double(), lay.video_start, lay.video_end, lay.num_frames,
                               lay.tokens_per_frame, list(lay.bounds), D ** -0.5, lay.anchor_frames)
    err = float((outs[0][0].double() - want).norm() / want.norm())
    assert err < 2e-2
