"""The FP8 projection entry point that allocates nothing.

Callers that cannot allocate device memory while they run (code inside a memory arena it
does not own, hosts that give the library a fixed device budget) use
``vdn_fp8_linear_noalloc``: the quantised activations, amax and scale live in the library's
own fixed-size device array.  This file checks, through the C ABI, that it returns what the
allocating path (``vdn_quant_fp8_tensor`` into caller buffers, then ``vdn_gemm``) returns,
on two calls in a row whose inputs differ, so a stale amax from the first call would show.
It is named to be collected last.
"""

from __future__ import annotations

import pytest
import torch

from __graft_entry__ import load_package

pytestmark = pytest.mark.gpu

pkg = load_package()


def _allocating_reference(x, w_q, w_scale):
    """Existing path: quantise x into caller-provided buffers, then the fp8 GEMM."""
    qa = pkg.quantize_tensor_fp8(x)
    return pkg.gemm(qa.data, w_q, kind=1, dev_scale0=qa.scale, dev_scale1=w_scale)


def _noalloc(x, w_q, w_scale, out):
    lib = pkg._lib
    status = lib.DeviceStatus(x.device)
    lib.call("vdn_fp8_linear_noalloc", x.data_ptr(), x.stride(0), x.shape[0], x.shape[1], w_q.data_ptr(),
             w_q.stride(0), w_q.shape[0], w_scale.data_ptr(), out.data_ptr(), out.stride(0), status.err_ptr,
             lib.stream_handle(x.device))
    return status


def test_noalloc_fp8_projection_matches_allocating_path_twice():
    dev = torch.device("cuda:0")
    g = torch.Generator().manual_seed(77)
    M, K, N = 600, 1024, 768
    w = (torch.randn(N, K, generator=g) * 0.02).to(dev)
    wq = pkg.quantize_tensor_fp8(w)
    for scale in (1.0, 0.05):  # second call has a much smaller amax than the first
        x = (torch.randn(M, K, generator=g) * scale).to(dev, torch.bfloat16)
        want = _allocating_reference(x, wq.data, wq.scale)
        out = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
        status = _noalloc(x, wq.data, wq.scale, out)
        torch.cuda.synchronize()
        status.raise_if_failed()
        rel = float((out.double() - want.double()).norm() / want.double().norm())
        assert rel < 1e-6, rel


def test_noalloc_rejects_problems_larger_than_its_scratch():
    dev = torch.device("cuda:0")
    M, K, N = 4096 + 1, 4096, 16  # 16,781,312 elements > 16,777,216
    x = torch.zeros(M, K, device=dev, dtype=torch.bfloat16)
    wq = torch.zeros(N, K, device=dev, dtype=torch.float8_e4m3fn)
    ws = torch.ones(1, device=dev)
    out = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="fixed device scratch"):
        _noalloc(x, wq, ws, out)


@pytest.mark.parametrize("bad", ["ldx", "ldw", "ldo"])
def test_noalloc_rejects_row_pitches_shorter_than_a_row(bad):
    """A pitch below its row length would make rows overlap: rejected before any launch."""
    dev = torch.device("cuda:0")
    M, K, N = 64, 256, 128
    x = torch.zeros(M, K, device=dev, dtype=torch.bfloat16)
    wq = torch.zeros(N, K, device=dev, dtype=torch.float8_e4m3fn)
    ws = torch.ones(1, device=dev)
    out = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
    lib = pkg._lib
    status = lib.DeviceStatus(dev)
    ldx, ldw, ldo = (K - 16 if bad == "ldx" else K), (K - 16 if bad == "ldw" else K), (N - 8 if bad == "ldo" else N)
    with pytest.raises(ValueError, match="invalid argument"):
        lib.call("vdn_fp8_linear_noalloc", x.data_ptr(), ldx, M, K, wq.data_ptr(), ldw, N, ws.data_ptr(),
                 out.data_ptr(), ldo, status.err_ptr, lib.stream_handle(dev))
