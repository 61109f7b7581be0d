"""Config 2 (INT8 projections at the config-1 shape, hidden 5120, H=40, D=128): the int8 codes
and the int32 accumulators of the two projection GEMMs the block runs, bit for bit against the
oracle, on a 512-row sample.

* QKV: the bench's seed-1 block input (512 rows spread over text and video) against the
  bench's W_qkv [15360, 5120] -- K = 5120.
* Output projection: the K-concatenated operand [attention rows | branch rows] against
  [W_out | W_to_out] [5120, 10240] -- K = 10240, the two halves read through the GEMM's
  second operand pointer exactly as the block reads them.

The oracle's exact products are float64 sums of int8 x int8 terms: |sum| <= 10240 * 127^2 <
2^31 < 2^53, so float64 holds them exactly.  The reference's rule (projection.py:259-268, the
plain per-row scheme of config 2) is restated in ``vo.int8_quantize_rows``.
"""

from __future__ import annotations

import pytest
import torch

import bench
from __graft_entry__ import load_package
from oracle import vdn_oracle as vo

pytestmark = pytest.mark.gpu

pkg = load_package()
DEV = torch.device("cuda:0") if torch.cuda.is_available() else None
ROWS = 512


def _exact(qa: torch.Tensor, qw: torch.Tensor) -> torch.Tensor:
    torch.set_num_threads(max(torch.get_num_threads(), 8))
    acc = qa.to(torch.float64) @ qw.to(torch.float64).T
    assert acc.abs().max() < 2**31
    return acc.to(torch.int32)


def _sample_rows(S: int) -> torch.Tensor:
    g = torch.Generator().manual_seed(7)
    return torch.sort(torch.randperm(S, generator=g)[:ROWS]).values


def test_int8_qkv_gemm_bit_exact_at_config1_shape():
    c = bench.CONFIGS[1]
    qkv, _, _, _, _ = bench.make_weights(c, "cpu")
    x = bench.bench_input(c)[_sample_rows(c["text"] + c["frames"] * c["grid"][0] * c["grid"][1])]
    assert qkv.shape == (3 * c["heads"] * c["dim"], c["hidden"]) and x.shape == (ROWS, c["hidden"])
    qa = pkg.quantize_rows_int8(x.to(DEV))
    qw = pkg.quantize_rows_int8(qkv.to(DEV, torch.bfloat16))
    oa, sa = vo.int8_quantize_rows(x.float())
    ow, sw = vo.int8_quantize_weight(qkv.to(torch.bfloat16).float())
    assert torch.equal(qa.data.cpu(), oa) and torch.equal(qa.scale.cpu(), sa)
    assert torch.equal(qw.data.cpu(), ow) and torch.equal(qw.scale.cpu(), sw)
    acc = pkg.gemm(qa.data, qw.data, kind=2, out_dtype=torch.int32)
    assert torch.equal(acc.cpu(), _exact(oa, ow))


def test_int8_output_projection_k_concat_bit_exact_at_config1_shape():
    c = bench.CONFIGS[1]
    _, _, _, out_w, branch = bench.make_weights(c, "cpu")
    inner = c["heads"] * c["dim"]
    w_cat = torch.cat([out_w, branch["to_out_linear.weight"]], dim=1).to(torch.bfloat16)  # [5120, 10240]
    g = torch.Generator().manual_seed(11)
    attn_rows = (torch.randn(ROWS, inner, generator=g) * 0.5).to(torch.bfloat16)
    branch_rows = (torch.randn(ROWS, inner, generator=g) * 2.0).to(torch.bfloat16)
    cat = torch.cat([attn_rows, branch_rows], dim=1)
    qa = pkg.quantize_rows_int8(cat.to(DEV))
    qw = pkg.quantize_rows_int8(w_cat.to(DEV))
    oa, _ = vo.int8_quantize_rows(cat.float())
    ow, _ = vo.int8_quantize_weight(w_cat.float())
    assert torch.equal(qa.data.cpu(), oa) and torch.equal(qw.data.cpu(), ow)
    # the block's K-concatenated read: first operand = columns [0, 5120), second = the rest
    a1 = qa.data[:, :inner]
    a2 = qa.data[:, inner:]
    acc = pkg.gemm(a1, qw.data, a2=a2, k_split=inner, kind=2, out_dtype=torch.int32)
    assert torch.equal(acc.cpu(), _exact(oa, ow))
