"""Projections on sm_100a tensor cores (replaces vdn_h3/projection.py + vdn_h3/fp8.py).

``project(rows, weights)`` keeps the reference dispatch on the stored weight
(projection.py:259-268): a bf16 ``to_out_linear.weight`` runs the bf16 tcgen05 GEMM; a
quantised ``to_out_linear.weight_fp8`` with ``to_out_linear.weight_scale`` runs the
e4m3 (per-tensor) or int8 (per-output-channel weight, per-token activation) GEMM with
the dequantisation fused into the epilogue.  ``prepare_projection_maps`` builds those
quantised masters (fp8.py:168-222, projection.py:139-232); the int8 scheme is the
config-2 one (symmetric, round-half-even, fp32 scales) unless ``convrot=True`` asks for
ConvRot (projection.py:74-97, :243-256): both operands rotated per group of 256 channels
by a regular Hadamard matrix before the same per-row quantisation; such a map carries
``to_out_linear.convrot_groupsize`` and ``project`` rotates the activations to match.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from . import _lib

BF16_WEIGHT_KEY = "to_out_linear.weight"
QUANT_WEIGHT_KEY = "to_out_linear.weight_fp8"
QUANT_SCALE_KEY = "to_out_linear.weight_scale"
PROJECTION_PRECISIONS = ("bf16", "fp8", "int8")
DEFAULT_FP8_SKIP_END_BLOCKS = 4  # fp8.py:35

KIND = {"bf16": 0, "fp8": 1, "int8": 2}
CONVROT_GROUP = 256  # projection.py:44 (INT8_CONVROT_GROUP)
CONVROT_KEY = "to_out_linear.convrot_groupsize"


@dataclass
class QuantizedMatrix:
    """A [N, K] weight (or [M, K] activation) quantised for the tcgen05 GEMM."""

    data: torch.Tensor  # int8 / float8_e4m3fn, row-major [rows, K]
    scale: torch.Tensor  # int8: [rows] fp32; fp8: [1] fp32 (device scalar)
    precision: str


def _stream(t):
    return _lib.stream_handle(t.device)


def quantize_rows_int8(x: torch.Tensor, out: QuantizedMatrix | None = None) -> QuantizedMatrix:
    """Per-row symmetric int8 of a bf16/fp32 [rows, K] tensor (round half to even)."""
    _lib.require_cuda(x)
    if x.stride(-1) != 1:
        x = x.contiguous()
    rows, K = x.shape
    if out is None:
        out = QuantizedMatrix(torch.empty(rows, K, device=x.device, dtype=torch.int8),
                              torch.empty(rows, device=x.device, dtype=torch.float32), "int8")
    src = 0 if x.dtype == torch.bfloat16 else 1
    if src == 1 and x.dtype != torch.float32:
        x = x.float()
    _lib.call("vdn_quant_int8_rows", src, x.data_ptr(), x.stride(0), rows, K, out.data.data_ptr(),
              out.data.stride(0), out.scale.data_ptr(), _stream(x))
    return out


def quantize_rows_int8_convrot(x: torch.Tensor, out: QuantizedMatrix | None = None,
                               group: int = CONVROT_GROUP) -> QuantizedMatrix:
    """ConvRot int8 of a [rows, K] tensor (its bf16 copy): every 256-channel group of a row
    rotated by R/16 (R the fourth Kronecker power of the regular Hadamard J - 2I), then the
    per-row rule of ``quantize_rows_int8``.  Rows are tokens for activations and output
    channels for weights (projection.py:74-97: the weight is quantised from bf16)."""
    _lib.require_cuda(x)
    if x.dtype != torch.bfloat16:
        x = x.to(torch.bfloat16)
    if x.stride(-1) != 1:
        x = x.contiguous()
    rows, K = x.shape
    if out is None:
        out = QuantizedMatrix(torch.empty(rows, K, device=x.device, dtype=torch.int8),
                              torch.empty(rows, device=x.device, dtype=torch.float32), "int8")
    _lib.call("vdn_quant_int8_rows_convrot", x.data_ptr(), x.stride(0), rows, K, int(group),
              out.data.data_ptr(), out.data.stride(0), out.scale.data_ptr(), _stream(x))
    return out


def quantize_tensor_fp8(x: torch.Tensor, out: QuantizedMatrix | None = None,
                        work: torch.Tensor | None = None, amax_reduce=None) -> QuantizedMatrix:
    """Per-tensor e4m3 of a bf16/fp32 [rows, K] tensor (fp8.py:99-133, per_tensor=True).
    ``amax_reduce(amax)``, when given, combines the device amax [1] fp32 in place (an
    all-reduce MAX over the ranks that each hold some rows of the tensor) before the cast."""
    _lib.require_cuda(x)
    if x.stride(-1) != 1:
        x = x.contiguous()
    rows, K = x.shape
    if out is None:
        out = QuantizedMatrix(torch.empty(rows, K, device=x.device, dtype=torch.float8_e4m3fn),
                              torch.empty(1, device=x.device, dtype=torch.float32), "fp8")
    if work is None:
        work = torch.empty(1, device=x.device, dtype=torch.float32)
    src = 0 if x.dtype == torch.bfloat16 else 1
    if src == 1 and x.dtype != torch.float32:
        x = x.float()
    if amax_reduce is None:
        _lib.call("vdn_quant_fp8_tensor", src, x.data_ptr(), x.stride(0), rows, K, out.data.data_ptr(),
                  out.data.stride(0), work.data_ptr(), out.scale.data_ptr(), _stream(x))
        return out
    _lib.call("vdn_fp8_amax", src, x.data_ptr(), x.stride(0), rows, K, work.data_ptr(), _stream(x))
    amax_reduce(work)
    _lib.call("vdn_fp8_cast", src, x.data_ptr(), x.stride(0), rows, K, work.data_ptr(), out.data.data_ptr(),
              out.data.stride(0), out.scale.data_ptr(), _stream(x))
    return out


def quantize_weight(w: torch.Tensor, precision: str, device, *, convrot: bool = False) -> QuantizedMatrix:
    if precision == "int8" and convrot:
        return quantize_rows_int8_convrot(w.detach().to(device=device, dtype=torch.bfloat16).contiguous())
    w = w.detach().to(device=device, dtype=torch.float32).contiguous()
    if precision == "int8":
        return quantize_rows_int8(w)
    if precision == "fp8":
        return quantize_tensor_fp8(w)
    raise ValueError(f"unknown quantised precision {precision!r}")


def convrot_matrix(group: int = CONVROT_GROUP) -> torch.Tensor:
    """The ConvRot group rotation R / sqrt(group) (float64, symmetric, its own inverse), R the
    Kronecker power of the order-4 regular Hadamard matrix J - 2I."""
    r4 = torch.ones(4, 4, dtype=torch.float64) - 2 * torch.eye(4, dtype=torch.float64)
    r = torch.ones(1, 1, dtype=torch.float64)
    while r.shape[0] < group:
        r = torch.kron(r, r4)
    if r.shape[0] != group:
        raise ValueError("ConvRot group must be a power of 4")
    return r / math.sqrt(group)


def dequantize_projection_weight(q: torch.Tensor, scale: torch.Tensor, convrot_group=None) -> torch.Tensor:
    """float32 [N, K] weight of a stored quantised ``to_out_linear`` master: int8 codes times
    their per-channel scale, or e4m3 codes times a per-tensor ([1, 1]) or per-channel ([1, N],
    fp8.py:88-96) scale; a ConvRot master is rotated back (the rotation is its own inverse).
    Setup-time only, on the host."""
    w = q.detach().to("cpu").to(torch.float64)
    s = scale.detach().to("cpu", torch.float64).reshape(-1)
    if s.numel() == 1:
        w = w * s[0]
    elif s.numel() == w.shape[0]:
        w = w * s[:, None]
    else:
        raise ValueError("quantised projection scale matches neither the tensor nor its rows")
    if convrot_group is not None:
        g = int(convrot_group)
        n, k = w.shape
        w = (w.reshape(n, k // g, g) @ convrot_matrix(g)).reshape(n, k)
    return w.to(torch.float32)


def gemm(a, b, *, out=None, out_dtype=torch.bfloat16, alpha=1.0, a2=None, k_split=None, row_scale=None,
         col_scale=None, dev_scale0=None, dev_scale1=None, col_bias=None, sigmoid=False, addend=None,
         status: _lib.DeviceStatus | None = None, kind=0):
    """out = epilogue(a @ b^T) on the tcgen05 GEMM.  a: [M, K1] (and a2 [M, K-K1]); b: [N, K]."""
    _lib.require_cuda(a, b)
    M = a.shape[0]
    N, K = b.shape
    if out is None:
        out = torch.empty(M, N, device=a.device, dtype=out_dtype)
    okind = {torch.bfloat16: 0, torch.float32: 1, torch.int32: 2}[out.dtype]
    st = status or _lib.DeviceStatus(a.device)
    _lib.call("vdn_gemm", kind, a.data_ptr(), a.stride(0), _lib.ptr(a2), a2.stride(0) if a2 is not None else 0,
              int(k_split or 0), b.data_ptr(), b.stride(0), out.data_ptr(), out.stride(0), okind, M, N, K,
              float(alpha), _lib.ptr(dev_scale0), _lib.ptr(dev_scale1), _lib.ptr(row_scale), _lib.ptr(col_scale),
              _lib.ptr(col_bias), int(sigmoid), _lib.ptr(addend), addend.stride(0) if addend is not None else 0,
              st.err_ptr, _stream(a))
    if status is None:
        st.raise_if_failed()
    return out


def gemm_grouped_k(a3, b, *, rows=None, out=None, out_dtype=torch.bfloat16, alpha=1.0,
                   status: _lib.DeviceStatus | None = None, kind=0):
    """out = a @ b^T where ``a3`` [G, M', Kg] is read as the K-concatenation of its G slabs
    (first ``rows`` rows of each).  b: [N, G * Kg]."""
    _lib.require_cuda(a3, b)
    if a3.ndim != 3 or a3.stride(-1) != 1:
        raise ValueError("grouped operand must be [groups, rows, kg] with unit inner stride")
    G, Mp, Kg = a3.shape
    M = Mp if rows is None else int(rows)
    N, K = b.shape
    if K != G * Kg or not 0 < M <= Mp:
        raise ValueError("grouped operand does not match the weight's K")
    if out is None:
        out = torch.empty(M, N, device=a3.device, dtype=out_dtype)
    okind = {torch.bfloat16: 0, torch.float32: 1, torch.int32: 2}[out.dtype]
    st = status or _lib.DeviceStatus(a3.device)
    _lib.call("vdn_gemm_grouped_k", kind, a3.data_ptr(), a3.stride(1), a3.stride(0), G, Kg, b.data_ptr(),
              b.stride(0), out.data_ptr(), out.stride(0), okind, M, N, float(alpha), None, None, None, None, None,
              0, None, 0, st.err_ptr, _stream(a3))
    if status is None:
        st.raise_if_failed()
    return out


def project(rows: torch.Tensor, weights) -> torch.Tensor:
    """Dispatch bf16 / fp8 / int8 like projection.py:259-268 (output dtype = rows.dtype)."""
    _lib.require_cuda(rows)
    x = rows.to(torch.bfloat16)
    if x.stride(-1) != 1:
        x = x.contiguous()
    if BF16_WEIGHT_KEY in weights and not isinstance(weights[BF16_WEIGHT_KEY], tuple):
        w = weights[BF16_WEIGHT_KEY].to(device=x.device, dtype=torch.bfloat16).contiguous()
        return gemm(x, w).to(rows.dtype)
    if QUANT_WEIGHT_KEY not in weights:
        raise KeyError("VDN projection state has no supported weight representation")
    q = weights[QUANT_WEIGHT_KEY].to(x.device)
    s = weights[QUANT_SCALE_KEY].to(device=x.device, dtype=torch.float32).reshape(-1).contiguous()
    if q.dtype == torch.int8:
        group = weights.get(CONVROT_KEY)
        if group is not None:
            xa = quantize_rows_int8_convrot(x, group=int(group))
        else:
            xa = quantize_rows_int8(x)
        return gemm(xa.data, q.contiguous(), row_scale=xa.scale, col_scale=s, kind=2).to(rows.dtype)
    xa = quantize_tensor_fp8(x)
    return gemm(xa.data, q.contiguous(), dev_scale0=xa.scale, dev_scale1=s, kind=1).to(rows.dtype)


def prepare_projection_maps(branch_maps, device, precision, *, skip_end_blocks=None, convrot=False):
    """Quantised ``to_out_linear`` masters per block; edge blocks stay bf16 (fp8.py:168-222).
    ``convrot=True`` (int8 only) quantises with ConvRot where K % 256 == 0, as
    projection.py:74-86 does, and marks such a map with ``to_out_linear.convrot_groupsize``."""
    if precision not in PROJECTION_PRECISIONS:
        raise ValueError(f"unknown VDN projection precision {precision!r}")
    if convrot and precision != "int8":
        raise ValueError("ConvRot applies to int8 projections only")
    if precision == "bf16":
        return tuple(dict(b) for b in branch_maps), None
    skip = (DEFAULT_FP8_SKIP_END_BLOCKS if precision == "fp8" else 0) if skip_end_blocks is None else int(skip_end_blocks)
    count = len(branch_maps)
    if count == 0:
        raise ValueError("branch_maps cannot be empty")
    if skip and skip * 2 >= count:
        raise ValueError(f"skip_end_blocks={skip} leaves no quantised interior blocks for {count} branches")
    out = []
    used_convrot = True
    for i, block in enumerate(branch_maps):
        if BF16_WEIGHT_KEY not in block:
            raise KeyError(f"VDN block {i} has no {BF16_WEIGHT_KEY!r}")
        if i < skip or i >= count - skip:
            out.append(dict(block))
            continue
        w = block[BF16_WEIGHT_KEY]
        use_convrot = bool(convrot) and precision == "int8" and w.shape[1] % CONVROT_GROUP == 0
        used_convrot = used_convrot and use_convrot
        qm = quantize_weight(w, precision, device, convrot=use_convrot)
        copied = dict(block)
        copied.pop(BF16_WEIGHT_KEY)
        copied[QUANT_WEIGHT_KEY] = qm.data
        copied[QUANT_SCALE_KEY] = qm.scale.reshape(1, 1) if precision == "fp8" else qm.scale
        if use_convrot:
            copied[CONVROT_KEY] = torch.tensor(CONVROT_GROUP, dtype=torch.int32)
        out.append(copied)
    info = {"precision": precision, "skip_end_blocks": skip}
    if precision == "int8":
        info.update(convrot=bool(convrot) and used_convrot, convrot_groupsize=CONVROT_GROUP)
    return tuple(out), info


__all__ = ["CONVROT_GROUP", "CONVROT_KEY", "PROJECTION_PRECISIONS", "QuantizedMatrix", "convrot_matrix",
           "dequantize_projection_weight", "gemm",
           "prepare_projection_maps", "project", "quantize_rows_int8", "quantize_rows_int8_convrot",
           "quantize_tensor_fp8", "quantize_weight"]
