"""B200-native (sm_100a) VDN-H3 hybrid attention hot path.

Drop-in for the hot path of hyukudan/ComfyUI-Kirei-VDN-H3: the exact local window
softmax, the Video Delta Attention branch, the gated sum and the bf16 / fp8 / int8
projections, behind the reference's operator API (``make_vdn_forward`` ->
``attn.forward(x, rope_freqs, transformer_options)``).  Compute runs in hand-written
CUDA for sm_100a loaded from the in-tree C-ABI library ``libvdn_b200.so``; there is no
CPU or library fallback.
"""

from . import _lib, dit, projection, shard
from ._lib import DeviceStatus
from .branch import B200LinearBranch, cholesky_runtime_scope
from .host_io import HostStreamer
from .dit import B200DiTBlock, make_fast_block_forward
from .hybrid import B200State, FusedBlock, GatedResidual, RopeTable, make_vdn_forward, rope_table, run_forward_checked
from .layout import (ANCHOR_FRAME_MODES, VDNLayout, current_layout, from_comfy_packed_layout, full_coverage,
                     layout_from_payload, make_layout, publish_layout, window_bounds, with_window)
from .projection import (gemm, gemm_grouped_k, prepare_projection_maps, project, quantize_rows_int8,
                         quantize_rows_int8_convrot, quantize_tensor_fp8)
from .shard import HeadShard
from .window import WindowPlanCache, build_window_plan, window_softmax_b200

__all__ = [
    "ANCHOR_FRAME_MODES", "B200DiTBlock", "B200LinearBranch", "B200State", "GatedResidual",
    "make_fast_block_forward", "from_comfy_packed_layout", "layout_from_payload", "DeviceStatus", "FusedBlock", "HeadShard", "HostStreamer", "VDNLayout",
    "RopeTable", "WindowPlanCache", "gemm_grouped_k", "rope_table",
    "build_window_plan", "cholesky_runtime_scope", "current_layout", "full_coverage", "gemm", "make_layout",
    "make_vdn_forward", "prepare_projection_maps", "project", "publish_layout", "quantize_rows_int8",
    "quantize_rows_int8_convrot",
    "quantize_tensor_fp8", "run_forward_checked", "window_bounds", "window_softmax_b200", "with_window", "_lib",
]
