"""Generate golden vectors by running the reference's own torch path on CPU.

Run where the reference (hyukudan/ComfyUI-Kirei-VDN-H3 v0.3.3) is mounted:

    python tests/golden/make_golden.py --reference <path-to-reference-checkout>

It imports the reference package ``vdn_h3`` read-only, feeds it the seeded inputs that
``oracle/vdn_oracle.py`` also builds (so only outputs need storing), and writes
``tests/golden/config0.npz``.  The fixture is committed; nothing on the GPU side reads
the reference at run time.

Reference entry points exercised (file:line inside the reference project):
  * window.window_softmax_grouped            vdn_h3/window.py:277-313
  * branch.frame_statistics                  vdn_h3/branch.py:246-282
  * branch.VdnDelta.factor_apply             vdn_h3/branch.py:148-160
  * branch.SanaDelta.factor_apply            vdn_h3/branch.py:163-177 (delta_rule="sana_scaled")
  * branch.run_scans_reference               vdn_h3/branch.py:297-312
  * branch.gather_linear_state               vdn_h3/branch.py:399-435
  * branch.conv_features                     vdn_h3/branch.py:443-480
  * runtime.OptimizedLinearBranch.projected_delta  vdn_h3/runtime.py:545-607
  * hybrid.make_vdn_forward (profile=reference)    vdn_h3/hybrid.py:409-579
"""

from __future__ import annotations

import argparse
import hashlib
import os
import sys

import numpy as np
import torch
import torch.nn as nn
import torch.nn.functional as F

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)

from oracle import vdn_oracle as vo  # noqa: E402


class _RMS(nn.Module):
    def __init__(self, weight):
        super().__init__()
        self.weight = nn.Parameter(weight.clone())
        self.eps = 1e-6

    def forward(self, x):
        return F.rms_norm(x, (x.shape[-1],), self.weight, self.eps)


class _Attn(nn.Module):
    """Minimal stand-in exposing what make_vdn_forward needs (hybrid.py:591)."""

    def __init__(self, bw: vo.BlockWeights, heads, dim):
        super().__init__()
        hidden = bw.qkv.shape[1]
        self.heads, self.head_dim = heads, dim
        self.qkv_proj = nn.Linear(hidden, 3 * heads * dim, bias=False)
        self.qkv_proj.weight.data.copy_(bw.qkv)
        self.out_proj = nn.Linear(heads * dim, hidden, bias=False)
        self.out_proj.weight.data.copy_(bw.out)
        self.q_norm = _RMS(bw.q_norm)
        self.k_norm = _RMS(bw.k_norm)

    def forward(self, x, rope_freqs=None, transformer_options=None):  # never used
        raise AssertionError("layout must be published")


def tensor_digest(*tensors) -> str:
    h = hashlib.sha256()
    for t in tensors:
        h.update(np.ascontiguousarray(t.detach().cpu().float().numpy()).tobytes())
    return h.hexdigest()[:16]


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    ap.add_argument("--out", default=os.path.join(HERE, "config0.npz"))
    args = ap.parse_args()
    sys.path.insert(0, os.path.abspath(args.reference))
    from vdn_h3 import branch, hybrid, layout, runtime, window  # noqa: E402

    torch.set_num_threads(max(1, os.cpu_count() or 1))
    c = vo.CONFIG0
    heads, dim, hidden = c["heads"], c["dim"], c["hidden"]
    lay = vo.config_layout(c)
    out = {}

    # ---- kernel level: window softmax, all anchor modes --------------------------------
    ki = vo.make_kernel_inputs(0, lay, heads, dim)
    out["input_digest"] = np.array(tensor_digest(ki["q"], ki["k"], ki["v"], ki["beta"], ki["alpha"]))
    for mode in window.ANCHOR_FRAME_MODES:
        got = window.window_softmax_grouped(
            ki["q"], ki["k"], ki["v"], lay.video_start, lay.video_end, lay.num_frames,
            lay.tokens_per_frame, list(lay.bounds), dim ** -0.5, anchor_frames=mode,
        )
        keep = got if mode == "both" else got[::4]  # every 4th row pins the other modes
        out[f"window_{mode}"] = keep.numpy().astype(np.float32)
    # A second geometry: chunk 0 (sliding radius 2) with globals at both ends.
    lay2 = vo.Layout(seq_len=24 + 9 * 16 + 8, video_start=24, video_end=24 + 9 * 16,
                     num_frames=9, tokens_per_frame=16, frame_size=(4, 4), text_start=0,
                     text_len=24, bounds=tuple(vo.window_bounds(9, 2, 0)), anchor_frames="columns")
    ki2 = vo.make_kernel_inputs(5, lay2, 2, dim)
    got = window.window_softmax_grouped(
        ki2["q"], ki2["k"], ki2["v"], lay2.video_start, lay2.video_end, lay2.num_frames,
        lay2.tokens_per_frame, list(lay2.bounds), dim ** -0.5, anchor_frames="columns",
    )
    out["window_sliding_columns"] = got.numpy().astype(np.float32)

    # ---- kernel level: statistics, factor, scans, gather (branch frames = F-2) ----------
    fb = lay.num_frames - 2
    tpf = lay.tokens_per_frame
    inner = slice(lay.video_start + tpf, lay.video_end - tpf)
    kf = ki["k"][inner].reshape(fb, tpf, heads, dim).permute(0, 2, 1, 3).contiguous()
    vf = ki["v"][inner].reshape(fb, tpf, heads, dim).permute(0, 2, 1, 3).contiguous()
    beta = ki["beta"][1:-1].contiguous()
    alpha = ki["alpha"][1:-1].contiguous()
    a, b = branch.frame_statistics(kf, vf, beta)
    backend = branch.VdnDelta()
    text = torch.randn(heads, dim, dim, generator=torch.Generator().manual_seed(11)) * 0.1
    prefix, suffix = branch.run_scans_reference(backend, alpha, a, b, text_state=text)
    bounds_b = [(lo - 1, hi - 1) for lo, hi in lay.bounds[1:-1]]
    state = branch.gather_linear_state(prefix, suffix, alpha, bounds_b, text_state=text)
    state_nt = branch.gather_linear_state(prefix, suffix, alpha, bounds_b, text_state=None)
    trans, inj = backend.factor_apply(alpha, a, b)
    out["stats_A_f03_h1"] = a[:4, 1].numpy().astype(np.float32)
    out["stats_B_f03_h1"] = b[:4, 1].numpy().astype(np.float32)
    out["inverse_T_f0"] = trans[0].numpy().astype(np.float32)
    out["inj_f0"] = inj[0].numpy().astype(np.float32)
    out["prefix_last"] = prefix[-1].numpy().astype(np.float32)
    out["suffix_first"] = suffix[0].numpy().astype(np.float32)
    out["state_h0"] = state[::2, 0].numpy().astype(np.float32)
    out["state_notext_h1"] = state_nt[1::3, 1].numpy().astype(np.float32)
    # the alternative delta rule on the same statistics
    sana = branch.SanaDelta(tpf)
    s_trans, s_inj = sana.factor_apply(alpha, a, b)
    s_prefix, s_suffix = branch.run_scans_reference(sana, alpha, a, b, text_state=text)
    out["sana_T_f0"] = s_trans[0].numpy().astype(np.float32)
    out["sana_inj_f0"] = s_inj[0].numpy().astype(np.float32)
    out["sana_prefix_last"] = s_prefix[-1].numpy().astype(np.float32)
    out["sana_suffix_first"] = s_suffix[0].numpy().astype(np.float32)

    # ---- conv features ----------------------------------------------------------------
    bw = vo.make_block(0, hidden, heads, dim)
    w = bw.branch
    conv_k = branch.conv_features(
        ki["k"][lay.video_start:lay.video_end], w["short_conv.k_sp.weight"],
        w["short_conv.k_tm.weight"], lay.num_frames, lay.frame_size, True, fhsd=True,
    )
    out["conv_k_f3"] = conv_k[3].numpy().astype(np.float32)

    # ---- block level: make_vdn_forward at profile=reference ----------------------------
    x = vo.make_x(0, lay.seq_len, hidden)
    attn = _Attn(bw, heads, dim)
    br = runtime.OptimizedLinearBranch(
        {k: v.clone() for k, v in w.items()}, heads, dim, delta_rule="vdn_solve", bridge="alpha",
        a_fp32=True, short_conv=("k", "v"), enable_text_state=True,
        kernel_backend="eager", compile_policy="off",
    )
    cfg = {"enable_softmax_gate": True, "enable_text_state": True, "linear_enabled": True}
    state_obj = hybrid.VDNState(
        "golden", cfg, [br], heads, dim, weight_mode="resident", attention_backend="grouped",
        inference=False, kernel_backend="eager", compile_policy="off",
    )
    ref_layout = layout.VDNLayout(
        seq_len=lay.seq_len, video_start=lay.video_start, video_end=lay.video_end,
        num_frames=lay.num_frames, tokens_per_frame=lay.tokens_per_frame,
        frame_size=lay.frame_size, text_start=lay.text_start, text_len=lay.text_len,
        bounds=lay.bounds, full_cover=lay.full_cover, anchor_frames=lay.anchor_frames,
    )
    fwd = hybrid.make_vdn_forward(attn, state_obj, 0)
    with torch.no_grad(), layout.publish_layout(ref_layout):
        y = fwd(x)
    out["block_out"] = y.numpy().astype(np.float32)
    # The branch delta alone, through the node's projected_delta entry.
    with torch.no_grad():
        qkv = attn.qkv_proj(x)
        inner_w = heads * dim
        q_raw = qkv[:, :inner_w].reshape(-1, heads, dim)
        k_raw = qkv[:, inner_w:2 * inner_w].reshape(-1, heads, dim)
        v_raw = qkv[:, 2 * inner_w:].reshape(-1, heads, dim)
        va, vb, ta, tb = lay.video_start, lay.video_end, lay.text_start, lay.text_start + lay.text_len
        delta = br.projected_delta(
            w, x[va:vb], q_raw[va:vb], k_raw[va:vb], v_raw[va:vb], lay.num_frames,
            lay.tokens_per_frame, list(lay.bounds), frame_size=lay.frame_size,
            text_x=x[ta:tb], text_k_raw=k_raw[ta:tb], text_v_raw=v_raw[ta:tb],
            skip_ends=True, inference=False,
        )
    out["branch_delta"] = delta.numpy().astype(np.float32)
    # the whole block with the sana_scaled rule
    br_s = runtime.OptimizedLinearBranch(
        {k: v.clone() for k, v in w.items()}, heads, dim, delta_rule="sana_scaled", bridge="alpha",
        a_fp32=True, short_conv=("k", "v"), enable_text_state=True,
        kernel_backend="eager", compile_policy="off",
    )
    state_s = hybrid.VDNState(
        "golden_sana", cfg, [br_s], heads, dim, weight_mode="resident", attention_backend="grouped",
        inference=False, kernel_backend="eager", compile_policy="off",
    )
    fwd_s = hybrid.make_vdn_forward(attn, state_s, 0)
    with torch.no_grad(), layout.publish_layout(ref_layout):
        y_s = fwd_s(x)
    out["sana_block_out"] = y_s.numpy().astype(np.float32)
    out["weights_digest"] = np.array(tensor_digest(x, bw.qkv, bw.out, *[w[k] for k in sorted(w)]))
    np.savez_compressed(args.out, **out)
    total = sum(v.nbytes for v in out.values())
    print(f"wrote {args.out}: {len(out)} arrays, {total / 1e6:.2f} MB raw")


if __name__ == "__main__":
    main()
