"""CPU checks of the arithmetic the int8 quantiser kernels rely on (no GPU needed).

* The ConvRot kernel (``int8_rows_convrot_kernel`` in csrc/quant.cu) spreads a 256-channel
  group over a warp, 8 consecutive channels per lane, and rotates the four base-4 digits of
  the channel index partly in registers and partly by ``shfl_xor``.  ``_warp_rotation`` replays
  that lane scheme in numpy float32 (a shuffle is an index permutation of the lane axis) and
  must reproduce the oracle's ``convrot_rotate`` bit for bit.
* The int8 kernels round x / scale through ``rint_quotient``: the product with the correctly
  rounded reciprocal, and the IEEE division only where that product lies within 2^-12 of a
  half-integer.  ``test_reciprocal_fast_path_matches_the_ieee_quotient`` checks the rule on
  random and adversarial quotients in numpy float32 (IEEE single precision, like the GPU).
"""

from __future__ import annotations

import numpy as np
import torch

from oracle import vdn_oracle as vo

F32 = np.float32


def _warp_rotation(group: np.ndarray) -> np.ndarray:
    """One 256-wide group through the kernel's lane scheme: v[lane][e] = group[8 lane + e]."""
    v = group.reshape(32, 8).astype(F32).copy()
    lanes = np.arange(32)
    for b in (0, 4):  # d0: e & 3, in registers
        s = (v[:, b] + v[:, b + 1]) + (v[:, b + 2] + v[:, b + 3])
        for t in range(4):
            v[:, b + t] = s - F32(2) * v[:, b + t]
    for t in range(4):  # d1: e bit 2 in registers, lane bit 0 by shuffle
        p = v[:, t] + v[:, t + 4]
        s = p + p[lanes ^ 1]
        v[:, t] = s - F32(2) * v[:, t]
        v[:, t + 4] = s - F32(2) * v[:, t + 4]
    for e in range(8):  # d2: lane bits 1-2
        p = v[:, e] + v[lanes ^ 2, e]
        s = p + p[lanes ^ 4]
        v[:, e] = s - F32(2) * v[:, e]
    for e in range(8):  # d3: lane bits 3-4, then the 1/16 scale
        p = v[:, e] + v[lanes ^ 8, e]
        s = p + p[lanes ^ 16]
        v[:, e] = (s - F32(2) * v[:, e]) * F32(0.0625)
    return v.reshape(256)


def test_convrot_lane_scheme_reproduces_the_oracle_bit_for_bit():
    rng = np.random.default_rng(0)
    x = rng.standard_normal((6, 768)).astype(F32)
    x[:, 5] *= 50  # an outlier channel
    x = torch.from_numpy(x).to(torch.bfloat16).float().numpy()  # the kernel reads bf16 rows
    got = np.stack([np.concatenate([_warp_rotation(r[g * 256:(g + 1) * 256]) for g in range(3)]) for r in x])
    want = vo.convrot_rotate(torch.from_numpy(x))
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def _rint_quotient(x: np.ndarray, s: F32) -> tuple[np.ndarray, np.ndarray]:
    """The kernel's rule: (code, fast-path mask)."""
    r = F32(1) / s
    q = (x * r).astype(F32)
    c = np.rint(q)
    fast = np.abs((q - c).astype(F32)) <= F32(0.5) - F32(2.0 ** -12)
    return np.where(fast, c, np.rint((x / s).astype(F32))), fast


def test_reciprocal_fast_path_matches_the_ieee_quotient():
    rng = np.random.default_rng(1)
    fast_total = n_total = 0
    for _ in range(12):
        amax = F32(abs(rng.standard_normal()) * 10 ** rng.uniform(-4, 4))
        s = max(F32(amax / F32(127)), F32(1e-12))
        x = (rng.uniform(-1, 1, 200_000).astype(F32) * amax).astype(F32)
        k = rng.integers(-127, 127, 100_000)
        near = ((k + 0.5) * s * (1 + rng.uniform(-2.0 ** -20, 2.0 ** -20, k.size))).astype(F32)
        x = np.clip(np.concatenate([x, near, [amax, -amax, 0]]).astype(F32), -amax, amax)
        got, fast = _rint_quotient(x, s)
        want = np.rint((x / s).astype(F32))
        assert np.array_equal(got, want)
        assert np.abs(want).max() <= 127  # the clamp never binds for |x| <= amax
        fast_total += int(fast.sum())
        n_total += x.size
    assert fast_total > 0.6 * n_total  # a third of the samples sit next to half-integers on purpose
