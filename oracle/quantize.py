"""Per-row symmetric absmax quantisation — numpy restatement (test infrastructure).

Follows kernels/int8_gemm/int8_gemm.py:157-161 of the reference:
    x_f32 = x.float()                                   (:157)
    scale = x_f32.abs().amax(dim=-1) / 127.0            (:158)  fp32 IEEE division
    x_q = (x_f32 / scale.unsqueeze(-1)).round()         (:159)  fp32 IEEE division, ties-to-even
    x_q = x_q.clamp(-128, 127).to(torch.int8)           (:160)
On the reference's CPU path a NaN quotient (0/0 for an all-zero row, inf/inf, NaN inputs)
casts to int8 code 0; that is restated explicitly here.
"""

from __future__ import annotations

import numpy as np


def _as_f32(x) -> np.ndarray:
    try:
        import torch

        if isinstance(x, torch.Tensor):
            return x.detach().to("cpu").float().numpy()
    except ImportError:  # pragma: no cover
        pass
    return np.asarray(x, dtype=np.float32)


def quantize_symmetric(x):
    """Returns (q int8 [..., K], scale fp32 [...]) as numpy arrays."""
    xf = _as_f32(x)
    with np.errstate(invalid="ignore", divide="ignore"):
        mag = np.abs(xf)
        # torch.amax propagates NaN; np.max does too.
        amax = mag.max(axis=-1)
        scale = (amax / np.float32(127.0)).astype(np.float32)
        t = (xf / scale[..., None]).astype(np.float32)
        nan = np.isnan(t)
        t = np.rint(t)  # round half to even, like torch.round
        t = np.clip(t, -128.0, 127.0)
        t[nan] = 0.0
    return t.astype(np.int8), scale
