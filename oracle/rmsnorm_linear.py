"""RMSNorm + Linear in fp32 on the CPU (test infrastructure).

Restates the reference's fallback kernels/fused_rmsnorm_linear/fused_ops.py:27-37
(``_rmsnorm_linear_ref``), the path its config-1 benchmark runs on a CPU:
    x_f = x.float(); rms = x_f.pow(2).mean(-1, keepdim=True).add(eps).rsqrt()
    x_norm = (x_f * rms * w_norm.float()).to(x.dtype); y = F.linear(x_norm, w_lin)
Here every step stays in fp32 (``out_dtype`` selects a final rounding), which is the
fp32 PyTorch RMSNorm+Linear path that the relative-error tolerance of 1e-2 is stated against.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F


@torch.no_grad()
def rmsnorm_linear_ref(x, w_norm, w_lin, eps: float = 1e-6, round_to_input_dtype: bool = False) -> torch.Tensor:
    xf = x.detach().to("cpu", torch.float32)
    rms = xf.pow(2).mean(-1, keepdim=True).add(eps).rsqrt()
    xn = xf * rms * w_norm.detach().to("cpu", torch.float32)
    if round_to_input_dtype:
        xn = xn.to(x.dtype).float()  # the reference's .to(x.dtype) (fused_ops.py:36)
    return F.linear(xn, w_lin.detach().to("cpu", torch.float32))
