"""Generates the golden vectors in this directory by running the REFERENCE's own code.

Run where a checkout of the reference is available (read-only is enough), naming it with
the first argument or the LK_REFERENCE_DIR environment variable:

    python tests/golden/make_golden.py /path/to/reference [op ...]
    LK_REFERENCE_DIR=/path/to/reference python tests/golden/make_golden.py [op ...]

(op: quantize, int8_gemm, flash_attn, flash_attn_bwd, rmsnorm_linear, gqa; default all)

What it runs (all on the CPU):
  * ``quantize_symmetric``     kernels/int8_gemm/int8_gemm.py:146-161 (pure torch)
  * ``int8_gemm_dequant_kernel`` kernels/int8_gemm/int8_gemm.py:33-90 (Triton, under
    TRITON_INTERPRET=1 so it executes on CPU tensors)
  * ``flash_attn_fwd_kernel`` / ``flash_attn_fwd_causal_kernel``
    kernels/flash_attn/flash_attn_fwd.py:6-128 (Triton, interpreted)
  * ``_rmsnorm_linear_ref``    kernels/fused_rmsnorm_linear/fused_ops.py:27-37 (pure torch)
  * ``GroupedQueryAttention`` / ``MultiQueryAttention``
    experiments/attention_ablation.py:70-141 (torch modules; dropout 0, eval mode, the
    output projection set to the identity so the module returns the attention output)
Outputs: one ``.npz`` per op.  The fixtures are small (tens of KB) and committed; the GPU
tests and the oracle tests read only the ``.npz`` files, never the reference.
"""

from __future__ import annotations

import os
import sys

os.environ["TRITON_INTERPRET"] = "1"  # must precede the triton import

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def _t2np(t: torch.Tensor) -> np.ndarray:
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy()  # bf16 stored as raw bits
    return t.numpy()


def make_quantize(ref):
    from kernels.int8_gemm.int8_gemm import quantize_symmetric

    out = {}
    g = torch.Generator().manual_seed(11)
    cases = {
        "f16": torch.randn(37, 200, generator=g).to(torch.float16),
        "f32": (torch.randn(16, 64, generator=g) * 3.0).float(),
        "bf16": torch.randn(9, 136, generator=g).to(torch.bfloat16),
        "f16_wide": torch.randn(4, 4096, generator=g).to(torch.float16),
    }
    sp = torch.randn(6, 24, generator=g).float()
    sp[0] = 0.0  # all-zero row: scale 0, codes 0
    sp[1, 3] = float("inf")  # inf row: scale inf, codes 0
    sp[2, 5] = float("nan")  # nan row: scale nan, codes 0
    sp[3] = torch.tensor([1e-45] * 12 + [-1e-45] * 6 + [0.0] * 6)  # subnormal: scale rounds to 0
    sp[4] = torch.tensor([127.0, 0.5, 1.5, 2.5, -0.5, -2.5, 63.5] + [0.0] * 17)  # ties to even
    sp[5] = -sp[5].abs()
    cases["f32_special"] = sp
    for name, x in cases.items():
        q, s = quantize_symmetric(x)
        out[f"{name}_x"] = _t2np(x)
        out[f"{name}_q"] = q.numpy()
        out[f"{name}_scale"] = s.numpy()
    np.savez_compressed(os.path.join(HERE, "quantize.npz"), **out)


def make_int8_gemm(ref):
    from kernels.int8_gemm.int8_gemm import int8_gemm_dequant_kernel, quantize_symmetric

    out = {}
    g = torch.Generator().manual_seed(12)
    for tag, (M, N, K) in {"sq": (128, 128, 128), "rag": (100, 72, 96)}.items():
        A_fp = torch.randn(M, K, generator=g).to(torch.float16)
        B_fp = torch.randn(K, N, generator=g).to(torch.float16)
        A_q, sa = quantize_symmetric(A_fp)
        B_q, sb = quantize_symmetric(B_fp.T)
        B_q = B_q.T.contiguous()  # [K, N] as in the reference README / tests
        C = torch.empty((M, N), dtype=torch.float16)
        grid = ((M + 63) // 64, (N + 63) // 64)
        int8_gemm_dequant_kernel[grid](A_q, B_q, C, sa, sb, M, N, K, BLOCK_M=64, BLOCK_N=64, BLOCK_K=32)
        out[f"{tag}_A"] = A_q.numpy()
        out[f"{tag}_B_kn"] = B_q.numpy()
        out[f"{tag}_sa"] = sa.numpy()
        out[f"{tag}_sb"] = sb.numpy()
        out[f"{tag}_C"] = C.numpy()
    np.savez_compressed(os.path.join(HERE, "int8_gemm.npz"), **out)


def make_flash_attn(ref):
    from kernels.flash_attn.flash_attn_fwd import flash_attn_fwd_causal_kernel, flash_attn_fwd_kernel

    out = {}
    g = torch.Generator().manual_seed(13)
    B, H, M, D = 1, 2, 128, 64
    q = torch.randn(B, H, M, D, generator=g).to(torch.float16)
    k = torch.randn(B, H, M, D, generator=g).to(torch.float16)
    v = torch.randn(B, H, M, D, generator=g).to(torch.float16)
    out["q"], out["k"], out["v"] = q.numpy(), k.numpy(), v.numpy()
    for causal, kern in ((0, flash_attn_fwd_kernel), (1, flash_attn_fwd_causal_kernel)):
        o = torch.empty_like(q)
        kern[(M // 64, B * H)](q, k, v, o, *q.stride(), *k.stride(), *v.stride(), *o.stride(), B, H, M, M, D,
                               BLOCK_M=64, BLOCK_N=64)
        out[f"out_causal{causal}"] = o.numpy()
    np.savez_compressed(os.path.join(HERE, "flash_attn.npz"), **out)


def make_flash_attn_bwd(ref):
    """The reference's training path, kernels/flash_attn/flash_attn_bwd.py: FlashAttnFunction
    (:245-334) with its forward-with-LSE kernel (:39-119) and backward kernel (:127-237), both
    interpreted.  As written the two kernels name the head dimension `D` without defining it
    (:85, :190); the module-level name is bound to the inputs' head dimension here, which is
    the only way they run.  Stored: the LSE of both modes and the non-causal dQ / dK / dV.  The
    causal backward is not stored: its key-tile loop visits query tiles [0, (pid_n + 1) BLOCK_N)
    (:200-202) -- the queries BEFORE the keys, which under the causal mask n <= m never see
    them -- so its causal gradients are not the gradients of its causal forward."""
    import kernels.flash_attn.flash_attn_bwd as bwd

    out = {}
    g = torch.Generator().manual_seed(16)
    B, H, M, D = 1, 2, 128, 64
    bwd.D = D
    q, k, v, do = (torch.randn(B, H, M, D, generator=g).to(torch.float16) for _ in range(4))
    out["q"], out["k"], out["v"], out["do"] = q.numpy(), k.numpy(), v.numpy(), do.numpy()
    for causal in (0, 1):
        qq, kk, vv = (t.clone().requires_grad_(True) for t in (q, k, v))
        o = bwd.FlashAttnFunction.apply(qq, kk, vv, bool(causal), 64, 64)
        out[f"out_causal{causal}"] = o.detach().numpy()
        out[f"lse_causal{causal}"] = o.grad_fn.saved_tensors[4].numpy()
        if not causal:
            o.backward(do)
            out["dq_causal0"], out["dk_causal0"], out["dv_causal0"] = (
                t.grad.numpy() for t in (qq, kk, vv))
    np.savez_compressed(os.path.join(HERE, "flash_attn_bwd.npz"), **out)


def make_rmsnorm_linear(ref):
    from kernels.fused_rmsnorm_linear.fused_ops import _rmsnorm_linear_ref

    out = {}
    g = torch.Generator().manual_seed(14)
    # The config-1 recipe at a small size: x ~N(0,1), w_norm = 1 + 0.1 N(0,1), w_lin ~N(0,1)/sqrt(d_in)
    for tag, dt in (("f32", torch.float32), ("f16", torch.float16)):
        x = torch.randn(16, 128, generator=g).to(dt)
        w_norm = (1 + 0.1 * torch.randn(128, generator=g)).to(dt)
        w_lin = (torch.randn(96, 128, generator=g) / 128 ** 0.5).to(dt)
        y = _rmsnorm_linear_ref(x, w_norm, w_lin, 1e-6)
        out[f"{tag}_x"], out[f"{tag}_w_norm"], out[f"{tag}_w_lin"] = x.numpy(), w_norm.numpy(), w_lin.numpy()
        out[f"{tag}_y"] = y.numpy()
    np.savez_compressed(os.path.join(HERE, "rmsnorm_linear.npz"), **out)


def make_gqa(ref):
    from experiments.attention_ablation import GroupedQueryAttention, MultiQueryAttention

    out = {}
    g = torch.Generator().manual_seed(15)
    B, T, C, H = 1, 64, 128, 8  # head dim 16
    D = C // H
    for tag, mod in (("gqa", GroupedQueryAttention(C, H, n_kv_heads=2, dropout=0.0)),
                     ("mqa", MultiQueryAttention(C, H, dropout=0.0))):
        mod.eval()
        with torch.no_grad():
            for p in mod.parameters():
                p.copy_(torch.randn(p.shape, generator=g) / C ** 0.5)
            mod.out_proj.weight.copy_(torch.eye(C))
            x = torch.randn(B, T, C, generator=g)
            kh = mod.k_proj.out_features // D
            out[f"{tag}_q"] = mod.q_proj(x).view(B, T, H, D).transpose(1, 2).contiguous().numpy()
            out[f"{tag}_k"] = mod.k_proj(x).view(B, T, kh, D).transpose(1, 2).contiguous().numpy()
            out[f"{tag}_v"] = mod.v_proj(x).view(B, T, kh, D).transpose(1, 2).contiguous().numpy()
            for causal in (0, 1):
                mask = torch.tril(torch.ones(T, T)) if causal else None
                y = mod(x, mask)  # [B, T, C] = attention output with heads concatenated
                out[f"{tag}_out_causal{causal}"] = y.view(B, T, H, D).transpose(1, 2).contiguous().numpy()
    np.savez_compressed(os.path.join(HERE, "gqa.npz"), **out)


MAKERS = {"quantize": make_quantize, "int8_gemm": make_int8_gemm, "flash_attn": make_flash_attn,
          "flash_attn_bwd": make_flash_attn_bwd, "rmsnorm_linear": make_rmsnorm_linear, "gqa": make_gqa}


def main():
    args = sys.argv[1:]
    if args and os.path.isdir(args[0]):
        ref, ops = args[0], args[1:]
    else:
        ref, ops = os.environ.get("LK_REFERENCE_DIR"), args
    if not ref or not os.path.isdir(ref):
        sys.exit("make_golden.py: name the reference checkout (first argument or LK_REFERENCE_DIR)")
    sys.path.insert(0, ref)
    for name in ops or list(MAKERS):
        MAKERS[name](ref)
    print("golden vectors written to", HERE)


if __name__ == "__main__":
    main()
