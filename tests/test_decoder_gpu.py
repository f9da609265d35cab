"""The decoder-layer op mix (config 5's composition) checked stage by stage against the
oracle: each stage is fed this library's output of the previous stage, so integer stages are
compared bit for bit and floating-point stages within their own tolerances."""

import numpy as np
import pytest
import torch

import llm_kernels
import oracle

pytestmark = pytest.mark.gpu


def test_decoder_layer_stagewise_parity():
    g = torch.Generator().manual_seed(4)
    layer = llm_kernels.DecoderLayerOps(d_model=512, n_heads=4, d_ff=1376).cuda()
    layer.init_weights(g)
    B, T = 2, 384
    x = torch.randn(B, T, 512, generator=g).to(torch.bfloat16).cuda()
    u, mid = layer(x, return_intermediates=True)
    assert u.shape == (B, T, 1376) and u.dtype == torch.float16
    # 1) fused RMSNorm + QKV projection: relative error <= 1e-2
    ref_qkv = oracle.rmsnorm_linear_ref(x.reshape(B * T, 512), layer.qkv.w_norm, layer.qkv.w_lin)
    qkv = mid["qkv"].reshape(B * T, 3 * 512).float().cpu()
    assert ((qkv - ref_qkv).abs().max() / ref_qkv.abs().max()).item() <= 1e-2
    # 2) causal attention on the (strided) q, k, v views: max-abs <= 1e-2 * max(1, |O|)
    q, k, v = (mid["qkv"][:, :, i].transpose(1, 2) for i in range(3))
    ref_attn = oracle.attention_fp32(q, k, v, causal=True)
    attn = mid["attn"].transpose(1, 2).float().cpu()
    assert ((attn - ref_attn).abs() / ref_attn.abs().clamp(min=1.0)).max().item() <= 1e-2
    # 3) O projection: quantise + int8 GEMM + dequant, bit-exact
    aq, sa = oracle.quantize_symmetric(mid["attn"].reshape(B * T, 512).cpu())
    ref_y = oracle.int8_gemm_dequant(aq, layer.o_proj.w_q.cpu().numpy(), sa, layer.o_proj.scale_w.cpu().numpy(), "nk")
    np.testing.assert_array_equal(mid["y"].cpu().numpy().view(np.uint16), ref_y.view(np.uint16))
    # 4) the O projection's own re-quantisation of y (fused into its epilogue): codes and
    #    scales bit-identical to quantize_symmetric(y)
    yq, sy = oracle.quantize_symmetric(mid["y"].cpu())
    np.testing.assert_array_equal(mid["y_q"].cpu().numpy(), yq)
    np.testing.assert_array_equal(mid["y_s"].cpu().numpy().view(np.uint32), sy.view(np.uint32))
    # 5) MLP up projection, bit-exact
    ref_u = oracle.int8_gemm_dequant(yq, layer.up.w_q.cpu().numpy(), sy, layer.up.scale_w.cpu().numpy(), "nk")
    np.testing.assert_array_equal(u.reshape(B * T, 1376).cpu().numpy().view(np.uint16), ref_u.view(np.uint16))


def test_flash_attn_out_argument_layouts():
    g = torch.Generator().manual_seed(8)
    q, k, v = (torch.randn(2, 3, 200, 128, generator=g).to(torch.bfloat16).cuda() for _ in range(3))
    ref = llm_kernels.flash_attn_forward(q, k, v, causal=True)
    buf = torch.empty(2, 200, 3, 128, dtype=torch.bfloat16, device="cuda")
    out = llm_kernels.flash_attn_forward(q, k, v, causal=True, out=buf.transpose(1, 2))
    assert out.data_ptr() == buf.data_ptr()
    assert torch.equal(buf.transpose(1, 2), ref)
    odd = torch.empty(2, 3, 200, 130, dtype=torch.bfloat16, device="cuda")[..., :128]  # unaligned rows
    llm_kernels.flash_attn_forward(q, k, v, causal=True, out=odd)
    assert torch.equal(odd, ref)
