"""Batched FP16 tensor-core GEMMs of attention (scores = Q K^T / 8 and O = P V, BERT-base
heads of 64) against a float32 torch reference of the same f16 inputs.  Tolerance: f32
accumulation against torch's f32 matmul, |Δ| <= 1e-4 (f32 output); f16 output adds its own
rounding, |Δ| <= 2e-3 + 2e-3 |y|."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _ref(a, b, alpha):
    import torch
    return torch.matmul(a.float().cpu(), b.float().cpu().transpose(-1, -2)) * alpha


@pytest.mark.parametrize("batch,heads,m,n,k", [(2, 3, 384, 384, 64), (1, 2, 200, 72, 64), (3, 1, 130, 257, 136)])
def test_gemm_f16_contiguous(cuda, batch, heads, m, n, k):
    import torch
    from lightship_b200 import ops
    g = torch.Generator().manual_seed(batch * 100 + m + n)
    a = torch.randn(batch, heads, m, k, generator=g).half().to(cuda)
    b = torch.randn(batch, heads, n, k, generator=g).half().to(cuda)
    for dt, tol in ((torch.float32, (1e-4, 1e-5)), (torch.float16, (2e-3, 2e-3))):
        out = torch.empty(batch, heads, m, n, dtype=dt, device=cuda)
        ops.gemm_f16_batched(a, b, out, batch, heads, m, n, k, alpha=0.125)
        torch.testing.assert_close(out.float().cpu(), _ref(a, b, 0.125), atol=tol[0], rtol=tol[1])


def test_attention_from_fused_qkv(cuda):
    """Q, K, V read in place from a fused [B, S, 3*H, 64] projection; scores [B, H, S, S];
    V transposed per head; O written straight into [B, S, H*64]."""
    import torch
    from lightship_b200 import ops
    B, S, H, D = 2, 384, 12, 64
    g = torch.Generator().manual_seed(5)
    qkv = (torch.randn(B, S, 3 * H, D, generator=g) * 0.5).half().to(cuda)
    q, k, v = qkv[:, :, :H], qkv[:, :, H:2 * H], qkv[:, :, 2 * H:]
    row, head, bat = 3 * H * D, D, S * 3 * H * D
    scores = torch.empty(B, H, S, S, dtype=torch.float16, device=cuda)
    ops.gemm_f16_batched(qkv, qkv, scores, B, H, S, S, D, alpha=0.125, a_strides=(row, head, bat),
                         b_strides=(row, head, bat), a_head0=0, b_head0=H)
    ref_s = torch.matmul(q.float().cpu().permute(0, 2, 1, 3), k.float().cpu().permute(0, 2, 3, 1)) * 0.125
    torch.testing.assert_close(scores.float().cpu(), ref_s, atol=2e-3, rtol=2e-3)
    p = torch.softmax(scores.float(), -1).half().contiguous()
    vt = torch.empty(B, H, D, S, dtype=torch.float16, device=cuda)
    ops.transpose_heads_f16(qkv, vt, B, H, S, D, (bat, head, row), head0=2 * H)
    torch.testing.assert_close(vt.cpu(), v.cpu().permute(0, 2, 3, 1))
    o = torch.empty(B, S, H * D, dtype=torch.float16, device=cuda)
    ops.gemm_f16_batched(p, vt, o, B, H, S, D, S, out_strides=(H * D, D, S * H * D))
    ref_o = torch.matmul(p.float().cpu(), v.float().cpu().permute(0, 2, 1, 3)).permute(0, 2, 1, 3).reshape(B, S, H * D)
    torch.testing.assert_close(o.float().cpu(), ref_o, atol=2e-3, rtol=2e-3)
