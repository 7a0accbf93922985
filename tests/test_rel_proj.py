"""Fused R_q/R_k projection (fna2_b200/rel_proj.py) against the reference's
composition (attention_fna2.py:315-316, :332-333: Linear, view, permute,
cast, contiguous), values and gradients; GPU leg: bf16 on the device and the
attention op consuming the strided views."""
import pytest
import torch
import torch.nn as nn

from fna2_b200.rel_proj import FusedRelProjection, compute_rq_rk


def _reference(x, lq, lk, H_G, R, dtype):
    if x.dim() == 3:
        B, S, _ = x.shape
        rq = lq(x).view(B, S, H_G, R).permute(0, 2, 1, 3).to(dtype)
        rk = lk(x).view(B, S, H_G, R).permute(0, 2, 1, 3).to(dtype)
    else:
        T = x.shape[0]
        rq, rk = lq(x).view(T, H_G, R).to(dtype), lk(x).view(T, H_G, R).to(dtype)
    return rq.contiguous(), rk.contiguous()


@pytest.mark.parametrize("shape", [(2, 37, 64), (53, 64)])
def test_fused_projection_matches_reference_composition(shape):
    torch.manual_seed(0)
    E, H_G, R = shape[-1], 3, 16
    lq, lk = nn.Linear(E, H_G * R, bias=False), nn.Linear(E, H_G * R, bias=False)
    x = torch.randn(*shape, requires_grad=True)
    m = FusedRelProjection.from_linears(lq, lk, H_G, R)
    rq, rk = m(x, dtype=torch.float32)
    xr = x.detach().clone().requires_grad_(True)
    rq_ref, rk_ref = _reference(xr, lq, lk, H_G, R, torch.float32)
    torch.testing.assert_close(rq, rq_ref, rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(rk, rk_ref, rtol=1e-5, atol=1e-6)
    g1, g2 = torch.randn_like(rq_ref), torch.randn_like(rk_ref)
    ((rq * g1).sum() + (rk * g2).sum()).backward()
    ((rq_ref * g1).sum() + (rk_ref * g2).sum()).backward()
    torch.testing.assert_close(x.grad, xr.grad, rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(m.weight.grad, torch.cat([lq.weight.grad, lk.weight.grad]), rtol=1e-5, atol=1e-6)


def test_views_not_copies():
    x = torch.randn(2, 5, 32)
    w = torch.randn(2 * 2 * 16, 32)
    rq, rk = compute_rq_rk(x, w, 2, 16, torch.float32)
    assert rq.shape == (2, 2, 5, 16) and rk.stride() == (5 * 64, 16, 64, 1)
    assert rq.untyped_storage().data_ptr() == rk.untyped_storage().data_ptr()


def test_bad_weight_shape():
    with pytest.raises(ValueError):
        compute_rq_rk(torch.randn(4, 32), torch.randn(10, 32), 2, 16)


@pytest.mark.gpu
def test_gpu_bf16_views_feed_attention():
    from fna2_b200.flash_naylis_attn import flash_naylis_attn
    torch.manual_seed(1)
    B, S, H, D, R = 2, 192, 4, 64, 16
    E = H * D
    lq = nn.Linear(E, H * R, bias=False).cuda().bfloat16()
    lk = nn.Linear(E, H * R, bias=False).cuda().bfloat16()
    x = torch.randn(B, S, E, device="cuda").bfloat16()
    m = FusedRelProjection.from_linears(lq, lk, H, R)
    rq, rk = m(x)
    rq_ref, rk_ref = _reference(x, lq, lk, H, R, torch.bfloat16)
    torch.testing.assert_close(rq.float(), rq_ref.float(), rtol=1e-2, atol=1e-2)
    q, k, v = (torch.randn(B, H, S, D, device="cuda").bfloat16() for _ in range(3))
    gs = torch.ones(H, device="cuda")
    o_views = flash_naylis_attn(q, k, v, rq, rk, gs)
    o_copies = flash_naylis_attn(q, k, v, rq.contiguous(), rk.contiguous(), gs)
    assert torch.equal(o_views, o_copies)
