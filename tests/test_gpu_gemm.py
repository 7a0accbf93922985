"""The tcgen05 GEMM behind the R_q / R_k projection (fna2_gemm): every operand
layout against a torch fp32 product of the same bf16 operands, ragged M / N / K,
the split-K fp32 reduction, argument checks, and the projection's forward and
both gradients against the reference's two-Linear composition
(attention_fna2.py:320-335)."""
import math

import pytest
import torch
import torch.nn as nn

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True, scope="module")
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from fna2_b200 import _lib
    _lib.load()
    yield
    assert _lib.load().fna2_device_status(1) == 0, "a kernel's bounded wait timed out"


def _operand(rows, k, mn, gen):
    """A logical [rows, k] bf16 operand stored K-major ([rows][k]) or MN-major
    ([k][rows]), with the leading dimension padded to a multiple of 8 elements
    (16 bytes, as TMA needs)."""
    t = torch.randn(rows, k, device="cuda", generator=gen).bfloat16()
    src = t.t() if mn else t
    ld = -(-src.shape[1] // 8) * 8
    st = torch.zeros(src.shape[0], ld, device="cuda", dtype=torch.bfloat16)
    st[:, :src.shape[1]] = src
    return t, st


@pytest.mark.parametrize("a_mn,b_mn", [(False, False), (False, True), (True, True), (True, False)])
@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (300, 96, 200), (1, 32, 1), (1000, 544, 1000)])
def test_gemm_layouts_vs_torch(a_mn, b_mn, M, N, K):
    from fna2_b200.rel_proj import _gemm
    g = torch.Generator(device="cuda").manual_seed(M + N + K)
    a, a_st = _operand(M, K, a_mn, g)
    b, b_st = _operand(N, K, b_mn, g)
    ref = a.float() @ b.float().t()
    c = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    _gemm(a_st, a_mn, b_st, b_mn, M, N, K, c)
    torch.testing.assert_close(c.float(), ref, rtol=1e-2, atol=1e-2 * math.sqrt(K))
    c32 = torch.zeros(M, N, device="cuda", dtype=torch.float32)
    _gemm(a_st, a_mn, b_st, b_mn, M, N, K, c32, split=3)
    torch.testing.assert_close(c32, ref, rtol=1e-4, atol=1e-4 * math.sqrt(K))


def test_gemm_fp32_accumulates_into_c():
    from fna2_b200.rel_proj import _gemm
    g = torch.Generator(device="cuda").manual_seed(7)
    a, _ = _operand(256, 512, False, g)
    b, _ = _operand(64, 512, False, g)
    c = torch.full((256, 64), 1.5, device="cuda")
    _gemm(a, False, b, False, 256, 64, 512, c, split=5)
    torch.testing.assert_close(c, a.float() @ b.float().t() + 1.5, rtol=1e-4, atol=1e-3)


def test_gemm_rejects_bad_arguments():
    from fna2_b200 import _lib
    from fna2_b200.rel_proj import _gemm
    a = torch.zeros(64, 64, device="cuda", dtype=torch.bfloat16)
    c = torch.zeros(64, 48, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="multiple of 32"):
        _gemm(a, False, a, False, 64, 48, 64, c)          # n % 32 != 0
    c2 = torch.zeros(64, 64, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="split_k"):
        _gemm(a, False, a, False, 64, 64, 64, c2, split=2)  # bf16 output cannot be split
    assert _lib.load().fna2_device_status(1) == 0


@pytest.mark.parametrize("shape", [(2, 192, 256), (3001, 512)])
def test_projection_on_gemm_matches_reference(shape):
    from fna2_b200.rel_proj import FusedRelProjection
    torch.manual_seed(3)
    E, H_G, R = shape[-1], 4, 16
    lq = nn.Linear(E, H_G * R, bias=False).cuda().bfloat16()
    lk = nn.Linear(E, H_G * R, bias=False).cuda().bfloat16()
    x = torch.randn(*shape, device="cuda").bfloat16().requires_grad_(True)
    m = FusedRelProjection.from_linears(lq, lk, H_G, R)
    rq, rk = m(x)
    xr = x.detach().clone().requires_grad_(True)
    lead = shape[:-1]
    if len(shape) == 3:
        rq_ref = lq(xr).view(*lead, H_G, R).permute(0, 2, 1, 3)
        rk_ref = lk(xr).view(*lead, H_G, R).permute(0, 2, 1, 3)
    else:
        rq_ref, rk_ref = lq(xr).view(*lead, H_G, R), lk(xr).view(*lead, H_G, R)
    torch.testing.assert_close(rq.float(), rq_ref.float(), rtol=1e-2, atol=1e-2)
    torch.testing.assert_close(rk.float(), rk_ref.float(), rtol=1e-2, atol=1e-2)
    g1, g2 = torch.randn_like(rq_ref), torch.randn_like(rk_ref)
    ((rq.float() * g1.float()).sum() + (rk.float() * g2.float()).sum()).backward()
    ((rq_ref.float() * g1.float()).sum() + (rk_ref.float() * g2.float()).sum()).backward()
    torch.testing.assert_close(x.grad.float(), xr.grad.float(), rtol=2e-2, atol=2e-2)
    gw_ref = torch.cat([lq.weight.grad, lk.weight.grad]).float()
    torch.testing.assert_close(m.weight.grad.float(), gw_ref, rtol=2e-2, atol=2e-2 * gw_ref.abs().max().item())
