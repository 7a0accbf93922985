"""GPU parity of the fused varlen QK-RMSNorm + RoPE kernels (through the C ABI
via fna2_b200.qk_prep) against the reference fixtures and the oracle."""
import types

import pytest
import torch

from oracle import qk_prep_oracle as Q
from tests.qkprep_golden import CASES, load

pytestmark = pytest.mark.gpu

REL_L2 = 1e-2
MAX_ABS = 2e-2


def _close(name, got, ref):
    got, ref = got.float().cpu(), ref.float().cpu()
    assert torch.isfinite(got).all(), f"{name}: non-finite"
    rel = ((got - ref).norm() / ref.norm().clamp_min(1e-30)).item()
    mab = (got - ref).abs().max().item()
    bound = MAX_ABS * max(1.0, ref.abs().max().item())
    assert rel < REL_L2 and mab < bound, f"{name}: rel_l2 {rel:.3g} max_abs {mab:.3g} (bound {bound:.3g})"


def _run(q, k, cu, wq, wk, eps, inv, dqo, dko, use_norm=True, use_rope=True):
    from fna2_b200.qk_prep import apply_qk_norm_rope_varlen
    dev = "cuda"
    ql = q.to(dev).requires_grad_(True)
    kl = k.to(dev).requires_grad_(True)
    norms = (None, None)
    if use_norm:
        norms = tuple(types.SimpleNamespace(weight=w.to(dev).requires_grad_(True), eps=eps) for w in (wq, wk))
    rope = types.SimpleNamespace(inv_freq=inv) if use_rope else None
    qo, ko = apply_qk_norm_rope_varlen(ql, kl, cu.to(dev), norms[0], norms[1], rope)
    lo, hi = int(cu[0]), int(cu[-1])
    loss = (qo[lo:hi].float() * dqo[lo:hi].to(dev).float()).sum() + (ko[lo:hi].float() * dko[lo:hi].to(dev).float()).sum()
    loss.backward()
    torch.cuda.synchronize()
    gw = (norms[0].weight.grad, norms[1].weight.grad) if use_norm else (None, None)
    return qo, ko, ql.grad, kl.grad, gw[0], gw[1]


@pytest.mark.parametrize("name", CASES)
def test_reference_fixture(name):
    rec, (q, k, wq, wk, inv, cu, dqo, dko) = load(name)
    qo, ko, gq, gk, gwq, gwk = _run(q, k, cu, wq, wk, rec["eps"], inv, dqo, dko)
    lo, hi = int(cu[0]), int(cu[-1])
    _close("q_out", qo[lo:hi], rec["q_out"][lo:hi])
    _close("k_out", ko[lo:hi], rec["k_out"][lo:hi])
    for n, got, want in (("dq", gq, rec["dq"]), ("dk", gk, rec["dk"]), ("dwq", gwq, rec["dwq"]), ("dwk", gwk, rec["dwk"])):
        assert got.dtype == want.dtype, n
        _close(n, got, want)


@pytest.mark.parametrize("use_norm,use_rope", [(True, False), (False, True)])
@pytest.mark.parametrize("D", [64, 128])
def test_partial_chains_vs_oracle(D, use_norm, use_rope):
    q, k, wq, wk, inv, cu, dqo, dko = Q.make_inputs([3, 0, 130, 1, 60], 4, 2, D, 21 + D)
    qo, ko, gq, gk, gwq, gwk = _run(q, k, cu, wq, wk, 1e-6, inv, dqo, dko, use_norm, use_rope)
    rq, rk, grads = Q.qk_prep_with_grads(q, k, cu, wq if use_norm else None, wk if use_norm else None, 1e-6,
                                         inv if use_rope else None, dqo, dko) if use_norm else (None, None, None)
    if not use_norm:
        leaves = [t.detach().clone().requires_grad_(True) for t in (q, k)]
        rq, rk = Q.qk_prep(leaves[0], leaves[1], cu, None, None, 1e-6, inv)
        ((rq.float() * dqo.float()).sum() + (rk.float() * dko.float()).sum()).backward()
        grads = [leaves[0].grad, leaves[1].grad, None, None]
    _close("q_out", qo, rq)
    _close("k_out", ko, rk)
    _close("dq", gq, grads[0])
    _close("dk", gk, grads[1])
    if use_norm:
        _close("dwq", gwq, grads[2])
        _close("dwk", gwk, grads[3])


def test_tokens_after_last_sequence_get_zero_gradient():
    q, k, wq, wk, inv, cu, dqo, dko = Q.make_inputs([10, 20], 2, 2, 128, 5, tail=6)
    _, _, gq, gk, _, _ = _run(q, k, cu, wq, wk, 1e-6, inv, dqo, dko)
    assert (gq[30:] == 0).all() and (gk[30:] == 0).all()


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("D", [64, 128])
def test_many_heads_strided_views_vs_oracle(D, dtype):
    """16 query and 8 key heads, so units of rows fall wholly inside q or k, and
    q, k as head slices of one packed qkv tensor (token stride != heads * D)."""
    H, H_KV, lengths = 16, 8, [300, 5, 1000, 1]
    T = sum(lengths)
    g = torch.Generator().manual_seed(40 + D)
    qkv = torch.randn(T, H + 2 * H_KV, D, generator=g).to(dtype).cuda()
    q, k = qkv[:, :H], qkv[:, H:H + H_KV]
    assert q.stride(0) == (H + 2 * H_KV) * D
    _, _, wq, wk, inv, cu, _, _ = Q.make_inputs(lengths, H, H_KV, D, 41 + D, dtype)
    dqo = torch.randn(T, H, D, generator=g).bfloat16()
    dko = torch.randn(T, H_KV, D, generator=g).bfloat16()
    qo, ko, gq, gk, gwq, gwk = _run(q, k, cu, wq, wk, 1e-6, inv, dqo, dko)
    rq, rk, grads = Q.qk_prep_with_grads(q.cpu().contiguous(), k.cpu().contiguous(), cu, wq, wk, 1e-6, inv, dqo, dko)
    _close("q_out", qo, rq)
    _close("k_out", ko, rk)
    for n, got, want in zip(("dq", "dk", "dwq", "dwk"), (gq, gk, gwq, gwk), grads):
        _close(n, got, want)
