"""CPU restatement of the reference's varlen QK-RMSNorm + RoPE transform.

TEST INFRASTRUCTURE ONLY: imported by tests/ (as the checker of the CUDA
kernels in fna2_b200/csrc/fna2_qkprep.cu); never by the product path.

Restates, in plain PyTorch with the reference's dtype behaviour:
  RMSNorm.forward                         FNA2/attention_fna2.py:100-102
  RotaryPositionalEmbedding._update_cache  :148-155  (cos/sin table built in the
                                                     dtype of the rotated tensor)
  RotaryPositionalEmbedding._rotate_half   :157-160
  RotaryPositionalEmbedding.forward        :162-170
  NaylisAttention._forward_varlen q/k steps :558-566, cast :568-572
  NaylisAttention._apply_rope_varlen       :620-647  (positions restart at 0 per
                                                     packed sequence)
Pinned against fixtures produced by the reference's own classes
(tests/golden/make_golden_qkprep.py).
"""
from __future__ import annotations

import torch


def make_inputs(lengths, H, H_KV, D, seed, dtype=torch.float32, lead=0, tail=0, yarn_scale=1.0,
                weights_dtype=None):
    """Seeded q [T,H,D], k [T,H_KV,D], RMSNorm weights [D] (x2), inv_freq [D/2],
    cu_seqlens [N+1] (int32), upstream gradients of the two bf16 outputs.
    `lead`/`tail` tokens lie outside every sequence (cu[0] = lead)."""
    g = torch.Generator().manual_seed(seed)
    T = lead + sum(lengths) + tail
    q = torch.randn(T, H, D, generator=g) * 1.5
    k = torch.randn(T, H_KV, D, generator=g) * 1.5
    wq = 1.0 + 0.1 * torch.randn(D, generator=g)
    wk = 1.0 + 0.1 * torch.randn(D, generator=g)
    dq = torch.randn(T, H, D, generator=g)
    dk = torch.randn(T, H_KV, D, generator=g)
    cu = torch.tensor([lead] + [lead + s for s in torch.tensor(lengths).cumsum(0).tolist()], dtype=torch.int32)
    inv_freq = rope_inv_freq(D, yarn_scale=yarn_scale)
    wdt = weights_dtype or dtype
    return (q.to(dtype), k.to(dtype), wq.to(wdt), wk.to(wdt), inv_freq, cu,
            dq.to(torch.bfloat16), dk.to(torch.bfloat16))


def rope_inv_freq(D, base=10000, yarn_scale=1.0):
    """RotaryPositionalEmbedding.inv_freq (attention_fna2.py:122-145), YaRN included."""
    freqs = torch.arange(0, D, 2).float() / D
    inv = 1.0 / (base ** freqs)
    if yarn_scale == 1.0:
        return inv
    beta = max(D // 2, int(D * 0.25))
    dims = torch.arange(0, D, 2).float()
    scale = torch.where(dims < beta, torch.ones_like(dims), 1 + (yarn_scale - 1) * (dims - beta) / (D - beta))
    return inv / scale


def rmsnorm(x, w, eps):
    """attention_fna2.py:100-102."""
    return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * w


def rotate_half(x):
    """attention_fna2.py:157-160."""
    h = x.shape[-1] // 2
    return torch.cat((-x[..., h:], x[..., :h]), dim=-1)


def rope_table(n, inv_freq, dtype):
    """cos/sin for positions 0..n-1, built in `dtype` (attention_fna2.py:148-155)."""
    t = torch.arange(n, dtype=dtype)
    freqs = torch.outer(t, inv_freq.to(dtype))
    emb = torch.cat((freqs, freqs), dim=-1)
    return emb.cos(), emb.sin()


def qk_prep(q, k, cu, wq=None, wk=None, eps=1e-6, inv_freq=None):
    """The reference's q/k path of _forward_varlen: norm, varlen RoPE, then the
    cast of fp32 to bf16.  Tokens outside every sequence come back as NaN when
    RoPE is on (the reference leaves them unset)."""
    if wq is not None:
        q = rmsnorm(q, wq, eps)
        k = rmsnorm(k, wk, eps)
    if inv_freq is not None:
        q_out = torch.full_like(q, float("nan"))
        k_out = torch.full_like(k, float("nan"))
        cu_l = cu.tolist()
        for s in range(len(cu_l) - 1):
            a, b = cu_l[s], cu_l[s + 1]
            if b <= a:
                continue
            cos, sin = rope_table(b - a, inv_freq, q.dtype)
            cos, sin = cos[:, None, :], sin[:, None, :]
            q_out[a:b] = q[a:b] * cos + rotate_half(q[a:b]) * sin
            k_out[a:b] = k[a:b] * cos + rotate_half(k[a:b]) * sin
        q, k = q_out, k_out
    return q.to(torch.bfloat16), k.to(torch.bfloat16)


def qk_prep_with_grads(q, k, cu, wq, wk, eps, inv_freq, dq_out, dk_out):
    """Outputs and the gradients of q, k and the weights for upstream gradients
    dq_out/dk_out (only tokens inside sequences carry gradient)."""
    leaves = [t.detach().clone().requires_grad_(True) for t in (q, k, wq, wk)]
    qo, ko = qk_prep(leaves[0], leaves[1], cu, leaves[2], leaves[3], eps, inv_freq)
    inside = torch.zeros(q.shape[0], dtype=torch.bool)
    cu_l = cu.tolist()
    inside[cu_l[0]:cu_l[-1]] = True
    loss = (torch.where(inside[:, None, None], qo.float(), 0.0) * dq_out.float()).sum() + \
           (torch.where(inside[:, None, None], ko.float(), 0.0) * dk_out.float()).sum()
    loss.backward()
    return qo, ko, [t.grad for t in leaves]
