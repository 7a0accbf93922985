"""CPU oracle for FNA2 fused relational-bias attention (TEST INFRASTRUCTURE ONLY).

This module is the checker, never the product: only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / reference arm
import it.  The CUDA path in ``fna2_b200`` never calls into it.

It restates, in plain PyTorch on the CPU, the arithmetic of the reference
implementation (myAiByMe/FNA2):

* forward  -- ``FNA2/flash_naylis_attn.py:146-201`` (dense) and ``:302-349``
  (varlen): ``S = scale*Q K^T + gs[h]*R_q R_k^T`` for graph heads ``h < H_G``
  (``:159-165``), ``S = scale*Q K^T`` for vanilla heads, causal mask on
  sequence-local positions (``:168-170``, ``:322-323``), online softmax with
  ``O = acc/(l+1e-6)`` and ``LSE = m + log(l+1e-6)`` (``:192,195``,
  ``:340-341``), GQA ``kv_head = h // (H/H_KV)`` (``:99``, ``:262``);
* backward -- ``:356-693`` and ``:900-1208``: ``Delta = rowsum(dO*O)``,
  ``P = exp(S-LSE)``, ``dS = P*(dP-Delta)``, ``dV = P^T dO``,
  ``dK = scale dS^T Q``, ``dQ = scale dS K``, ``dR_k = gs dS^T R_q``,
  ``dR_q = gs dS R_k``, ``d_gs[h] = sum(dS * R_q R_k^T)`` (``:518-553``,
  ``:673-693``);
* the validation suite's eager path ``_sdpa_reference``
  (``FNA2/validate_fna2.py:84-112``): materialised ``[B,H,S,S]`` bias added to
  a causal ``-inf`` mask, fed to ``F.scaled_dot_product_attention``;
* varlen checks are per-sequence dense calls concatenated with ``d_gs``
  summed, as ``validate_fna2.py:218-240`` and ``:288-325`` do.

The oracle is pinned against golden vectors produced by the reference itself
(``tests/golden/make_golden.py``): the reference's ``_sdpa_reference`` run in
fp32 on the CPU, and the reference's Triton kernels run in fp32 by the Triton
CPU interpreter.
"""
from __future__ import annotations

import math
from typing import Dict, List, Optional, Sequence, Tuple

import torch
import torch.nn.functional as F

EPS = 1e-6  # flash_naylis_attn.py:192,195 -- added to l before division / log


def _expand_kv(t: torch.Tensor, h: int) -> torch.Tensor:
    """GQA: repeat each KV head H/H_KV times (validate_fna2.py:94-95)."""
    g = h // t.shape[1]
    return t.repeat_interleave(g, dim=1) if g > 1 else t


def _bias(r_q: torch.Tensor, r_k: torch.Tensor, gs: torch.Tensor, h: int) -> torch.Tensor:
    """gs[h] * R_q R_k^T for graph heads, zero for vanilla heads
    (flash_naylis_attn.py:122-130,159-165; validate_fna2.py:98-102)."""
    b, hg, s_q, _ = r_q.shape
    s_k = r_k.shape[2]
    bias = torch.zeros(b, h, s_q, s_k, dtype=r_q.dtype)
    if hg > 0:
        bias[:, :hg] = torch.einsum("bhir,bhjr->bhij", r_q, r_k) * gs.view(1, hg, 1, 1).to(r_q.dtype)
    return bias


def _mask(s_q: int, s_k: int, causal: bool) -> torch.Tensor:
    """True where attention is allowed: local positions, top-left aligned
    (flash_naylis_attn.py:169,322)."""
    if not causal:
        return torch.ones(s_q, s_k, dtype=torch.bool)
    i = torch.arange(s_q).view(-1, 1)
    j = torch.arange(s_k).view(1, -1)
    return i >= j


def scores(q, k, r_q, r_k, gs, scale, causal):
    """Masked logits S (fp64/fp32 as given), shape [B,H,S_q,S_k]."""
    h = q.shape[1]
    ke = _expand_kv(k, h)
    s = scale * torch.einsum("bhid,bhjd->bhij", q, ke) + _bias(r_q, r_k, gs, h)
    m = _mask(q.shape[2], k.shape[2], causal)
    return s.masked_fill(~m, float("-inf"))


def attention_fwd(q, k, v, r_q, r_k, gs, scale: float, causal: bool = True):
    """Dense forward with the kernel's exact normalisation.

    Shapes: q [B,H,S,D], k/v [B,H_KV,S,D], r_q/r_k [B,H_G,S,r], gs [H_G].
    Returns (out [B,H,S,D], lse [B,H,S]) in the dtype of the inputs.
    Rows with no visible key give out = 0 and lse = -inf, as the reference
    does when its KV loop is empty (flash_naylis_attn.py:300-302).
    """
    h = q.shape[1]
    s = scores(q, k, r_q, r_k, gs, scale, causal)
    m = s.amax(dim=-1, keepdim=True)
    m_safe = torch.where(torch.isfinite(m), m, torch.zeros_like(m))
    p = torch.exp(s - m_safe)
    l = p.sum(-1, keepdim=True)
    out = torch.einsum("bhij,bhjd->bhid", p, _expand_kv(v, h)) / (l + EPS)
    lse = (m + torch.log(l + EPS)).squeeze(-1)
    return out, lse


def attention_bwd(q, k, v, r_q, r_k, gs, out, lse, dout, scale: float, causal: bool = True,
                  ds_bf16: bool = False, dgs_terms: bool = False):
    """Explicit FA2-style backward (flash_naylis_attn.py:356-693).

    Returns (dq, dk, dv, dr_q, dr_k, d_gs); dk/dv are summed over the query
    heads that share a KV head (the reference's atomic_add, :546-547).

    ``ds_bf16`` rounds dS to bf16 before every contraction that consumes it
    (dq, dk, dr_q, dr_k and d_gs): the arithmetic of the sm_100a kernels,
    which feed dS to the tensor cores in bf16 and form d_gs from the same
    contraction.  The reference rounds dS to bf16 for dq/dk/dr (``ds.to(
    q.dtype)``, :529,:535,:679,:683) but sums d_gs from the fp32 dS (:537-538).
    ``dgs_terms`` appends, per graph head, the sum of squares of the d_gs
    summands dS_ij * (R_q R_k^T)_ij (its conditioning: rounding each summand
    by a relative eps moves the sum by about eps times its square root).
    """
    b, h, s_q, d = q.shape
    hkv = k.shape[1]
    hg = r_q.shape[1]
    g = h // hkv
    s = scores(q, k, r_q, r_k, gs, scale, causal)
    p = torch.exp(s - lse.unsqueeze(-1))
    p = torch.where(torch.isfinite(s), p, torch.zeros_like(p))
    delta = (dout * out).sum(-1, keepdim=True)                    # :381
    ve = _expand_kv(v, h)
    ke = _expand_kv(k, h)
    dp = torch.einsum("bhid,bhjd->bhij", dout, ve)                 # :522
    ds = p * (dp - delta)                                          # :523
    if ds_bf16:
        ds = ds.to(torch.bfloat16).to(ds.dtype)
    dv_e = torch.einsum("bhij,bhid->bhjd", p, dout)                # :527
    dk_e = scale * torch.einsum("bhij,bhid->bhjd", ds, q)          # :529
    dq = scale * torch.einsum("bhij,bhjd->bhid", ds, ke)           # :679
    dv = dv_e.view(b, hkv, g, -1, d).sum(2)
    dk = dk_e.view(b, hkv, g, -1, d).sum(2)
    dsg = ds[:, :hg]
    gsv = gs.view(1, hg, 1, 1).to(q.dtype)
    dr_q = gsv * torch.einsum("bhij,bhjr->bhir", dsg, r_k)         # :683
    dr_k = gsv * torch.einsum("bhij,bhir->bhjr", dsg, r_q)         # :535
    raw = torch.einsum("bhir,bhjr->bhij", r_q, r_k)
    d_gs = (dsg * raw).sum(dim=(0, 2, 3))                          # :537-538,553
    if dgs_terms:
        return dq, dk, dv, dr_q, dr_k, d_gs, (dsg * raw).square().sum(dim=(0, 2, 3))
    return dq, dk, dv, dr_q, dr_k, d_gs


def sdpa_reference(q, k, v, r_q, r_k, gs, scale: float, causal: bool = True):
    """Restatement of the validation suite's eager path
    ``_sdpa_reference`` (validate_fna2.py:84-112): materialised bias
    ``[B,H,S,S]`` plus a ``-inf`` causal mask, fed to SDPA.  Differentiable
    through autograd (the reference's T2 test takes its grads this way,
    validate_fna2.py:150-159).  No ``+1e-6`` (SDPA normalises exactly)."""
    h = q.shape[1]
    ke, ve = _expand_kv(k, h), _expand_kv(v, h)
    bias = torch.zeros(q.shape[0], h, q.shape[2], k.shape[2], dtype=q.dtype)
    hg = r_q.shape[1]
    if hg > 0:
        bias = torch.cat([
            torch.einsum("bhir,bhjr->bhij", r_q, r_k) * gs.view(1, hg, 1, 1).to(q.dtype),
            bias[:, hg:]], dim=1)
    if causal:
        cm = torch.triu(torch.full((q.shape[2], k.shape[2]), float("-inf"), dtype=q.dtype), diagonal=1)
        bias = bias + cm
    return F.scaled_dot_product_attention(q, ke, ve, attn_mask=bias, is_causal=False, scale=scale)


# ----------------------------------------------------------------------------
# varlen: per-sequence dense calls (validate_fna2.py:218-240, 288-325)
# ----------------------------------------------------------------------------

def _seq_view(t: torch.Tensor, a: int, b: int) -> torch.Tensor:
    """[T, H*, X] slice -> [1, H*, L, X]."""
    return t[a:b].transpose(0, 1).unsqueeze(0)


def varlen_fwd(q, k, v, r_q, r_k, gs, cu_q: Sequence[int], cu_k: Sequence[int], scale: float):
    """Packed forward, always causal (flash_naylis_attn.py:1327-1332).

    q [T,H,D], k/v [T,H_KV,D], r [T,H_G,r]; returns out [T,H,D] and lse
    [T,H] (the reference's varlen LSE layout, :782)."""
    out = torch.zeros_like(q)
    lse = torch.full((q.shape[0], q.shape[1]), float("-inf"), dtype=q.dtype)
    for i in range(len(cu_q) - 1):
        a, b = int(cu_q[i]), int(cu_q[i + 1])
        c, d = int(cu_k[i]), int(cu_k[i + 1])
        if b == a:
            continue
        if d == c:  # no keys: the reference's KV loop is empty -> O = 0, LSE = -inf
            continue
        o, l = attention_fwd(_seq_view(q, a, b), _seq_view(k, c, d), _seq_view(v, c, d),
                             _seq_view(r_q, a, b), _seq_view(r_k, c, d), gs, scale, True)
        out[a:b] = o[0].transpose(0, 1)
        lse[a:b] = l[0].transpose(0, 1)
    return out, lse


def varlen_bwd(q, k, v, r_q, r_k, gs, out, lse, dout, cu_q, cu_k, scale: float, ds_bf16: bool = False,
               dgs_terms: bool = False):
    """Packed backward: per-sequence explicit backward, concatenated, d_gs summed
    (with ``dgs_terms``, the summed squares of the d_gs summands appended)."""
    dq, dk, dv = torch.zeros_like(q), torch.zeros_like(k), torch.zeros_like(v)
    drq, drk = torch.zeros_like(r_q), torch.zeros_like(r_k)
    dgs = torch.zeros_like(gs, dtype=q.dtype)
    terms = torch.zeros_like(gs, dtype=q.dtype)
    for i in range(len(cu_q) - 1):
        a, b = int(cu_q[i]), int(cu_q[i + 1])
        c, d = int(cu_k[i]), int(cu_k[i + 1])
        if b == a or d == c:
            continue
        g = attention_bwd(_seq_view(q, a, b), _seq_view(k, c, d), _seq_view(v, c, d),
                          _seq_view(r_q, a, b), _seq_view(r_k, c, d), gs,
                          _seq_view(out, a, b), lse[a:b].transpose(0, 1).unsqueeze(0),
                          _seq_view(dout, a, b), scale, True, ds_bf16, dgs_terms)
        dq[a:b] = g[0][0].transpose(0, 1)
        dk[c:d] += g[1][0].transpose(0, 1)
        dv[c:d] += g[2][0].transpose(0, 1)
        drq[a:b] = g[3][0].transpose(0, 1)
        drk[c:d] += g[4][0].transpose(0, 1)
        dgs += g[5]
        if dgs_terms:
            terms += g[6]
    if dgs_terms:
        return dq, dk, dv, drq, drk, dgs, terms
    return dq, dk, dv, drq, drk, dgs


# ----------------------------------------------------------------------------
# blocked restatement for full-size checks (any device, fp32 arithmetic)
# ----------------------------------------------------------------------------

def blocked_sequence(q, k, v, r_q, r_k, gs, dout, scale: float, causal: bool = True, block: int = 512,
                     grads: bool = True):
    """Forward and backward of ONE sequence, the same formulas as
    ``attention_fwd`` / ``attention_bwd`` (flash_naylis_attn.py:146-201,
    356-693), evaluated over blocks of ``block`` query rows so that the score
    matrix is never held beyond ``[H, block, L_k]``: full-size BASELINE
    sequences (L up to 32768) fit on a GPU.  Arithmetic is fp32 on whatever
    device the inputs live on (callers disable TF32).

    Packed-slice layout: q/dout ``[L_q, H, D]``, k/v ``[L_k, H_KV, D]``,
    r_q ``[L_q, H_G, r]``, r_k ``[L_k, H_G, r]``, gs ``[H_G]``.  Causal is
    top-left aligned on local positions (key j visible to query i iff j <= i).
    Returns a dict of out, lse ``[L_q, H]`` and, with ``grads``, dq, dk, dv,
    drq, drk (input layouts) and dgs (fp64 sum, ``[H_G]``).
    """
    f32 = torch.float32
    Lq, H, D = q.shape
    Lk, HKV = k.shape[0], k.shape[1]
    HG = r_q.shape[1]
    g = H // HKV
    dev = q.device
    qf = q.to(f32).transpose(0, 1)                                   # [H, Lq, D]
    kf = k.to(f32).transpose(0, 1).repeat_interleave(g, 0)           # [H, Lk, D]
    vf = v.to(f32).transpose(0, 1).repeat_interleave(g, 0)
    rqf = r_q.to(f32).transpose(0, 1)                                # [HG, Lq, r]
    rkf = r_k.to(f32).transpose(0, 1)                                # [HG, Lk, r]
    gsf = gs.to(f32).view(HG, 1, 1)
    out = torch.zeros(H, Lq, D, dtype=f32, device=dev)
    lse = torch.full((H, Lq), float("-inf"), dtype=f32, device=dev)

    def logits(i0, i1):
        kend = min(Lk, i1) if causal else Lk
        s = scale * torch.matmul(qf[:, i0:i1], kf[:, :kend].transpose(1, 2))
        if HG:
            s[:HG] += gsf * torch.matmul(rqf[:, i0:i1], rkf[:, :kend].transpose(1, 2))
        if causal:
            ok = torch.arange(i0, i1, device=dev).view(-1, 1) >= torch.arange(kend, device=dev).view(1, -1)
            s.masked_fill_(~ok, float("-inf"))
        return s, kend

    if Lk > 0:
        for i0 in range(0, Lq, block):
            i1 = min(Lq, i0 + block)
            s, kend = logits(i0, i1)
            m = s.amax(-1, keepdim=True)
            m = torch.where(torch.isfinite(m), m, torch.zeros_like(m))
            p = torch.exp(s - m)
            l = p.sum(-1, keepdim=True)
            out[:, i0:i1] = torch.matmul(p, vf[:, :kend]) / (l + EPS)          # :192
            lse[:, i0:i1] = (m + torch.log(l + EPS)).squeeze(-1)               # :195
    res = {"out": out.transpose(0, 1), "lse": lse.transpose(0, 1)}
    if not grads:
        return res
    dof = dout.to(f32).transpose(0, 1)
    delta = (dof * out).sum(-1, keepdim=True)                                   # :381
    dq = torch.zeros_like(qf)
    dk = torch.zeros(H, Lk, D, dtype=f32, device=dev)
    dv = torch.zeros(H, Lk, D, dtype=f32, device=dev)
    drq = torch.zeros_like(rqf)
    drk = torch.zeros(HG, Lk, rkf.shape[-1], dtype=f32, device=dev)
    dgs = torch.zeros(HG, dtype=torch.float64, device=dev)
    if Lk > 0:
        for i0 in range(0, Lq, block):
            i1 = min(Lq, i0 + block)
            s, kend = logits(i0, i1)
            p = torch.exp(s - lse[:, i0:i1].unsqueeze(-1))                      # :518
            p = torch.where(torch.isfinite(s), p, torch.zeros_like(p))
            dp = torch.matmul(dof[:, i0:i1], vf[:, :kend].transpose(1, 2))     # :522
            ds = p * (dp - delta[:, i0:i1])                                     # :523
            dq[:, i0:i1] = scale * torch.matmul(ds, kf[:, :kend])              # :679
            dk[:, :kend] += scale * torch.matmul(ds.transpose(1, 2), qf[:, i0:i1])   # :529
            dv[:, :kend] += torch.matmul(p.transpose(1, 2), dof[:, i0:i1])     # :527
            if HG:
                dsg = ds[:HG]
                drq[:, i0:i1] = gsf * torch.matmul(dsg, rkf[:, :kend])         # :683
                drk[:, :kend] += gsf * torch.matmul(dsg.transpose(1, 2), rqf[:, i0:i1])  # :535
                raw = torch.matmul(rqf[:, i0:i1], rkf[:, :kend].transpose(1, 2))
                dgs += (dsg * raw).sum(dim=(1, 2)).double()                    # :537-538
    res.update(dq=dq.transpose(0, 1),
               dk=dk.view(HKV, g, Lk, D).sum(1).transpose(0, 1),
               dv=dv.view(HKV, g, Lk, D).sum(1).transpose(0, 1),
               drq=drq.transpose(0, 1), drk=drk.transpose(0, 1), dgs=dgs)
    return res


# ----------------------------------------------------------------------------
# error metrics (validate_fna2.py:115-122 reports max/mean abs; rel-L2 added)
# ----------------------------------------------------------------------------

def errors(ref: torch.Tensor, got: torch.Tensor) -> Dict[str, float]:
    ref = ref.double()
    got = got.double()
    diff = (ref - got)
    scale = ref.abs().max().item() if ref.numel() else 0.0
    return {
        "max_abs": diff.abs().max().item() if ref.numel() else 0.0,
        "mean_abs": diff.abs().mean().item() if ref.numel() else 0.0,
        "rel_l2": (diff.norm() / ref.norm().clamp_min(1e-30)).item() if ref.numel() else 0.0,
        "ref_max": scale,
    }


# ----------------------------------------------------------------------------
# seeded inputs for the BASELINE configurations
# ----------------------------------------------------------------------------

def make_dense_inputs(B, H, S, D, r, H_KV=None, H_G=None, seed=0, gs_value=None,
                      dtype=torch.float32):
    """Q,K,V ~ N(0,1); R ~ N(0,1/r); dO ~ N(0,1); draw order q,k,v,r_q,r_k,dO
    with ``torch.Generator().manual_seed(seed)``; gs = ones (north-star formula)
    unless ``gs_value='randn'`` (drawn last) or a float."""
    H_KV = H if H_KV is None else H_KV
    H_G = H if H_G is None else H_G
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, H, S, D, generator=g, dtype=dtype)
    k = torch.randn(B, H_KV, S, D, generator=g, dtype=dtype)
    v = torch.randn(B, H_KV, S, D, generator=g, dtype=dtype)
    rq = torch.randn(B, H_G, S, r, generator=g, dtype=dtype) / math.sqrt(r)
    rk = torch.randn(B, H_G, S, r, generator=g, dtype=dtype) / math.sqrt(r)
    do = torch.randn(B, H, S, D, generator=g, dtype=dtype)
    if gs_value is None:
        gs = torch.ones(H_G, dtype=torch.float32)
    elif gs_value == "randn":
        gs = torch.randn(H_G, generator=g, dtype=torch.float32)
    else:
        gs = torch.full((H_G,), float(gs_value), dtype=torch.float32)
    return q, k, v, rq, rk, gs, do


def make_varlen_inputs(lengths: Sequence[int], H, D, r, H_KV=None, H_G=None, seed=0,
                       gs_value=None, dtype=torch.float32):
    """Packed [T,H*,X] inputs with cu_seqlens (int list); same draw order."""
    H_KV = H if H_KV is None else H_KV
    H_G = H if H_G is None else H_G
    T = int(sum(lengths))
    cu = [0]
    for L in lengths:
        cu.append(cu[-1] + int(L))
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(T, H, D, generator=g, dtype=dtype)
    k = torch.randn(T, H_KV, D, generator=g, dtype=dtype)
    v = torch.randn(T, H_KV, D, generator=g, dtype=dtype)
    rq = torch.randn(T, H_G, r, generator=g, dtype=dtype) / math.sqrt(r)
    rk = torch.randn(T, H_G, r, generator=g, dtype=dtype) / math.sqrt(r)
    do = torch.randn(T, H, D, generator=g, dtype=dtype)
    if gs_value is None:
        gs = torch.ones(H_G, dtype=torch.float32)
    elif gs_value == "randn":
        gs = torch.randn(H_G, generator=g, dtype=torch.float32)
    else:
        gs = torch.full((H_G,), float(gs_value), dtype=torch.float32)
    return q, k, v, rq, rk, gs, do, cu


def bf16_round(*ts):
    """Round fp32 tensors to bf16-representable fp32 values (inputs the GPU
    kernel sees exactly)."""
    return tuple(t.to(torch.bfloat16).to(torch.float32) if t.dtype == torch.float32 and t.dim() > 1 else t
                 for t in ts)
