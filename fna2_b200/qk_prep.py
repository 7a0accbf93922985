"""Varlen QK-RMSNorm + RoPE before the attention, fused into one CUDA pass.

Drop-in for the q/k steps of ``NaylisAttention._forward_varlen``
(FNA2/attention_fna2.py:558-572): ``q_norm(q)``, ``k_norm(k)``,
``_apply_rope_varlen(q, k, cu_seqlens)`` (:620-647) and the cast of fp32 to
bf16.  The reference rotates every packed sequence in a host loop after a
``.tolist()`` sync; here one kernel handles all tokens and heads, with each
token's position found from ``cu_seqlens`` on the device.  Gradients flow to
q, k and both RMSNorm weights.

``cu_seqlens`` gives absolute token offsets (as for ``flash_naylis_attn``);
the reference's loop assumes ``cu_seqlens[0] == 0``.
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch

from . import _lib

_DT = {torch.float32: _lib.FNA2_DTYPE_F32, torch.bfloat16: _lib.FNA2_DTYPE_BF16}


def _rows(t: Optional[torch.Tensor]) -> _lib.Fna2Rows:
    if t is None:
        return _lib.Fna2Rows()
    return _lib.Fna2Rows(t.data_ptr(), t.stride(0), t.stride(1))


def _prep_rows(t: torch.Tensor) -> torch.Tensor:
    # column stride 1, 16-byte aligned rows; anything else is copied once
    vec = 16 // t.element_size()
    if t.stride(2) != 1 or t.stride(0) % vec or t.stride(1) % vec or t.data_ptr() % 16:
        t = t.contiguous()
    return t


def _args(q, k, cu, wq, wk, eps, inv_freq, rope_dtype) -> _lib.Fna2QkPrepArgs:
    a = _lib.Fna2QkPrepArgs()
    a.total_tokens = q.shape[0]
    a.num_seqs = 0 if cu is None else cu.numel() - 1
    a.cu_seqlens = None if cu is None else cu.data_ptr()
    a.heads_q, a.heads_k, a.head_dim = q.shape[1], k.shape[1], q.shape[2]
    a.in_dtype = _DT[q.dtype]
    a.weight_dtype = _DT[wq.dtype] if wq is not None else _lib.FNA2_DTYPE_F32
    a.rope_dtype = _DT[rope_dtype]
    a.q_in, a.k_in = _rows(q), _rows(k)
    a.q_weight = None if wq is None else wq.data_ptr()
    a.k_weight = None if wk is None else wk.data_ptr()
    a.eps = float(eps)
    a.inv_freq = None if inv_freq is None else inv_freq.data_ptr()
    return a


class QkNormRopeVarlenFunc(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, cu, wq, wk, eps, inv_freq, rope_dtype):
        lib = _lib.load()
        q, k = _prep_rows(q), _prep_rows(k)
        qo = torch.empty(q.shape, dtype=torch.bfloat16, device=q.device)
        ko = torch.empty(k.shape, dtype=torch.bfloat16, device=k.device)
        a = _args(q, k, cu, wq, wk, eps, inv_freq, rope_dtype)
        a.q_out, a.k_out = _rows(qo), _rows(ko)
        _lib.check(lib.fna2_qk_prep_fwd(a, torch.cuda.current_stream(q.device).cuda_stream), "fna2_qk_prep_fwd")
        ctx.save_for_backward(q, k, cu, wq, wk, inv_freq)
        ctx.eps, ctx.rope_dtype = eps, rope_dtype
        return qo, ko

    @staticmethod
    def backward(ctx, gqo, gko):
        lib = _lib.load()
        q, k, cu, wq, wk, inv_freq = ctx.saved_tensors
        gqo = _prep_rows(torch.zeros_like(q, dtype=torch.bfloat16) if gqo is None else gqo.to(torch.bfloat16))
        gko = _prep_rows(torch.zeros_like(k, dtype=torch.bfloat16) if gko is None else gko.to(torch.bfloat16))
        dq, dk = torch.empty_like(q), torch.empty_like(k)
        dwq = dwk = None
        b = _lib.Fna2QkPrepBwdArgs()
        b.fwd = _args(q, k, cu, wq, wk, ctx.eps, inv_freq, ctx.rope_dtype)
        b.dq_out, b.dk_out, b.dq_in, b.dk_in = _rows(gqo), _rows(gko), _rows(dq), _rows(dk)
        if wq is not None:
            dwq = torch.zeros(wq.shape, dtype=torch.float32, device=q.device)
            dwk = torch.zeros(wk.shape, dtype=torch.float32, device=q.device)
            b.dq_weight, b.dk_weight = dwq.data_ptr(), dwk.data_ptr()
        _lib.check(lib.fna2_qk_prep_bwd(b, torch.cuda.current_stream(q.device).cuda_stream), "fna2_qk_prep_bwd")
        if wq is not None:
            dwq, dwk = dwq.to(wq.dtype), dwk.to(wk.dtype)
        return dq, dk, None, dwq, dwk, None, None, None


def apply_qk_norm_rope_varlen(q: torch.Tensor, k: torch.Tensor, cu_seqlens: Optional[torch.Tensor],
                              q_norm=None, k_norm=None, rope=None) -> Tuple[torch.Tensor, torch.Tensor]:
    """q [T, H, D], k [T, H_KV, D] (fp32 or bf16, CUDA); cu_seqlens int32 [N+1]
    (needed when ``rope`` is given).  ``q_norm``/``k_norm``: the reference's
    ``RMSNorm`` modules (anything with ``.weight`` and ``.eps``) or None;
    ``rope``: its ``RotaryPositionalEmbedding`` (anything with ``.inv_freq``)
    or None.  Returns bf16 (q, k) as ``_forward_varlen`` hands them to
    ``flash_naylis_attn``.  head_dim must be 64 or 128."""
    assert q.is_cuda and k.is_cuda, "q and k must be CUDA tensors"
    assert q.dim() == 3 and k.dim() == 3 and q.shape[0] == k.shape[0] and q.shape[2] == k.shape[2]
    assert q.dtype in _DT and k.dtype == q.dtype, "q, k: fp32 or bf16, same dtype"
    assert (q_norm is None) == (k_norm is None), "give both norms or neither"
    wq = wk = None
    eps = 1e-6
    rope_dtype = q.dtype
    if q_norm is not None:
        wq, wk = q_norm.weight, k_norm.weight
        assert wq.dtype in _DT and wk.dtype == wq.dtype, "norm weights: fp32 or bf16, same dtype"
        assert float(q_norm.eps) == float(k_norm.eps), "the two norms must share eps"
        eps = float(q_norm.eps)
        rope_dtype = torch.promote_types(q.dtype, wq.dtype)  # dtype of x * rms * weight
    inv_freq = None
    if rope is not None:
        assert cu_seqlens is not None and cu_seqlens.dtype == torch.int32 and cu_seqlens.is_cuda
        inv_freq = rope.inv_freq.detach().to(device=q.device, dtype=torch.float32).contiguous()
    cu = None if cu_seqlens is None else cu_seqlens.contiguous()
    return QkNormRopeVarlenFunc.apply(q, k, cu, wq, wk, eps, inv_freq, rope_dtype)
