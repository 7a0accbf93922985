"""KV-cache decode with the relational bias (one new query token per sequence).

The reference has no such path: NaylisAttention's decode step
(FNA2/attention_fna2.py:428-432) bypasses FNA2 when past_kv is set and drops
graph_bias, since R_k of earlier tokens is not kept.  Here R_k is cached per
graph head beside K and V and the bias is applied exactly as the prefill op
applies it to the last query row of a sequence:

    S[h, j] = scale * <q_h, k_j> + graph_scale[h] * <r_q,h, r_k[j, h]>   (h < H_G)
    out = softmax(S) V with out = acc / (l + 1e-6), lse = m + log(l + 1e-6)

Keys are slots [0, cache_seqlens[b]) of sequence b, plus the new key when
k/v (and r_k) are given: the call writes them into slot cache_seqlens[b] of
the caches and attends to them; the caller advances cache_seqlens (NaylisKVCache
below does both).  The work runs in fna2_decode of libfna2_b200.so.
"""
import ctypes
import math
from typing import Optional

import torch

from . import _lib


def _check(t: torch.Tensor, name: str, dims: int):
    if t.dtype != torch.bfloat16:
        raise TypeError(f"{name} must be bfloat16 (got {t.dtype})")
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor")
    if t.dim() != dims:
        raise ValueError(f"{name} must have {dims} dims (got shape {tuple(t.shape)})")
    if t.stride(-1) != 1:
        raise ValueError(f"{name} must have unit stride in its last dim")


def _ptr(t: Optional[torch.Tensor]) -> int:
    return 0 if t is None else t.data_ptr()


def flash_naylis_decode(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                        cache_seqlens: torch.Tensor, r_q: Optional[torch.Tensor] = None,
                        rk_cache: Optional[torch.Tensor] = None, graph_scale: Optional[torch.Tensor] = None,
                        k: Optional[torch.Tensor] = None, v: Optional[torch.Tensor] = None,
                        r_k: Optional[torch.Tensor] = None, softmax_scale: Optional[float] = None,
                        cache_offsets: Optional[torch.Tensor] = None, capacity: Optional[int] = None,
                        return_lse: bool = False, num_splits: int = 0):
    """One decode step.

    q [B, H, D] bf16; r_q [B, H_G, R] bf16 (None: no graph heads); graph_scale [H_G].
    Caches: k_cache, v_cache [B, S_max, H_KV, D] and rk_cache [B, S_max, H_G, R]
    (any strides with a unit last one, e.g. the reference's [B, H_KV, S, D]
    cache passed as .transpose(1, 2)); with cache_offsets [B] int32 they are
    packed instead, [rows, H_KV, D] / [rows, H_G, R], sequence b starting at
    row cache_offsets[b] (give `capacity`, the slots each sequence owns).
    cache_seqlens [B] int32 on the device.  k, v [B, H_KV, D] and r_k [B, H_G, R]:
    the new token's key, appended at slot cache_seqlens[b].
    Returns out [B, H, D] bf16 (and lse [B, H] fp32 if return_lse).
    """
    _check(q, "q", 3)
    B, H, D = q.shape
    packed = cache_offsets is not None
    cdims = 3 if packed else 4
    _check(k_cache, "k_cache", cdims)
    _check(v_cache, "v_cache", cdims)
    H_KV = k_cache.shape[-2]
    H_G, R = 0, 16
    if r_q is not None:
        _check(r_q, "r_q", 3)
        H_G, R = r_q.shape[1], r_q.shape[2]
        if rk_cache is None or graph_scale is None:
            raise ValueError("graph heads (r_q) need rk_cache and graph_scale")
        _check(rk_cache, "rk_cache", cdims)
    if cache_seqlens.dtype != torch.int32 or not cache_seqlens.is_cuda or cache_seqlens.numel() != B:
        raise ValueError("cache_seqlens must be a CUDA int32 tensor of B entries")
    if (k is None) != (v is None) or (k is not None and H_G > 0 and r_k is None):
        raise ValueError("k and v (and r_k when there are graph heads) go together")
    if k is not None:
        _check(k, "k", 3)
        _check(v, "v", 3)
        if r_k is not None:
            _check(r_k, "r_k", 3)
    if capacity is None:
        capacity = k_cache.shape[0] if packed else k_cache.shape[1]
    scale = softmax_scale if softmax_scale is not None else 1.0 / math.sqrt(D)
    out = torch.empty(B, H, D, device=q.device, dtype=torch.bfloat16)
    lse = torch.empty(B, H, device=q.device, dtype=torch.float32) if return_lse else None
    gs = None if graph_scale is None else graph_scale.detach().to(device=q.device, dtype=torch.float32).contiguous()
    seqlens = cache_seqlens.contiguous()
    offsets = None if cache_offsets is None else cache_offsets.to(torch.int32).contiguous()

    def cstrides(t):  # (batch, token, head)
        if t is None:
            return 0, 0, 0
        return (0, t.stride(0), t.stride(1)) if packed else (t.stride(0), t.stride(1), t.stride(2))

    a = _lib.Fna2DecodeArgs()
    a.batch, a.heads, a.kv_heads, a.graph_heads, a.head_dim, a.rank = B, H, H_KV, H_G, D, R
    a.capacity, a.softmax_scale = int(capacity), float(scale)
    a.q, a.q_batch_stride, a.q_head_stride = q.data_ptr(), q.stride(0), q.stride(1)
    if r_q is not None:
        a.r_q, a.rq_batch_stride, a.rq_head_stride = r_q.data_ptr(), r_q.stride(0), r_q.stride(1)
    a.k_cache = k_cache.data_ptr()
    a.k_batch_stride, a.k_token_stride, a.k_head_stride = cstrides(k_cache)
    a.v_cache = v_cache.data_ptr()
    a.v_batch_stride, a.v_token_stride, a.v_head_stride = cstrides(v_cache)
    a.rk_cache = _ptr(rk_cache)
    a.rk_batch_stride, a.rk_token_stride, a.rk_head_stride = cstrides(rk_cache)
    a.graph_scale, a.cache_seqlens, a.cache_offsets = _ptr(gs), seqlens.data_ptr(), _ptr(offsets)
    if k is not None:
        a.k_new, a.kn_batch_stride, a.kn_head_stride = k.data_ptr(), k.stride(0), k.stride(1)
        a.v_new, a.vn_batch_stride, a.vn_head_stride = v.data_ptr(), v.stride(0), v.stride(1)
        if r_k is not None:
            a.rk_new, a.rkn_batch_stride, a.rkn_head_stride = r_k.data_ptr(), r_k.stride(0), r_k.stride(1)
    a.out, a.out_batch_stride, a.out_head_stride = out.data_ptr(), out.stride(0), out.stride(1)
    a.lse, a.num_splits = _ptr(lse), int(num_splits)
    lib = _lib.load()
    ws_bytes = lib.fna2_decode_workspace_size(ctypes.byref(a))
    if ws_bytes == 0 and lib.fna2_last_error():
        raise ValueError(lib.fna2_last_error().decode())
    ws = torch.empty((ws_bytes + 3) // 4, device=q.device, dtype=torch.float32) if ws_bytes else None
    rc = lib.fna2_decode(ctypes.byref(a), _ptr(ws), ws_bytes, torch.cuda.current_stream(q.device).cuda_stream)
    if rc != 0:
        raise RuntimeError(f"fna2_decode failed ({rc}): {lib.fna2_last_error().decode()}")
    return (out, lse) if return_lse else out


class NaylisKVCache:
    """Preallocated per-sequence caches of K, V and R_k for decode.

    k, v: [B, capacity, H_KV, D] bf16; r_k: [B, capacity, H_G, R] bf16;
    seqlens: [B] int32 on the device.  step() appends the new token's k, v,
    r_k and returns its attention output, then advances seqlens."""

    def __init__(self, batch, capacity, kv_heads, head_dim, graph_heads=0, rank=16, device="cuda"):
        self.k = torch.zeros(batch, capacity, kv_heads, head_dim, device=device, dtype=torch.bfloat16)
        self.v = torch.zeros_like(self.k)
        self.r_k = (torch.zeros(batch, capacity, graph_heads, rank, device=device, dtype=torch.bfloat16)
                    if graph_heads else None)
        self.seqlens = torch.zeros(batch, device=device, dtype=torch.int32)
        self.capacity = capacity

    def prefill(self, k, v, r_k=None, lengths=None):
        """Copy prompt keys [B, S, H_KV, D] (r_k [B, S, H_G, R]) into slots [0, S);
        `lengths` [B] (default S) sets each sequence's cached length."""
        S = k.shape[1]
        self.k[:, :S].copy_(k)
        self.v[:, :S].copy_(v)
        if r_k is not None:
            self.r_k[:, :S].copy_(r_k)
        if lengths is None:
            self.seqlens.fill_(S)
        else:
            self.seqlens.copy_(torch.as_tensor(lengths, dtype=torch.int32))

    def step(self, q, k, v, r_q=None, r_k=None, graph_scale=None, softmax_scale=None, return_lse=False):
        res = flash_naylis_decode(q, self.k, self.v, self.seqlens, r_q, self.r_k, graph_scale, k, v, r_k,
                                  softmax_scale, return_lse=return_lse)
        self.seqlens += 1
        return res
