"""Fused R_q / R_k projection feeding the attention op.

The reference computes the relational factors with two Linear layers and
materialises each result (FNA2/attention_fna2.py:301-335):

    dense   R = rel_proj(x).view(B, S, H_G, R).permute(0, 2, 1, 3).to(dtype).contiguous()
    varlen  R = rel_proj(x).view(T, H_G, R).to(dtype).contiguous()

for rel_q_proj and rel_k_proj in turn.  Here both weights form one
[2*H_G*R, E] matrix, so x is read once by one GEMM, and R_q, R_k are returned
as strided views of its [..., 2*H_G*R] output in the layouts flash_naylis_attn
takes directly (any 16-byte aligned strides): no permute copy, no contiguous()
copy.  For bf16 inputs on the GPU the three products -- Y = X W^T, dX = dY W
and dW = dY^T X -- run on the library's own tcgen05 GEMM (fna2_gemm in
libfna2_b200.so: operands read K-major or MN-major in place, so no transposed
copies; dW reduces over all tokens in fp32 within one CTA per output tile).  Other
dtypes and CPU tensors use torch.nn.functional.linear.  Values equal the
reference's (the same dot products with fp32 accumulation, rounded once to
`dtype`).
"""
import ctypes
import math
from typing import Optional, Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F


def _split(y: torch.Tensor, graph_heads: int, rank: int, varlen: bool) -> Tuple[torch.Tensor, torch.Tensor]:
    n = graph_heads * rank
    if varlen:  # y [T, 2n] -> [T, H_G, R] views, token stride 2n
        return y[:, :n].unflatten(-1, (graph_heads, rank)), y[:, n:].unflatten(-1, (graph_heads, rank))
    # y [B, S, 2n] -> [B, H_G, S, R] views (strides (S*2n, R, 2n, 1))
    return (y[..., :n].unflatten(-1, (graph_heads, rank)).permute(0, 2, 1, 3),
            y[..., n:].unflatten(-1, (graph_heads, rank)).permute(0, 2, 1, 3))


def _gemm(a: torch.Tensor, a_mn: bool, b: torch.Tensor, b_mn: bool, m: int, n: int, k: int, c: torch.Tensor,
          split: int = 1) -> None:
    """C = A B^T (bf16 c: stored) or C += A B^T (fp32 c), A / B read from their
    row-major storage as K-major or MN-major operands (fna2_gemm)."""
    from . import _lib
    lib = _lib.load()
    args = _lib.Fna2GemmArgs(m, n, k, a.data_ptr(), a.stride(0), int(a_mn), b.data_ptr(), b.stride(0), int(b_mn),
                             c.data_ptr(), c.stride(0),
                             _lib.FNA2_DTYPE_F32 if c.dtype == torch.float32 else _lib.FNA2_DTYPE_BF16, split)
    _lib.check(lib.fna2_gemm(ctypes.byref(args), ctypes.c_void_p(torch.cuda.current_stream(c.device).cuda_stream)),
               "fna2_gemm")


class _StackedProjection(torch.autograd.Function):
    """Y = X W^T for X [T, E], W [2n, E] (bf16, contiguous) on fna2_gemm; the
    backward forms dX = dY W and dW = dY^T X with the same kernel."""

    @staticmethod
    def forward(ctx, x2: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
        T, E = x2.shape
        N = w.shape[0]
        y = torch.empty(T, N, device=x2.device, dtype=torch.bfloat16)
        _gemm(x2, False, w, False, T, N, E, y)
        ctx.save_for_backward(x2, w)
        return y

    @staticmethod
    def backward(ctx, gy: torch.Tensor):
        x2, w = ctx.saved_tensors
        T, E = x2.shape
        N = w.shape[0]
        gy = gy.to(torch.bfloat16).contiguous()
        gx = gw = None
        if ctx.needs_input_grad[0]:  # dX[t][e] = sum_j dY[t][j] W[j][e]: W read N-major in place
            gx = torch.empty(T, E, device=x2.device, dtype=torch.bfloat16)
            _gemm(gy, False, w, True, T, E, N, gx)
        if ctx.needs_input_grad[1]:  # dW[j][e] = sum_t dY[t][j] X[t][e]: both read M/N-major in place
            gw32 = torch.zeros(N, E, device=x2.device, dtype=torch.float32)
            _gemm(gy, True, x2, True, N, E, T, gw32)  # one CTA per output tile, over all tokens
            gw = gw32.to(w.dtype)
        return gx, gw


def _kernel_path(x: torch.Tensor, weight: torch.Tensor) -> bool:
    return (x.is_cuda and weight.is_cuda and x.dtype == torch.bfloat16 and weight.dtype == torch.bfloat16
            and x.shape[-1] % 32 == 0 and weight.shape[0] % 32 == 0 and x.numel() > 0)


def compute_rq_rk(x: torch.Tensor, weight: torch.Tensor, graph_heads: int, rank: int,
                  dtype: torch.dtype = torch.bfloat16) -> Tuple[torch.Tensor, torch.Tensor]:
    """R_q, R_k from x ([B, S, E] dense or [T, E] packed) and the stacked weight
    [rel_q_proj.weight; rel_k_proj.weight] ([2*H_G*R, E])."""
    if x.dim() not in (2, 3):
        raise ValueError(f"x must be [B, S, E] or [T, E] (got {tuple(x.shape)})")
    if weight.shape != (2 * graph_heads * rank, x.shape[-1]):
        raise ValueError(f"weight must be [{2 * graph_heads * rank}, {x.shape[-1]}] (got {tuple(weight.shape)})")
    if _kernel_path(x, weight):
        E = x.shape[-1]
        y = _StackedProjection.apply(x.reshape(-1, E).contiguous(), weight.contiguous())
        y = y.view(*x.shape[:-1], weight.shape[0])
    else:
        y = F.linear(x, weight)
    if y.dtype != dtype:
        y = y.to(dtype)
    return _split(y, graph_heads, rank, varlen=x.dim() == 2)


class FusedRelProjection(nn.Module):
    """Drop-in for NaylisAttention's rel_q_proj + rel_k_proj pair (one stacked
    weight, one GEMM).  forward(x) -> (R_q, R_k) as compute_rq_rk."""

    def __init__(self, embed_dim: int, graph_heads: int, rank: int, device=None, dtype=None):
        super().__init__()
        self.graph_heads, self.rank = graph_heads, rank
        self.weight = nn.Parameter(torch.empty(2 * graph_heads * rank, embed_dim, device=device, dtype=dtype))
        nn.init.normal_(self.weight, std=0.01)  # as the reference initialises both (attention_fna2.py:281-282)

    @classmethod
    def from_linears(cls, rel_q_proj: nn.Linear, rel_k_proj: nn.Linear, graph_heads: int, rank: int):
        m = cls(rel_q_proj.in_features, graph_heads, rank, device=rel_q_proj.weight.device,
                dtype=rel_q_proj.weight.dtype)
        with torch.no_grad():
            m.weight.copy_(torch.cat([rel_q_proj.weight, rel_k_proj.weight]))
        return m

    @property
    def rel_q_weight(self) -> torch.Tensor:
        return self.weight[: self.graph_heads * self.rank]

    @property
    def rel_k_weight(self) -> torch.Tensor:
        return self.weight[self.graph_heads * self.rank:]

    def forward(self, x: torch.Tensor, dtype: Optional[torch.dtype] = torch.bfloat16):
        return compute_rq_rk(x, self.weight, self.graph_heads, self.rank, dtype)
