"""Fused R_q / R_k projection feeding the attention op.

The reference computes the relational factors with two Linear layers and
materialises each result (FNA2/attention_fna2.py:301-335):

    dense   R = rel_proj(x).view(B, S, H_G, R).permute(0, 2, 1, 3).to(dtype).contiguous()
    varlen  R = rel_proj(x).view(T, H_G, R).to(dtype).contiguous()

for rel_q_proj and rel_k_proj in turn.  Here both weights form one
[2*H_G*R, E] matrix, so x is read once by one GEMM (a plain library GEMM:
cuBLAS through torch), and R_q, R_k are returned as strided views of its
[..., 2*H_G*R] output in the layouts flash_naylis_attn takes directly (any
16-byte aligned strides): no permute copy, no contiguous() copy.  Values equal
the reference's (the same dot products, rounded once to `dtype`); autograd
runs through the GEMM and the views (dX = dY W, dW = dY^T X).
"""
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


def compute_rq_rk(x: torch.Tensor, weight: torch.Tensor, graph_heads: int, rank: int,
                  dtype: torch.dtype = torch.bfloat16) -> Tuple[torch.Tensor, torch.Tensor]:
    """R_q, R_k from x ([B, S, E] dense or [T, E] packed) and the stacked weight
    [rel_q_proj.weight; rel_k_proj.weight] ([2*H_G*R, E])."""
    if x.dim() not in (2, 3):
        raise ValueError(f"x must be [B, S, E] or [T, E] (got {tuple(x.shape)})")
    if weight.shape != (2 * graph_heads * rank, x.shape[-1]):
        raise ValueError(f"weight must be [{2 * graph_heads * rank}, {x.shape[-1]}] (got {tuple(weight.shape)})")
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
