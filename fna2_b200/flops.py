"""Algorithmic FLOP and byte counts of the FNA2 path (FlashAttention convention).

Per (sequence of length L, query head), with head_dim D and rank r (graph
heads only; vanilla heads have r = 0):

* forward  ``4*D*L^2 + 2*r*L^2``   (S = QK^T + R_q R_k^T, O = P V)
* backward ``10*D*L^2 + 6*r*L^2``  (S recompute, dP = dO V^T, dV = P^T dO,
  dK = dS^T Q, dQ = dS K; bias recompute, dR_k, dR_q)

both halved when causal.  Recomputation beyond these GEMMs (this library's
second score recompute in the dQ kernel) is not counted.
"""
from __future__ import annotations

from typing import Iterable, Sequence


def _heads_terms(H: int, H_G: int, D: int, r: int):
    return H * D, H_G * r


def fwd_flops(lengths: Iterable[int], H: int, H_G: int, D: int, r: int, causal: bool = True) -> float:
    hd, hr = _heads_terms(H, H_G, D, r)
    f = 0.5 if causal else 1.0
    return f * sum((4 * hd + 2 * hr) * float(L) ** 2 for L in lengths)


def bwd_flops(lengths: Iterable[int], H: int, H_G: int, D: int, r: int, causal: bool = True) -> float:
    hd, hr = _heads_terms(H, H_G, D, r)
    f = 0.5 if causal else 1.0
    return f * sum((10 * hd + 6 * hr) * float(L) ** 2 for L in lengths)


def total_flops(lengths: Sequence[int], H: int, H_G: int, D: int, r: int, causal: bool = True) -> float:
    """fwd+bwd = sum_seq (7*D*H + 4*r*H_G) * L^2 for causal."""
    return fwd_flops(lengths, H, H_G, D, r, causal) + bwd_flops(lengths, H, H_G, D, r, causal)


def dkdv_flops(lengths, H, H_G, D, r, causal=True) -> float:
    """Algorithmic share of the key-stationary backward kernel:
    S^T recompute + bias, dP^T, dV, dK, dR_k = (8*D + 4*r) * L^2 (halved if causal)."""
    hd, hr = _heads_terms(H, H_G, D, r)
    f = 0.5 if causal else 1.0
    return f * sum((8 * hd + 4 * hr) * float(L) ** 2 for L in lengths)


def dq_flops(lengths, H, H_G, D, r, causal=True) -> float:
    """Algorithmic share of the query-stationary backward kernel: dQ, dR_q = (2*D + 2*r) * L^2."""
    hd, hr = _heads_terms(H, H_G, D, r)
    f = 0.5 if causal else 1.0
    return f * sum((2 * hd + 2 * hr) * float(L) ** 2 for L in lengths)


def token_bytes(T: int, H: int, H_KV: int, H_G: int, D: int, r: int) -> dict:
    """Compulsory HBM bytes (bf16 tensors read/written once) of one fwd+bwd."""
    q = T * H * D * 2
    kv = T * H_KV * D * 2
    rr = T * H_G * r * 2
    fwd = q + 2 * kv + 2 * rr + q + T * H * 4          # read q,k,v,r_q,r_k; write o, lse
    bwd = (q + 2 * kv + 2 * rr + 2 * q + T * H * 4      # read q,k,v,r,o,dO,lse
           + q + 2 * kv + 2 * rr)                       # write dq,dk,dv,dr_q,dr_k
    return {"fwd": fwd, "bwd": bwd, "total": fwd + bwd}
