"""CPU restatement of KV-cache decode with the relational bias.

TEST INFRASTRUCTURE ONLY: imported by tests/ and bench.py's CPU leg (as the
checker of fna2_b200/csrc/fna2_decode.cu); never by the product path.

The reference has no decode path with the bias (FNA2/attention_fna2.py:428-432
drops graph_bias once past_kv is set), so this restates the op's definition
for the last query row of a sequence: the logits, GQA mapping and
normalisation of the prefill kernels (FNA2/flash_naylis_attn.py:99,159-165,
192,195), with the query placed after every key (no mask).  Its agreement with
the prefill oracle's last row (oracle/fna2_oracle.py, pinned to the
reference's golden vectors) is checked in tests/test_decode_oracle.py.
"""
from __future__ import annotations

import math

import torch

EPS = 1e-6


def decode(q, k_cache, v_cache, cache_seqlens, r_q=None, rk_cache=None, graph_scale=None, k_new=None, v_new=None,
           rk_new=None, scale=None):
    """q [B,H,D]; caches [B,S,H_KV,D] / [B,S,H_G,R]; cache_seqlens [B] (host ints).
    Returns (out [B,H,D] fp32, lse [B,H] fp32)."""
    B, H, D = q.shape
    h_kv = k_cache.shape[2]
    grp = H // h_kv
    hg = 0 if r_q is None else r_q.shape[1]
    scale = scale if scale is not None else 1.0 / math.sqrt(D)
    out = torch.zeros(B, H, D, dtype=torch.float64)
    lse = torch.full((B, H), float("-inf"), dtype=torch.float64)
    for b in range(B):
        n = int(cache_seqlens[b])
        ks, vs = k_cache[b, :n].double(), v_cache[b, :n].double()
        rks = rk_cache[b, :n].double() if hg else None
        if k_new is not None:
            ks = torch.cat([ks, k_new[b][None].double()])
            vs = torch.cat([vs, v_new[b][None].double()])
            if hg:
                rks = torch.cat([rks, rk_new[b][None].double()])
        if ks.shape[0] == 0:
            continue
        for h in range(H):
            kh = h // grp
            s = scale * (ks[:, kh] @ q[b, h].double())
            if h < hg:
                s = s + float(graph_scale[h]) * (rks[:, h] @ r_q[b, h].double())
            m = s.max()
            e = torch.exp(s - m)
            l = e.sum()
            out[b, h] = (e @ vs[:, kh]) / (l + EPS)
            lse[b, h] = m + torch.log(l + EPS)
    return out.float(), lse.float()
