"""The decode oracle equals the last query row of the prefill oracle (which is
pinned to the reference's golden vectors), with and without the appended
token, for GQA and mixed graph/vanilla heads."""
import math

import pytest
import torch

from oracle import decode_oracle as DO
from oracle import fna2_oracle as FO


@pytest.mark.parametrize("H,H_KV,H_G,D,R", [(4, 4, 4, 64, 16), (6, 2, 3, 32, 32)])
@pytest.mark.parametrize("append", [False, True])
def test_decode_oracle_is_prefill_last_row(H, H_KV, H_G, D, R, append):
    g = torch.Generator().manual_seed(H * 100 + D + append)
    lens = [1, 9, 40]
    S = max(lens) + 1
    B = len(lens)
    k = torch.randn(B, S, H_KV, D, generator=g)
    v = torch.randn(B, S, H_KV, D, generator=g)
    rk = torch.randn(B, S, H_G, R, generator=g) * 0.3
    gs = torch.randn(H_G, generator=g)
    scale = 1.0 / math.sqrt(D)
    for b, n in enumerate(lens):  # sequence b holds n + 1 tokens; the last one is the query
        q_all = torch.randn(1, H, n + 1, D, generator=g)
        rq_all = torch.randn(1, H_G, n + 1, R, generator=g) * 0.3
        kb, vb = k[b:b + 1, :n + 1].transpose(1, 2), v[b:b + 1, :n + 1].transpose(1, 2)
        rkb = rk[b:b + 1, :n + 1].transpose(1, 2)
        o_ref, lse_ref = FO.attention_fwd(q_all.double(), kb.double(), vb.double(), rq_all.double(),
                                          rkb.double(), gs.double(), scale, True)
        cached = n if append else n + 1
        kw = dict(k_new=k[b:b + 1, n], v_new=v[b:b + 1, n], rk_new=rk[b:b + 1, n]) if append else {}
        o, lse = DO.decode(q_all[:, :, n], k[b:b + 1], v[b:b + 1], [cached], rq_all[:, :, n], rk[b:b + 1], gs,
                           scale=scale, **kw)
        torch.testing.assert_close(o[0].double(), o_ref[0, :, n], atol=1e-5, rtol=1e-5)
        torch.testing.assert_close(lse[0].double(), lse_ref[0, :, n].double(), atol=1e-5, rtol=1e-5)
