"""Packing helpers (fna2_b200/packing.py) against fixtures made by the
reference's own pack_batch / pack_documents (tests/golden/packing_cases.json)
and against the oracle restatement; a GPU leg checks the pinned-memory path
and that the produced cu_seqlens drive the varlen attention op."""
import json
import os
import random

import pytest
import torch

from fna2_b200 import packing as P
from oracle import packing_oracle as O

FIX = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "packing_cases.json")


def _fixtures():
    with open(FIX) as f:
        return json.load(f)


@pytest.mark.parametrize("impl", [P.pack_documents, O.pack_documents], ids=["product", "oracle"])
def test_pack_documents_matches_reference(impl):
    for c in _fixtures()["pack_documents"]:
        assert impl(c["docs"], c["max_seq_len"], c["eos_id"]) == c["bins"], c["max_seq_len"]


@pytest.mark.parametrize("impl", [P.pack_batch, O.pack_batch], ids=["product", "oracle"])
def test_pack_batch_matches_reference(impl):
    for c in _fixtures()["pack_batch"]:
        seqs = [torch.tensor(s, dtype=torch.int64).reshape([len(s)] + c["feat"]) for s in c["sequences"]]
        x, cu, mx = impl(seqs, "cpu")
        assert x.tolist() == c["x_packed"]
        assert cu.dtype == torch.int32 and str(cu.dtype) == c["cu_dtype"]
        assert cu.tolist() == c["cu_seqlens"]
        assert mx == c["max_seqlen"] and isinstance(mx, int)


def test_pack_batch_empty_list_is_an_error():
    with pytest.raises(RuntimeError):
        P.pack_batch([], "cpu")


def test_pack_documents_random_vs_oracle():
    rng = random.Random(3)
    for _ in range(200):
        docs = [[rng.randrange(100) for _ in range(rng.randrange(0, 40))] for _ in range(rng.randrange(0, 30))]
        m, eos = rng.randrange(-2, 80), rng.randrange(5)
        assert P.pack_documents(docs, m, eos) == O.pack_documents(docs, m, eos)


def test_pack_documents_batch_chains_both():
    docs = [[5] * 10, [6] * 3, [7] * 30]
    x, cu, mx = P.pack_documents_batch(docs, 16, "cpu")
    bins = O.pack_documents(docs, 16)
    assert x.tolist() == sum(bins, []) and cu.tolist() == [0, 15, 31] and mx == 16


@pytest.mark.gpu
def test_pack_batch_to_gpu_and_varlen_attention():
    from fna2_b200.flash_naylis_attn import flash_naylis_attn
    g = torch.Generator().manual_seed(0)
    lengths = [130, 1, 257, 64]
    seqs = [torch.randint(0, 1000, (n,), generator=g) for n in lengths]
    x, cu, mx = P.pack_batch(seqs, "cuda")
    xc, cuc, mxc = O.pack_batch(seqs, "cpu")
    assert x.is_cuda and cu.is_cuda and cu.dtype == torch.int32
    assert torch.equal(x.cpu(), xc) and torch.equal(cu.cpu(), cuc) and mx == mxc
    # the produced format drives the varlen op: each packed sequence equals the same sequence run alone
    H, D, R = 2, 64, 16
    T = int(cu[-1])
    q, k, v = (torch.randn(T, H, D, generator=g).bfloat16().cuda() for _ in range(3))
    rq, rk = ((torch.randn(T, H, R, generator=g) * 0.25).bfloat16().cuda() for _ in range(2))
    gs = torch.ones(H, device="cuda")
    o = flash_naylis_attn(q, k, v, rq, rk, gs, is_causal=True, cu_seqlens_q=cu, cu_seqlens_k=cu,
                          max_seqlen_q=mx, max_seqlen_k=mx)
    offs = cu.tolist()
    for i in range(len(lengths)):
        a, b = offs[i], offs[i + 1]
        one = lambda t: t[a:b].transpose(0, 1).unsqueeze(0)
        od = flash_naylis_attn(one(q), one(k), one(v), one(rq), one(rk), gs, is_causal=True)
        torch.testing.assert_close(o[a:b].float(), od[0].transpose(0, 1).float(), atol=2e-2, rtol=2e-2)
