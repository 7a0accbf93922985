"""GPU parity of the KV-cache decode kernel (through the C ABI via
fna2_b200.decode) against the decode oracle, the cache append, packed caches,
key splits, and agreement with the prefill op's last row."""
import math

import pytest
import torch

from oracle import decode_oracle as DO

pytestmark = pytest.mark.gpu

REL_L2 = 1e-2
MAX_ABS = 2e-2


def _close(name, got, ref):
    got, ref = got.float().cpu(), ref.float().cpu()
    assert torch.isfinite(got).all(), f"{name}: non-finite"
    rel = ((got - ref).norm() / ref.norm().clamp_min(1e-30)).item()
    mab = (got - ref).abs().max().item()
    assert rel < REL_L2 and mab < MAX_ABS * max(1.0, ref.abs().max().item()), f"{name}: rel {rel:.3g} max {mab:.3g}"


def _inputs(lens, H, H_KV, H_G, D, R, cap, seed, append):
    g = torch.Generator().manual_seed(seed)
    B = len(lens)
    q = torch.randn(B, H, D, generator=g).bfloat16()
    kc = torch.randn(B, cap, H_KV, D, generator=g).bfloat16()
    vc = torch.randn(B, cap, H_KV, D, generator=g).bfloat16()
    rq = (torch.randn(B, H_G, R, generator=g) * 0.5).bfloat16() if H_G else None
    rkc = (torch.randn(B, cap, H_G, R, generator=g) * 0.5).bfloat16() if H_G else None
    gs = torch.randn(H_G, generator=g) if H_G else None
    new = None
    if append:
        new = (torch.randn(B, H_KV, D, generator=g).bfloat16(), torch.randn(B, H_KV, D, generator=g).bfloat16(),
               (torch.randn(B, H_G, R, generator=g) * 0.5).bfloat16() if H_G else None)
    return q, kc, vc, rq, rkc, gs, new


def _cuda(t):
    return None if t is None else t.cuda()


@pytest.mark.parametrize("H,H_KV,H_G,D,R", [(4, 4, 4, 128, 16), (8, 2, 5, 64, 32), (24, 1, 24, 128, 16),
                                             (6, 3, 0, 64, 16)])
@pytest.mark.parametrize("append", [False, True])
def test_decode_vs_oracle(H, H_KV, H_G, D, R, append):
    from fna2_b200.decode import flash_naylis_decode
    lens = [0, 1, 17, 300, 1000] if not append else [0, 5, 64, 999]
    cap = max(lens) + 1
    q, kc, vc, rq, rkc, gs, new = _inputs(lens, H, H_KV, H_G, D, R, cap, 7 + H + D, append)
    kc_d, vc_d, rkc_d = kc.cuda(), vc.cuda(), _cuda(rkc)
    kw = {}
    if append:
        kw = dict(k=new[0].cuda(), v=new[1].cuda(), r_k=_cuda(new[2]))
    seq = torch.tensor(lens, dtype=torch.int32, device="cuda")
    out, lse = flash_naylis_decode(q.cuda(), kc_d, vc_d, seq, _cuda(rq), rkc_d, _cuda(gs), return_lse=True, **kw)
    okw = dict(k_new=new[0], v_new=new[1], rk_new=new[2]) if append else {}
    ro, rl = DO.decode(q, kc, vc, lens, rq, rkc, gs, **okw)
    nonempty = torch.tensor([(n + append) > 0 for n in lens])
    _close("out", out, ro)
    assert (out[~nonempty.cuda()] == 0).all()
    _close("lse", lse[nonempty.cuda()], rl[nonempty])
    if append:  # the new rows landed in slot lens[b], bit for bit; nothing else moved
        for b, n in enumerate(lens):
            assert torch.equal(kc_d[b, n].cpu(), new[0][b]) and torch.equal(vc_d[b, n].cpu(), new[1][b])
            if H_G:
                assert torch.equal(rkc_d[b, n].cpu(), new[2][b])
        mask = torch.ones(len(lens), cap, dtype=torch.bool)
        for b, n in enumerate(lens):
            mask[b, n] = False
        assert torch.equal(kc_d.cpu()[mask], kc[mask]) and torch.equal(vc_d.cpu()[mask], vc[mask])


@pytest.mark.parametrize("splits", [1, 3, 17])
def test_forced_splits_agree(splits):
    from fna2_b200.decode import flash_naylis_decode
    lens = [700, 33, 2048]
    q, kc, vc, rq, rkc, gs, _ = _inputs(lens, 8, 4, 8, 128, 16, 2048, 3, False)
    seq = torch.tensor(lens, dtype=torch.int32, device="cuda")
    out = flash_naylis_decode(q.cuda(), kc.cuda(), vc.cuda(), seq, rq.cuda(), rkc.cuda(), gs.cuda(), num_splits=splits)
    ro, _ = DO.decode(q, kc, vc, lens, rq, rkc, gs)
    _close(f"out splits={splits}", out, ro)


def test_packed_cache_with_offsets():
    from fna2_b200.decode import flash_naylis_decode
    lens, H, H_KV, D, R = [10, 0, 257], 4, 2, 128, 16
    q, kc, vc, rq, rkc, gs, new = _inputs(lens, H, H_KV, H, D, R, 258, 11, True)
    cap = 258
    offs = [0, cap, 2 * cap]
    pk = torch.cat([kc[b] for b in range(3)]).cuda()
    pv = torch.cat([vc[b] for b in range(3)]).cuda()
    prk = torch.cat([rkc[b] for b in range(3)]).cuda()
    out = flash_naylis_decode(q.cuda(), pk, pv, torch.tensor(lens, dtype=torch.int32, device="cuda"), rq.cuda(), prk,
                              gs.cuda(), k=new[0].cuda(), v=new[1].cuda(), r_k=new[2].cuda(),
                              cache_offsets=torch.tensor(offs, dtype=torch.int32, device="cuda"), capacity=cap)
    ro, _ = DO.decode(q, kc, vc, lens, rq, rkc, gs, k_new=new[0], v_new=new[1], rk_new=new[2])
    _close("out", out, ro)
    for b, n in enumerate(lens):
        assert torch.equal(pk[offs[b] + n].cpu(), new[0][b])


def test_decode_matches_prefill_last_row():
    """Each sequence's last token decoded against the cache of its first L tokens
    equals row L of the varlen prefill op over the whole sequence."""
    from fna2_b200.decode import NaylisKVCache
    from fna2_b200.flash_naylis_attn import flash_naylis_attn
    g = torch.Generator().manual_seed(5)
    H, H_KV, D, R = 8, 4, 128, 16
    lens = [1, 130, 511]
    T = sum(lens)
    q, k, v = (torch.randn(T, h, D, generator=g).bfloat16().cuda() for h in (H, H_KV, H_KV))
    rq, rk = ((torch.randn(T, H, R, generator=g) * 0.5).bfloat16().cuda() for _ in range(2))
    gs = torch.randn(H, generator=g).cuda()
    cu = torch.tensor([0, 1, 131, 642], dtype=torch.int32, device="cuda")
    o_pre = flash_naylis_attn(q, k, v, rq, rk, gs, is_causal=True, cu_seqlens_q=cu, cu_seqlens_k=cu,
                              max_seqlen_q=max(lens), max_seqlen_k=max(lens))
    cache = NaylisKVCache(3, 600, H_KV, D, graph_heads=H, rank=R)
    offs = cu.tolist()
    for b, n in enumerate(lens):
        a = offs[b]
        cache.k[b, :n - 1] = k[a:a + n - 1]
        cache.v[b, :n - 1] = v[a:a + n - 1]
        cache.r_k[b, :n - 1] = rk[a:a + n - 1]
    cache.seqlens.copy_(torch.tensor([n - 1 for n in lens], dtype=torch.int32))
    last = [offs[b + 1] - 1 for b in range(3)]
    out = cache.step(q[last], k[last], v[last], rq[last], rk[last], gs)
    _close("decode vs prefill", out, o_pre[last])
    assert cache.seqlens.tolist() == lens


def test_bad_length_sets_status_and_writes_zeros():
    from fna2_b200 import _lib
    from fna2_b200.decode import flash_naylis_decode
    lib = _lib.load()
    lib.fna2_device_status(1)
    q, kc, vc, rq, rkc, gs, _ = _inputs([4, 4], 2, 2, 2, 64, 16, 8, 1, False)
    seq = torch.tensor([4, 9], dtype=torch.int32, device="cuda")  # 9 > capacity 8
    out = flash_naylis_decode(q.cuda(), kc.cuda(), vc.cuda(), seq, rq.cuda(), rkc.cuda(), gs.cuda())
    assert lib.fna2_device_status(1) == 601
    assert (out[1] == 0).all()
    assert lib.fna2_device_status(0) == 0


def test_reference_cache_layout_and_largest_head_block():
    """Caches in the reference's [B, H_KV, S, D] layout passed as .transpose(1, 2),
    16 graph heads per KV head at rank 32 (the largest shared-memory layout)."""
    from fna2_b200.decode import flash_naylis_decode
    lens, H, H_KV, D, R = [5, 300, 64], 32, 2, 128, 32
    cap = 320
    q, kc, vc, rq, rkc, gs, new = _inputs(lens, H, H_KV, H, D, R, cap, 23, True)
    k_ref = kc.transpose(1, 2).contiguous().cuda()  # [B, H_KV, S, D] storage
    v_ref = vc.transpose(1, 2).contiguous().cuda()
    seq = torch.tensor(lens, dtype=torch.int32, device="cuda")
    out = flash_naylis_decode(q.cuda(), k_ref.transpose(1, 2), v_ref.transpose(1, 2), seq, rq.cuda(), rkc.cuda(),
                              gs.cuda(), k=new[0].cuda(), v=new[1].cuda(), r_k=new[2].cuda())
    ro, _ = DO.decode(q, kc, vc, lens, rq, rkc, gs, k_new=new[0], v_new=new[1], rk_new=new[2])
    _close("out", out, ro)
    for b, n in enumerate(lens):
        assert torch.equal(k_ref[b, :, n].cpu(), new[0][b])
