"""Parity at the sizes the benchmark numbers are quoted on.

BASELINE config 5 (the whole 512-sequence packed batch, T = 1.8 M tokens,
H = 32, the metric's workload), config 4 (one 32768-row sequence, H = 32,
r = 32: every row of every head), config 3 (16 packed sequences) and config 2
(dense B = 8, L = 2048) go through the public op, forward and backward, and
are compared with the blocked fp32 restatement of the oracle
(``oracle.fna2_oracle.blocked_sequence``, pinned to the reference's golden
vectors by tests/test_oracle.py) run on the same GPU with TF32 off.  Errors are
accumulated over whole tensors (relative L2 over every element, max-abs over
every element) and recorded per tensor in ``tests.parity.REPORT``.
"""
import math

import pytest
import torch

from fna2_b200 import partition as PT
from oracle import fna2_oracle as O
from tests import parity

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True, scope="module")
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from fna2_b200 import _lib
    _lib.load()
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False  # the oracle computes in true fp32
    yield
    torch.backends.cuda.matmul.allow_tf32 = prev
    assert _lib.load().fna2_device_status(1) == 0, "a kernel recorded a device status"


class Acc:
    """Whole-tensor error figures accumulated from per-sequence slices."""

    def __init__(self):
        self.d = {}

    def add(self, name, ref, got):
        ref, got = ref.double(), got.double()
        diff = ref - got
        a = self.d.setdefault(name, [0.0, 0.0, 0.0, 0.0])
        a[0] += diff.square().sum().item()
        a[1] += ref.square().sum().item()
        a[2] = max(a[2], diff.abs().max().item() if diff.numel() else 0.0)
        a[3] = max(a[3], ref.abs().max().item() if ref.numel() else 0.0)

    def assert_ok(self, label):
        bad = []
        for name, (d2, r2, mx, rmax) in self.d.items():
            rel = math.sqrt(d2 / max(r2, 1e-300))
            flat = mx <= parity.MAX_ABS
            bound = parity.MAX_ABS if flat else parity.MAX_ABS * max(1.0, rmax)
            parity.record(f"{label} {name}", mx, rel, rmax, bound, "flat" if flat else "scaled by max|ref|")
            if not (rel <= parity.REL_L2 and mx <= bound):
                bad.append((name, rel, mx, bound))
        assert not bad, f"{label}: {bad}"


def _rand(shape, gen, scale=None):
    t = torch.randn(shape, device="cuda", dtype=torch.bfloat16, generator=gen)
    return t if scale is None else t.mul_(scale)


def _packed_inputs(lengths, H, D, r, seed, gs_randn):
    g = torch.Generator(device="cuda").manual_seed(seed)
    T = sum(lengths)
    q, k, v = (_rand((T, H, D), g) for _ in range(3))
    rq, rk = (_rand((T, H, r), g, r ** -0.5) for _ in range(2))
    do = _rand((T, H, D), g)
    gs = torch.randn(H, device="cuda", generator=g) if gs_randn else torch.ones(H, device="cuda")
    return q, k, v, rq, rk, gs, do


def _run_packed(q, k, v, rq, rk, gs, do, lengths):
    from fna2_b200 import flash_naylis_attn
    cu = PT.cu_seqlens(lengths)
    cu_t = torch.tensor(cu, dtype=torch.int32, device="cuda")
    leaves = [t.requires_grad_(True) for t in (q, k, v, rq, rk)]
    g = gs.clone().requires_grad_(True)
    out = flash_naylis_attn(*leaves, g, is_causal=True, cu_seqlens_q=cu_t, cu_seqlens_k=cu_t,
                            max_seqlen_q=max(lengths), max_seqlen_k=max(lengths))
    out.backward(do)
    torch.cuda.synchronize()
    grads = [t.grad for t in leaves] + [g.grad]
    for t in leaves:
        t.requires_grad_(False)
        t.grad = None
    return cu, out.detach(), grads


def _check_packed(label, q, k, v, rq, rk, gs, do, lengths, picks=()):
    """Whole batch against the blocked oracle; sequences in ``picks`` are also
    recorded on their own."""
    D = q.shape[-1]
    scale = 1.0 / math.sqrt(D)
    cu, out, (dq, dk, dv, drq, drk, dgs) = _run_packed(q, k, v, rq, rk, gs, do, lengths)
    acc = Acc()
    dgs_ref = torch.zeros(gs.shape[0], dtype=torch.float64, device="cuda")
    got = {"out": out, "dq": dq, "dk": dk, "dv": dv, "drq": drq, "drk": drk}
    for i, L in enumerate(lengths):
        a, b = cu[i], cu[i + 1]
        block = 256 if L > 4096 else 1024
        res = O.blocked_sequence(q[a:b], k[a:b], v[a:b], rq[a:b], rk[a:b], gs, do[a:b], scale, True, block=block)
        one = Acc() if i in picks else None
        for n, t in got.items():
            acc.add(n, res[n], t[a:b])
            if one is not None:
                one.add(n, res[n], t[a:b])
        if one is not None:
            one.assert_ok(f"{label} seq {i} (L={L})")
        dgs_ref += res["dgs"]
        del res
    acc.assert_ok(f"{label} all {len(lengths)} seqs")
    parity.check(f"{label} dgs", dgs_ref.cpu(), dgs)


def test_cfg5_whole_batch():
    """BASELINE config 5 exactly as bench.py runs it (lengths log-uniform in
    [128, 16384], seed 0; H = 32, D = 128, r = 16, gs = 1): every sequence,
    O and all six gradients.  The longest sequence, one near 4096, the shortest
    ones and the first and last of the pack are also judged on their own."""
    lengths = PT.loguniform_lengths(512, 128, 16384, seed=0)
    q, k, v, rq, rk, gs, do = _packed_inputs(lengths, 32, 128, 16, seed=5, gs_randn=False)
    order = sorted(range(len(lengths)), key=lambda i: lengths[i])
    near4k = min(range(len(lengths)), key=lambda i: abs(lengths[i] - 4096))
    picks = {order[-1], near4k, order[0], order[1], order[2], 0, len(lengths) - 1}
    _check_packed("cfg5", q, k, v, rq, rk, gs, do, lengths, picks)


def test_cfg3_whole_batch():
    """16 sequences, lengths uniform-int in [64, 4096]
    (seed 0), H = 16, D = 128, r = 16, gs ~ N(0, 1)."""
    lengths = PT.uniform_int_lengths(16, 64, 4096, seed=0)
    q, k, v, rq, rk, gs, do = _packed_inputs(lengths, 16, 128, 16, seed=3, gs_randn=True)
    _check_packed("cfg3", q, k, v, rq, rk, gs, do, lengths, picks={0, 15})


def _check_dense(label, B, H, S, D, r, seed, head_chunk):
    from fna2_b200 import flash_naylis_attn
    g = torch.Generator(device="cuda").manual_seed(seed)
    q, k, v = (_rand((B, H, S, D), g) for _ in range(3))
    rq, rk = (_rand((B, H, S, r), g, r ** -0.5) for _ in range(2))
    do = _rand((B, H, S, D), g)
    gs = torch.randn(H, device="cuda", generator=g)
    leaves = [t.requires_grad_(True) for t in (q, k, v, rq, rk)]
    gl = gs.clone().requires_grad_(True)
    out = flash_naylis_attn(*leaves, gl, is_causal=True)
    out.backward(do)
    torch.cuda.synchronize()
    got = dict(zip(("out", "dq", "dk", "dv", "drq", "drk"), [out.detach()] + [t.grad for t in leaves]))
    scale = 1.0 / math.sqrt(D)
    acc = Acc()
    dgs_ref = torch.zeros(H, dtype=torch.float64, device="cuda")
    tr = lambda t, b, h0: t.detach()[b, h0:h0 + head_chunk].transpose(0, 1)  # [S, hc, X]
    for b in range(B):
        for h0 in range(0, H, head_chunk):
            res = O.blocked_sequence(tr(q, b, h0), tr(k, b, h0), tr(v, b, h0), tr(rq, b, h0), tr(rk, b, h0),
                                     gs[h0:h0 + head_chunk], tr(do, b, h0), scale, True, block=256)
            for n, t in got.items():
                acc.add(n, res[n], tr(t, b, h0))
            dgs_ref[h0:h0 + head_chunk] += res["dgs"]
    acc.assert_ok(f"{label} all rows, all heads")
    parity.check(f"{label} dgs", dgs_ref.cpu(), gl.grad)


def test_cfg4_long_context_all_rows():
    """B = 1, H = 32, L = 32768, r = 32, causal: every one
    of the 32768 rows of all 32 heads, forward and the full backward."""
    _check_dense("cfg4", 1, 32, 32768, 128, 32, seed=4, head_chunk=8)


def test_cfg2_dense_all():
    """B = 8, H = 16, L = 2048, r = 16, causal, every
    (batch, head)."""
    _check_dense("cfg2", 8, 16, 2048, 128, 16, seed=2, head_chunk=16)


def test_packed_equals_per_sequence_calls():
    """The reference's T3b check (validate_fna2.py:248-334) made exact: a packed
    batch gives the same O and per-sequence gradients as one dense call per
    sequence through the same op, bit for bit (both go through the same tiles
    in the same order); d_graph_scale is the sum of the per-sequence ones up to
    fp32 summation order."""
    from fna2_b200 import flash_naylis_attn
    lengths = [300, 1, 4096, 129, 2000, 64]
    H, HKV, HG, D, r = 8, 4, 6, 128, 16
    g = torch.Generator(device="cuda").manual_seed(17)
    T = sum(lengths)
    q = _rand((T, H, D), g)
    k, v = _rand((T, HKV, D), g), _rand((T, HKV, D), g)
    rq, rk = _rand((T, HG, r), g, r ** -0.5), _rand((T, HG, r), g, r ** -0.5)
    do = _rand((T, H, D), g)
    gs = torch.randn(HG, device="cuda", generator=g)
    cu, out, grads = _run_packed(q, k, v, rq, rk, gs, do, lengths)
    dgs_sum = torch.zeros(HG, device="cuda")
    for i in range(len(lengths)):
        a, b = cu[i], cu[i + 1]
        d4 = lambda t: t[a:b].transpose(0, 1).unsqueeze(0).detach().requires_grad_(True)
        ts = [d4(t) for t in (q, k, v, rq, rk)]
        gl = gs.clone().requires_grad_(True)
        o = flash_naylis_attn(*ts, gl, is_causal=True)
        o.backward(do[a:b].transpose(0, 1).unsqueeze(0))
        back = lambda t: t[0].transpose(0, 1)
        assert torch.equal(back(o.detach()), out[a:b]), f"seq {i}: out differs"
        for n, t, gp in zip(("dq", "dk", "dv", "drq", "drk"), ts, grads[:5]):
            assert torch.equal(back(t.grad), gp[a:b]), f"seq {i}: {n} differs"
        dgs_sum += gl.grad
    torch.testing.assert_close(grads[5], dgs_sum, rtol=2e-5, atol=1e-5)


def test_varlen_distinct_q_and_k_lengths():
    """cu_seqlens_q != cu_seqlens_k (the reference's varlen kernels read both,
    flash_naylis_attn.py:249-255): causal on local positions, top-left aligned;
    includes a sequence with no query rows and one with a single key."""
    lq = [100, 300, 5, 0, 64, 129]
    lk = [250, 120, 5, 10, 1, 200]
    H, HKV, HG, D, r = 4, 2, 3, 128, 16
    cuq, cuk = PT.cu_seqlens(lq), PT.cu_seqlens(lk)
    gen = torch.Generator().manual_seed(23)
    q = torch.randn(cuq[-1], H, D, generator=gen)
    k, v = torch.randn(cuk[-1], HKV, D, generator=gen), torch.randn(cuk[-1], HKV, D, generator=gen)
    rq = torch.randn(cuq[-1], HG, r, generator=gen) / 4
    rk = torch.randn(cuk[-1], HG, r, generator=gen) / 4
    do = torch.randn(cuq[-1], H, D, generator=gen)
    gs = torch.randn(HG, generator=gen)
    q, k, v, rq, rk, do = O.bf16_round(q, k, v, rq, rk, do)
    scale = 1.0 / math.sqrt(D)
    got = parity.run_cuda(q, k, v, rq, rk, gs, do, scale, True, cuq, max(lq), cu_k=cuk, max_seqlen_k=max(lk))
    ref = parity.run_oracle(q, k, v, rq, rk, gs, do, scale, True, cuq, cu_k=cuk)
    parity.compare(ref, got, label="cu_q!=cu_k ")


def test_varlen_many_sequences_tile_tables():
    """More than 3 x 128 packed sequences, so that the pre-pass builds both tile
    tables across several 128-sequence scan chunks (the running offset carried
    from chunk to chunk): short lengths with empty, 1-tile and multi-tile
    sequences mixed."""
    import random
    rnd = random.Random(41)
    choices = [0, 0, 1, 7, 64, 100, 127, 128, 129, 200, 256, 257, 400]
    lengths = [rnd.choice(choices) for _ in range(420)]
    H, HKV, HG, D, r = 2, 2, 1, 128, 16
    q, k, v, rq, rk, g, do, cu = O.make_varlen_inputs(lengths, H, D, r, HKV, HG, seed=42, gs_value="randn")
    q, k, v, rq, rk, do = O.bf16_round(q, k, v, rq, rk, do)
    scale = 1.0 / math.sqrt(D)
    got = parity.run_cuda(q, k, v, rq, rk, g, do, scale, True, cu, max(lengths))
    ref = parity.run_oracle(q, k, v, rq, rk, g, do, scale, True, cu)
    parity.compare(ref, got, label="420 seqs ")


@pytest.mark.parametrize("case", ["past_end", "negative_length", "negative_start", "over_max_seqlen"])
def test_invalid_cu_seqlens_reported_and_skipped(case):
    """A packed sequence whose cu_seqlens entries are inconsistent is skipped by
    the kernels before any access and reported through the device status (621
    forward, 622 backward); the other sequences are still exact.  The
    reference does not check cu_seqlens at all."""
    from fna2_b200 import _lib, flash_naylis_attn
    lib = _lib.load()
    lengths = [100, 200, 150]
    T = sum(lengths)
    cu, msl, bad = [0, 100, 300, 450], 200, None
    if case == "past_end":
        cu, bad = [0, 100, 300, 460], 2
    elif case == "negative_length":
        cu, bad = [0, 100, 300, 250], 2
    elif case == "negative_start":
        cu, bad = [-8, 100, 300, 450], 0
    else:
        msl, bad = 180, 1
    H, D, r = 2, 64, 16
    q, k, v, rq, rk, gs, do, _ = O.make_varlen_inputs(lengths, H, D, r, seed=31, gs_value="randn")
    q, k, v, rq, rk, do = O.bf16_round(q, k, v, rq, rk, do)
    dev = [t.cuda().bfloat16().requires_grad_(True) for t in (q, k, v, rq, rk)]
    g = gs.cuda().requires_grad_(True)
    cu_t = torch.tensor(cu, dtype=torch.int32, device="cuda")
    assert lib.fna2_device_status(1) == 0
    out = flash_naylis_attn(*dev, g, is_causal=True, cu_seqlens_q=cu_t, cu_seqlens_k=cu_t, max_seqlen_q=msl,
                            max_seqlen_k=msl)
    assert lib.fna2_device_status(1) == 621
    out.backward(do.cuda().bfloat16())
    assert lib.fna2_device_status(1) == 622
    scale = 1.0 / math.sqrt(D)
    for i in range(3):
        if i == bad:
            continue
        a, b = cu[i], cu[i + 1]
        s4 = lambda t: t[a:b].transpose(0, 1).unsqueeze(0).double()
        o_ref, lse = O.attention_fwd(s4(q), s4(k), s4(v), s4(rq), s4(rk), gs.double(), scale, True)
        gr = O.attention_bwd(s4(q), s4(k), s4(v), s4(rq), s4(rk), gs.double(), o_ref, lse, s4(do), scale, True)
        back = lambda t: t[0].transpose(0, 1)
        parity.check(f"{case} seq {i} out", back(o_ref), out.detach()[a:b])
        for n, ref, t in zip(("dq", "dk", "dv", "drq", "drk"), gr, dev):
            parity.check(f"{case} seq {i} {n}", back(ref), t.grad[a:b])
