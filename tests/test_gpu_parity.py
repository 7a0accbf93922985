"""GPU parity of the sm_100a kernels (through the C ABI) against the CPU oracle
and the reference's golden vectors."""
import math

import pytest
import torch

from oracle import fna2_oracle as O
from tests import parity
from tests.golden_io import CASES, load

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True, scope="module")
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from fna2_b200 import _lib
    _lib.load()
    yield
    assert _lib.load().fna2_device_status(1) == 0, "a kernel's bounded wait timed out"


@pytest.mark.parametrize("name", CASES)
def test_golden_vectors(name):
    """Kernel vs the reference's own outputs (eager fp32 path / Triton kernels in
    the CPU interpreter) on the fixture's bf16-exact inputs."""
    rec, (q, k, v, rq, rk, gs, do, cu) = load(name)
    msl = max(rec["lengths"]) if cu is not None else 0
    got = parity.run_cuda(q, k, v, rq, rk, gs, do, rec["scale"], rec["causal"], cu, msl)
    parity.compare({n: rec[n] for n in ("out",) + parity.GRADS}, got, label=name + ":")


DENSE = [
    # B, H, HKV, HG, S, D, r, causal, gs
    (1, 1, 1, 1, 1, 64, 16, True, "randn"),
    (1, 2, 2, 2, 63, 64, 16, True, "randn"),
    (1, 2, 1, 2, 64, 128, 16, True, "randn"),
    (2, 2, 2, 1, 65, 128, 32, True, "randn"),
    (1, 4, 2, 2, 127, 64, 8, True, "randn"),
    (1, 2, 2, 2, 129, 128, 16, False, "randn"),
    (1, 4, 1, 3, 300, 128, 24, True, "randn"),
    (2, 2, 2, 0, 256, 128, 16, True, None),
    (1, 3, 3, 3, 257, 64, 32, False, 1.0),
    (1, 2, 2, 2, 384, 128, 16, True, 0.0),
]


@pytest.mark.parametrize("B,H,HKV,HG,S,D,r,causal,gs", DENSE)
def test_dense_vs_oracle(B, H, HKV, HG, S, D, r, causal, gs):
    q, k, v, rq, rk, g, do = O.make_dense_inputs(B, H, S, D, r, HKV, HG, seed=S + D + r, gs_value=gs)
    q, k, v, rq, rk, do = O.bf16_round(q, k, v, rq, rk, do)
    scale = 1.0 / math.sqrt(D)
    got = parity.run_cuda(q, k, v, rq, rk, g, do, scale, causal)
    ref = parity.run_oracle(q, k, v, rq, rk, g, do, scale, causal)
    parity.compare(ref, got)


VARLEN = [
    # lengths, H, HKV, HG, D, r
    ([1], 2, 2, 2, 64, 16),
    ([5, 0, 130, 1, 64], 2, 1, 2, 128, 16),
    ([129, 17, 256, 300], 4, 2, 2, 128, 32),
    ([64, 63, 65, 127, 128, 129], 2, 2, 1, 64, 8),
]


@pytest.mark.parametrize("lengths,H,HKV,HG,D,r", VARLEN)
def test_varlen_vs_oracle(lengths, H, HKV, HG, D, r):
    q, k, v, rq, rk, g, do, cu = O.make_varlen_inputs(lengths, H, D, r, HKV, HG, seed=len(lengths) + D,
                                                      gs_value="randn")
    q, k, v, rq, rk, do = O.bf16_round(q, k, v, rq, rk, do)
    scale = 1.0 / math.sqrt(D)
    got = parity.run_cuda(q, k, v, rq, rk, g, do, scale, True, cu, max(lengths))
    ref = parity.run_oracle(q, k, v, rq, rk, g, do, scale, True, cu)
    parity.compare(ref, got)


def test_varlen_max_seqlen_unknown():
    """max_seqlen = 0 (the signature default) is bounded by the token count."""
    lengths = [40, 200]
    q, k, v, rq, rk, g, do, cu = O.make_varlen_inputs(lengths, 2, 64, 16, seed=11, gs_value="randn")
    q, k, v, rq, rk, do = O.bf16_round(q, k, v, rq, rk, do)
    got = parity.run_cuda(q, k, v, rq, rk, g, do, 0.125, True, cu, 0)
    ref = parity.run_oracle(q, k, v, rq, rk, g, do, 0.125, True, cu)
    parity.compare(ref, got)


def test_noncontiguous_dense_layout():
    """q/k/v as NaylisAttention builds them: view(B,S,H,D).transpose(1,2)
    (attention_fna2.py:404-406) -- strided, consumed without copies."""
    from fna2_b200 import flash_naylis_attn
    B, S, H, D, r = 2, 200, 4, 128, 16
    torch.manual_seed(0)
    x = torch.randn(B, S, 3, H, D)
    q, k, v = (x[:, :, i].transpose(1, 2) for i in range(3))
    rq = torch.randn(B, H, S, r) / 4
    rk = torch.randn(B, H, S, r) / 4
    g = torch.randn(H)
    q, k, v, rq, rk = O.bf16_round(q.contiguous(), k.contiguous(), v.contiguous(), rq, rk)
    xs = torch.stack([q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2)], dim=2).cuda().bfloat16()
    qs, ks, vs = (xs[:, :, i].transpose(1, 2) for i in range(3))
    assert not qs.is_contiguous()
    out = flash_naylis_attn(qs, ks, vs, rq.cuda().bfloat16(), rk.cuda().bfloat16(), g.cuda(), is_causal=True)
    ref = O.attention_fwd(q.double(), k.double(), v.double(), rq.double(), rk.double(), g.double(),
                          1 / math.sqrt(D), True)[0]
    parity.check("strided out", ref, out)


def test_gs_zero_matches_plain_causal_sdpa():
    """graph_scale = 0 reduces to plain causal attention (validate_fna2.py:341-369)."""
    from fna2_b200 import flash_naylis_attn
    q, k, v, rq, rk, g, do = O.make_dense_inputs(2, 4, 256, 64, 32, H_KV=2, H_G=4, seed=7, gs_value=0.0)
    q, k, v, rq, rk = O.bf16_round(q, k, v, rq, rk)
    out = flash_naylis_attn(*(t.cuda().bfloat16() for t in (q, k, v, rq, rk)), g.cuda(), is_causal=True)
    ke, ve = k.repeat_interleave(2, 1), v.repeat_interleave(2, 1)
    ref = torch.nn.functional.scaled_dot_product_attention(q.double(), ke.double(), ve.double(), is_causal=True)
    parity.check("gs0", ref, out)


@pytest.mark.parametrize("cfg", ["cfg2_slices", "cfg4_slice"])
def test_full_size_head_slices(cfg):
    """BASELINE configs at full size on the GPU; (batch, head) slices, which are
    independent, are checked against the fp32 oracle."""
    if cfg == "cfg2_slices":
        B, H, S, D, r = 8, 16, 2048, 128, 16
        picks = [(0, 0), (7, 15)]
    else:
        B, H, S, D, r = 1, 32, 32768, 128, 32
        picks = [(0, 31)]
    q, k, v, rq, rk, g, do = O.make_dense_inputs(B, H, S, D, r, seed=1, gs_value="randn")
    from fna2_b200 import flash_naylis_attn
    dev = [t.cuda().bfloat16().requires_grad_(True) for t in (q, k, v, rq, rk)]
    gd = g.cuda().requires_grad_(True)
    out = flash_naylis_attn(*dev, gd, is_causal=True)
    dd = do.cuda().bfloat16()
    out.backward(dd)
    scale = 1 / math.sqrt(D)
    Sc = S if cfg == "cfg2_slices" else 4096  # the long-context oracle checks the first 4096 rows
    for b, h in picks:
        sl = lambda t: t[b:b + 1, h:h + 1, :Sc].detach().float().cpu()
        ref = parity.run_oracle(sl(dev[0]), sl(dev[1]), sl(dev[2]), sl(dev[3]), sl(dev[4]), g[h:h + 1],
                                sl(dd), scale, True, dtype=torch.float32, backward=(cfg == "cfg2_slices"))
        parity.check(f"{cfg} out[{b},{h}]", ref["out"], sl(out))
        if cfg == "cfg2_slices":
            for n, t in (("dq", dev[0]), ("dk", dev[1]), ("dv", dev[2]), ("drq", dev[3]), ("drk", dev[4])):
                parity.check(f"{cfg} {n}[{b},{h}]", ref[n], t.grad[b:b + 1, h:h + 1].float().cpu())
