"""Pin the CPU oracle against golden vectors produced by the reference itself
(its fp32 eager path and its Triton kernels under the CPU interpreter)."""
import pytest
import torch

from oracle import fna2_oracle as O
from tests.golden_io import CASES, load

GRADS = ["dq", "dk", "dv", "drq", "drk", "dgs"]


def _oracle(rec, inputs, dtype=torch.float64):
    q, k, v, rq, rk, gs, do, cu = inputs
    c = lambda t: t.to(dtype)
    if rec["kind"] == "dense":
        out, lse = O.attention_fwd(c(q), c(k), c(v), c(rq), c(rk), c(gs), rec["scale"], rec["causal"])
        grads = O.attention_bwd(c(q), c(k), c(v), c(rq), c(rk), c(gs), out, lse, c(do), rec["scale"],
                                rec["causal"])
    else:
        out, lse = O.varlen_fwd(c(q), c(k), c(v), c(rq), c(rk), c(gs), cu, cu, rec["scale"])
        grads = O.varlen_bwd(c(q), c(k), c(v), c(rq), c(rk), c(gs), out, lse, c(do), cu, cu, rec["scale"])
    return out, lse, dict(zip(GRADS, grads))


@pytest.mark.parametrize("name", CASES)
def test_oracle_matches_reference(name):
    rec, inputs = load(name)
    out, lse, grads = _oracle(rec, inputs)
    e = O.errors(rec["out"], out)
    assert e["rel_l2"] < 2e-6 and e["max_abs"] < 2e-5, e
    if "lse" in rec:
        e = O.errors(rec["lse"], lse)
        assert e["max_abs"] < 2e-5, e
    for g in GRADS:
        e = O.errors(rec[g], grads[g])
        assert e["rel_l2"] < 5e-6, (g, e)


@pytest.mark.parametrize("name", CASES)
def test_blocked_oracle_matches_reference(name):
    """The blocked restatement used by the full-size GPU checks
    (oracle.fna2_oracle.blocked_sequence, fp32) reproduces the same golden
    vectors, with a block size that splits every case into several blocks."""
    rec, (q, k, v, rq, rk, gs, do, cu) = load(name)
    if rec["kind"] == "dense":
        seqs = [(b, None) for b in range(q.shape[0])]
        sl = lambda t, b, _: t[b].transpose(0, 1)            # [H, S, X] -> [S, H, X]
        put = lambda t, b, _: t[b].transpose(0, 1)
    else:
        seqs = [(cu[i], cu[i + 1]) for i in range(len(cu) - 1)]
        sl = lambda t, a, b: t[a:b]
        put = sl
    dgs = torch.zeros_like(gs, dtype=torch.float64)
    for a, b in seqs:
        res = O.blocked_sequence(sl(q, a, b), sl(k, a, b), sl(v, a, b), sl(rq, a, b), sl(rk, a, b), gs,
                                 sl(do, a, b), rec["scale"], rec["causal"], block=24)
        for n in ("out", "dq", "dk", "dv", "drq", "drk"):
            ref = put(rec[n], a, b)
            if ref.numel():
                e = O.errors(ref, res[n])
                assert e["max_abs"] < 5e-5 and (e["rel_l2"] < 5e-6 or ref.abs().max() < 1e-3), (n, a, e)
        dgs += res["dgs"]
    e = O.errors(rec["dgs"], dgs)
    assert e["rel_l2"] < 5e-6, e


def test_oracle_autograd_agrees_with_explicit_backward():
    q, k, v, rq, rk, gs, do = O.make_dense_inputs(1, 4, 70, 32, 16, H_KV=2, H_G=2, seed=3, gs_value="randn")
    ts = [t.double().requires_grad_(True) for t in (q, k, v, rq, rk, gs)]
    out, lse = O.attention_fwd(*ts, 0.2, True)
    out.backward(do.double())
    ex = O.attention_bwd(*[t.detach() for t in ts], out.detach(), lse.detach(), do.double(), 0.2, True)
    for t, g in zip(ts, ex):
        # the +1e-6 in O = acc/(l+1e-6) perturbs autograd by ~1e-6 relative
        assert torch.allclose(t.grad, g, rtol=1e-5, atol=1e-5)


def test_sdpa_restatement_matches_reference_eager_fixture():
    rec, (q, k, v, rq, rk, gs, do, _) = load("gqa_vanilla_sdpa")
    out = O.sdpa_reference(q, k, v, rq, rk, gs, rec["scale"], True)
    assert O.errors(rec["out"], out)["max_abs"] < 1e-5


def test_varlen_equals_per_sequence_dense():
    lengths = [5, 1, 17]
    q, k, v, rq, rk, gs, do, cu = O.make_varlen_inputs(lengths, 2, 16, 8, seed=9, gs_value="randn")
    out, lse = O.varlen_fwd(q.double(), k.double(), v.double(), rq.double(), rk.double(), gs.double(), cu, cu, 0.25)
    for i in range(len(lengths)):
        a, b = cu[i], cu[i + 1]
        v4 = lambda t: t[a:b].transpose(0, 1).unsqueeze(0).double()
        o, l = O.attention_fwd(v4(q), v4(k), v4(v), v4(rq), v4(rk), gs.double(), 0.25, True)
        assert torch.allclose(out[a:b], o[0].transpose(0, 1))


def test_gs_zero_is_plain_causal_attention():
    q, k, v, rq, rk, gs, do = O.make_dense_inputs(1, 2, 40, 16, 8, seed=7, gs_value=0.0)
    out, _ = O.attention_fwd(q.double(), k.double(), v.double(), rq.double(), rk.double(), gs.double(), 0.25, True)
    ref = torch.nn.functional.scaled_dot_product_attention(q.double(), k.double(), v.double(), is_causal=True, scale=0.25)
    assert (out - ref).abs().max() < 1e-5


def test_planted_error_is_detected():
    """A mistake planted in the oracle's output must fail the pinning bound."""
    rec, inputs = load("interp_dense_causal_d64")
    out, _, _ = _oracle(rec, inputs)
    out = out.clone()
    out[0, 0, 5, 3] += 1e-3
    assert O.errors(rec["out"], out)["max_abs"] > 2e-5
