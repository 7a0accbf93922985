"""The drop-in boundary as PyTorch custom ops (fna2::fwd, fna2::bwd) on a
GPU: torch.library.opcheck of both ops on dense and packed problems, and a
torch.compile(fullgraph=True) module that calls flash_naylis_attn giving the
eager results bit for bit."""
import math

import pytest
import torch

from oracle import fna2_oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True, scope="module")
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    import fna2_b200  # noqa: F401  (registers the ops)
    yield


def _dense(seed=0):
    q, k, v, rq, rk, gs, do = O.make_dense_inputs(2, 4, 200, 128, 16, H_KV=2, H_G=3, seed=seed, gs_value="randn")
    c = lambda t: t.cuda().bfloat16()
    return [c(q), c(k), c(v), c(rq), c(rk), gs.cuda(), c(do)], None


def _packed(seed=0):
    lengths = [70, 1, 200, 0, 129]
    q, k, v, rq, rk, gs, do, cu = O.make_varlen_inputs(lengths, 4, 64, 16, 2, 4, seed=seed, gs_value="randn")
    c = lambda t: t.cuda().bfloat16()
    return [c(q), c(k), c(v), c(rq), c(rk), gs.cuda(), c(do)], (torch.tensor(cu, dtype=torch.int32, device="cuda"),
                                                                max(lengths))


@pytest.mark.parametrize("mode", ["dense", "packed"])
def test_opcheck(mode):
    (q, k, v, rq, rk, gs, do), cu = _dense() if mode == "dense" else _packed()
    scale = 1.0 / math.sqrt(q.shape[-1])
    cu_t, msl = (cu if cu else (None, 0))
    fwd_args = (q, k, v, rq, rk, gs, scale, True, cu_t, cu_t, msl, msl)
    torch.library.opcheck(torch.ops.fna2.fwd.default, fwd_args)
    ins = [t.clone().requires_grad_(True) for t in (q, k, v, rq, rk, gs)]
    torch.library.opcheck(torch.ops.fna2.fwd.default, tuple(ins) + fwd_args[6:])
    out, lse = torch.ops.fna2.fwd(*fwd_args)
    torch.library.opcheck(torch.ops.fna2.bwd.default,
                          (do, q, k, v, rq, rk, gs, out, lse, scale, True, cu_t, cu_t, msl, msl))


@pytest.mark.parametrize("mode", ["dense", "packed"])
def test_compiled_module_matches_eager(mode):
    from fna2_b200 import flash_naylis_attn
    (q, k, v, rq, rk, gs, do), cu = _dense(1) if mode == "dense" else _packed(1)
    kw = {} if cu is None else dict(cu_seqlens_q=cu[0], cu_seqlens_k=cu[0], max_seqlen_q=cu[1], max_seqlen_k=cu[1])

    def f(q, k, v, rq, rk, gs):
        return flash_naylis_attn(q, k, v, rq, rk, gs, is_causal=True, **kw) * 2.0

    def run(fn):
        ts = [t.clone().requires_grad_(True) for t in (q, k, v, rq, rk, gs)]
        out = fn(*ts)
        out.backward(do)
        return [out.detach()] + [t.grad for t in ts]

    eager = run(f)
    torch._dynamo.reset()
    compiled = run(torch.compile(f, fullgraph=True))
    names = ("out", "dq", "dk", "dv", "drq", "drk", "dgs")
    for n, a, b in zip(names, eager, compiled):
        if n == "dgs":  # summed with fp32 atomics: equal up to summation order
            torch.testing.assert_close(a, b, rtol=1e-5, atol=1e-5)
        else:
            assert torch.equal(a, b), n
