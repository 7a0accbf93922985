"""Shared helpers of the GPU parity tests: run the CUDA op and the CPU oracle on
the same (bf16-exact) inputs and compare with the stated tolerance."""
import math

import torch

from oracle import fna2_oracle as O

# Tolerance (bf16 kernel vs fp32/fp64 oracle on identical bf16-representable
# inputs): relative L2 <= 1e-2 and max-abs <= 2e-2, the max-abs bound scaled by
# the tensor's magnitude when that exceeds 1 (bf16 carries 8 significant bits,
# so an element of size 4 is itself only representable to 1.6e-2).
REL_L2 = 1e-2
MAX_ABS = 2e-2

GRADS = ("dq", "dk", "dv", "drq", "drk", "dgs")


def check(name, ref, got, rel_l2=REL_L2, max_abs=MAX_ABS):
    ref = ref.detach().cpu()
    got = got.detach().float().cpu()
    e = O.errors(ref, got)
    bound = max_abs * max(1.0, e["ref_max"])
    assert math.isfinite(e["max_abs"]), f"{name}: non-finite values {e}"
    # relative L2 with a noise floor: a tensor whose true values are ~1e-6
    # (e.g. dQ of a single-token sequence, zero up to the +1e-6 normalisation)
    # is judged by max-abs alone
    floor = 1e-3 * math.sqrt(max(ref.numel(), 1))
    rel = (ref.double() - got.double()).norm().item() / max(ref.double().norm().item(), floor)
    e["rel_l2_floored"] = rel
    assert rel <= rel_l2 and e["max_abs"] <= bound, f"{name}: {e} (bound max_abs {bound:.3g})"
    return e


def run_cuda(q, k, v, rq, rk, gs, do, scale, causal, cu=None, max_seqlen=0, backward=True):
    """Call the drop-in op on CUDA copies; returns dict of CPU fp32 results."""
    from fna2_b200 import flash_naylis_attn
    dev = "cuda"
    t = [x.to(dev, torch.bfloat16).requires_grad_(backward) for x in (q, k, v, rq, rk)]
    g = gs.to(dev, torch.float32).requires_grad_(backward)
    kw = {}
    if cu is not None:
        cu_t = torch.tensor(cu, dtype=torch.int32, device=dev)
        kw = dict(cu_seqlens_q=cu_t, cu_seqlens_k=cu_t, max_seqlen_q=max_seqlen, max_seqlen_k=max_seqlen)
    out = flash_naylis_attn(*t, g, softmax_scale=scale, is_causal=causal, **kw)
    res = {"out": out.detach().float().cpu()}
    if backward:
        out.backward(do.to(dev, torch.bfloat16))
        for name, x in zip(GRADS, t + [g]):
            res[name] = x.grad.detach().float().cpu()
    return res


def run_oracle(q, k, v, rq, rk, gs, do, scale, causal, cu=None, dtype=torch.float64, backward=True):
    c = lambda x: x.to(dtype)
    if cu is None:
        out, lse = O.attention_fwd(c(q), c(k), c(v), c(rq), c(rk), c(gs), scale, causal)
        res = {"out": out, "lse": lse}
        if backward:
            g = O.attention_bwd(c(q), c(k), c(v), c(rq), c(rk), c(gs), out, lse, c(do), scale, causal)
            res.update(dict(zip(GRADS, g)))
    else:
        out, lse = O.varlen_fwd(c(q), c(k), c(v), c(rq), c(rk), c(gs), cu, cu, scale)
        res = {"out": out, "lse": lse}
        if backward:
            g = O.varlen_bwd(c(q), c(k), c(v), c(rq), c(rk), c(gs), out, lse, c(do), cu, cu, scale)
            res.update(dict(zip(GRADS, g)))
    return res


def compare(ref, got, names=("out",) + GRADS, label=""):
    errs = {}
    for n in names:
        if n in got and n in ref:
            if ref[n].numel() == 0:
                continue
            errs[n] = check(f"{label}{n}", ref[n], got[n])
    return errs
