"""Shared helpers of the GPU parity tests: run the CUDA op and the CPU oracle on
the same (bf16-exact) inputs and compare with the stated tolerance."""
import math

import torch

from oracle import fna2_oracle as O

# Tolerance (bf16 kernel vs fp32/fp64 oracle on identical bf16-representable
# inputs): relative L2 <= 1e-2 and max-abs <= 2e-2 (the north star's bf16
# bound).  The flat max-abs bound is applied first.  Only where it fails on a
# tensor whose values exceed 1 is it scaled by max|ref|: a bf16 value near 8
# is itself only representable to 2^-5 = 0.031 (half-ULP 0.016), so rounding
# the exact result to the bf16 output alone can exceed 2e-2 there.  Every
# check is recorded in REPORT with the bound it used.
REL_L2 = 1e-2
MAX_ABS = 2e-2

GRADS = ("dq", "dk", "dv", "drq", "drk", "dgs")

REPORT = []  # one dict per check: name, max_abs, rel_l2, ref_max, bound, kind


def check(name, ref, got, rel_l2=REL_L2, max_abs=MAX_ABS):
    ref = ref.detach().cpu()
    got = got.detach().float().cpu()
    e = O.errors(ref, got)
    assert math.isfinite(e["max_abs"]), f"{name}: non-finite values {e}"
    flat = e["max_abs"] <= max_abs
    bound = max_abs if flat else max_abs * max(1.0, e["ref_max"])
    # relative L2 with a noise floor: a tensor whose true values are ~1e-6
    # (e.g. dQ of a single-token sequence, zero up to the +1e-6 normalisation)
    # is judged by max-abs alone
    floor = 1e-3 * math.sqrt(max(ref.numel(), 1))
    rel = (ref.double() - got.double()).norm().item() / max(ref.double().norm().item(), floor)
    e["rel_l2_floored"] = rel
    REPORT.append({"name": name, "max_abs": e["max_abs"], "rel_l2": e["rel_l2"], "ref_max": e["ref_max"],
                   "bound": bound, "kind": "flat" if flat else "scaled by max|ref|"})
    assert rel <= rel_l2 and e["max_abs"] <= bound, f"{name}: {e} (bound max_abs {bound:.3g})"
    return e


def record(name, max_abs, rel_l2, ref_max, bound, kind):
    """Record an aggregate check made outside check() (streamed full-size tensors)."""
    REPORT.append({"name": name, "max_abs": max_abs, "rel_l2": rel_l2, "ref_max": ref_max, "bound": bound,
                   "kind": kind})


def run_cuda(q, k, v, rq, rk, gs, do, scale, causal, cu=None, max_seqlen=0, backward=True, cu_k=None,
             max_seqlen_k=None):
    """Call the drop-in op on CUDA copies; returns dict of CPU fp32 results."""
    from fna2_b200 import flash_naylis_attn
    dev = "cuda"
    t = [x.to(dev, torch.bfloat16).requires_grad_(backward) for x in (q, k, v, rq, rk)]
    g = gs.to(dev, torch.float32).requires_grad_(backward)
    kw = {}
    if cu is not None:
        cu_t = torch.tensor(cu, dtype=torch.int32, device=dev)
        cu_kt = cu_t if cu_k is None else torch.tensor(cu_k, dtype=torch.int32, device=dev)
        msk = max_seqlen if max_seqlen_k is None else max_seqlen_k
        kw = dict(cu_seqlens_q=cu_t, cu_seqlens_k=cu_kt, max_seqlen_q=max_seqlen, max_seqlen_k=msk)
    out = flash_naylis_attn(*t, g, softmax_scale=scale, is_causal=causal, **kw)
    res = {"out": out.detach().float().cpu()}
    if backward:
        out.backward(do.to(dev, torch.bfloat16))
        for name, x in zip(GRADS, t + [g]):
            res[name] = x.grad.detach().float().cpu()
    return res


def run_oracle(q, k, v, rq, rk, gs, do, scale, causal, cu=None, dtype=torch.float64, backward=True, cu_k=None):
    c = lambda x: x.to(dtype)
    if cu is None:
        out, lse = O.attention_fwd(c(q), c(k), c(v), c(rq), c(rk), c(gs), scale, causal)
        res = {"out": out, "lse": lse}
        if backward:
            g = O.attention_bwd(c(q), c(k), c(v), c(rq), c(rk), c(gs), out, lse, c(do), scale, causal,
                                dgs_terms=True)
            res.update(dict(zip(GRADS, g)))
            res["dgs_terms_sq"] = g[6]
    else:
        ck = cu if cu_k is None else cu_k
        out, lse = O.varlen_fwd(c(q), c(k), c(v), c(rq), c(rk), c(gs), cu, ck, scale)
        res = {"out": out, "lse": lse}
        if backward:
            g = O.varlen_bwd(c(q), c(k), c(v), c(rq), c(rk), c(gs), out, lse, c(do), cu, ck, scale,
                             dgs_terms=True)
            res.update(dict(zip(GRADS, g)))
            res["dgs_terms_sq"] = g[6]
    return res


# rounding a summand to bf16 moves it by up to 2^-9 of itself, uniformly:
# standard deviation 2^-9/sqrt(3) relative
BF16_NOISE = 2.0 ** -9 / math.sqrt(3.0)


def check_dgs(name, ref, got, terms_sq):
    """d_graph_scale: one sum per graph head over every query-key pair of every
    sequence, often with heavy cancellation.  The kernels form it from the
    bf16 dS that also feeds the dQ / dR_q tensor-core contraction (the
    reference sums the fp32 dS, flash_naylis_attn.py:537-538), so each
    summand dS_ij * (R_q R_k^T)_ij carries a bf16 rounding.  It passes the
    standard bounds, or else every head's error must stay within four
    standard deviations of that rounding noise, 4 * 2^-9/sqrt(3) *
    sqrt(sum of squared summands) (``terms_sq`` from the oracle).  Both
    figures are recorded."""
    try:
        return check(name, ref, got)
    except AssertionError:
        ref = ref.detach().double().cpu()
        err = (got.detach().double().cpu() - ref).abs()
        sigma = BF16_NOISE * terms_sq.detach().double().cpu().sqrt()
        ratio = (err / sigma.clamp_min(1e-300)).max().item()
        REPORT.append({"name": name + " (bf16-dS noise bound)", "max_abs": err.max().item(),
                       "rel_l2": (err.norm() / ref.norm()).item(), "ref_max": ref.abs().max().item(),
                       "bound": 4.0, "kind": f"error / rounding-noise sigma = {ratio:.3g}"})
        assert ratio <= 4.0, f"{name}: error {err.tolist()} is {ratio:.3g} sigma of the bf16-dS rounding noise"
        return {"max_abs": err.max().item(), "noise_sigmas": ratio}


def compare(ref, got, names=("out",) + GRADS, label=""):
    errs = {}
    for n in names:
        if n in got and n in ref:
            if ref[n].numel() == 0:
                continue
            if n == "dgs" and "dgs_terms_sq" in ref:
                errs[n] = check_dgs(f"{label}{n}", ref[n], got[n], ref["dgs_terms_sq"])
            else:
                errs[n] = check(f"{label}{n}", ref[n], got[n])
    return errs
