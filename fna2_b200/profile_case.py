"""Run forward + backward of one dense causal problem a few times, for profilers.

    python -m fna2_b200.profile_case --batch 1 --heads 16 --seqlen 4096 --head-dim 128 --rank 16 --reps 2

Inputs are seeded synthetic tensors (q, k, v, dO ~ N(0, 1); r_q, r_k ~ N(0, 1)/4;
graph_scale = 1, all heads graph heads).  Each repetition launches the forward kernel
and the three backward kernels once, in that order, so a profiler can skip the first
repetition's launches (e.g. ``ncu -k regex:fna2_... -s 3 -c 3``).

    python -m fna2_b200.profile_case --op qk_prep --batch 32 --heads 32 --seqlen 2048 --head-dim 128 --reps 2

runs the varlen QK-RMSNorm + RoPE transform instead: ``batch`` packed sequences of
``seqlen`` tokens, ``heads`` query and key heads (bf16), bf16 norm weights, RoPE
on; each repetition launches its forward and its backward kernel once.

    python -m fna2_b200.profile_case --op decode --batch 32 --heads 32 --seqlen 4096 --head-dim 128 --rank 16 --reps 2

runs one KV-cache decode step per repetition: ``batch`` sequences with
``seqlen`` cached keys each (dense caches, H_KV = heads, all graph heads), one
new token per sequence appended and attended.
"""
import argparse
import math

import torch

from .flash_naylis_attn import _fna2_backward, _fna2_forward


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--heads", type=int, default=16)
    ap.add_argument("--seqlen", type=int, default=4096)
    ap.add_argument("--head-dim", type=int, default=128)
    ap.add_argument("--rank", type=int, default=16)
    ap.add_argument("--reps", type=int, default=2)
    ap.add_argument("--op", default="attention", choices=["attention", "qk_prep", "decode"])
    a = ap.parse_args(argv)
    if a.op == "qk_prep":
        return qk_prep_case(a)
    if a.op == "decode":
        return decode_case(a)
    g = torch.Generator(device="cuda").manual_seed(0)
    shape = (a.batch, a.heads, a.seqlen, a.head_dim)
    q, k, v, do = (torch.randn(shape, device="cuda", generator=g).bfloat16() for _ in range(4))
    rshape = (a.batch, a.heads, a.seqlen, a.rank)
    rq, rk = ((torch.randn(rshape, device="cuda", generator=g) * 0.25).bfloat16() for _ in range(2))
    gs = torch.ones(a.heads, device="cuda")
    scale = 1.0 / math.sqrt(a.head_dim)
    for _ in range(a.reps):
        out, lse = _fna2_forward(q, k, v, rq, rk, gs, scale, True)
        _fna2_backward(do, q, k, v, rq, rk, gs, out, lse, scale, True)
    torch.cuda.synchronize()
    print("ok")


def qk_prep_case(a):
    import types

    from .qk_prep import apply_qk_norm_rope_varlen

    g = torch.Generator(device="cuda").manual_seed(0)
    T, D = a.batch * a.seqlen, a.head_dim
    cu = torch.arange(0, T + 1, a.seqlen, dtype=torch.int32, device="cuda")
    q, k, dq_out, dk_out = (torch.randn(T, a.heads, D, device="cuda", generator=g).bfloat16() for _ in range(4))
    q.requires_grad_(True)
    k.requires_grad_(True)
    norms = [types.SimpleNamespace(weight=torch.ones(D, device="cuda", dtype=torch.bfloat16, requires_grad=True),
                                   eps=1e-6) for _ in range(2)]
    inv_freq = 1.0 / (10000.0 ** (torch.arange(0, D, 2, device="cuda").float() / D))
    rope = types.SimpleNamespace(inv_freq=inv_freq)
    for _ in range(a.reps):
        qo, ko = apply_qk_norm_rope_varlen(q, k, cu, norms[0], norms[1], rope)
        torch.autograd.backward((qo, ko), (dq_out, dk_out))
    torch.cuda.synchronize()
    print("ok")


def decode_case(a):
    from .decode import flash_naylis_decode

    g = torch.Generator(device="cuda").manual_seed(0)
    B, H, D, R, L = a.batch, a.heads, a.head_dim, a.rank, a.seqlen
    kc, vc = (torch.randn(B, L + 1, H, D, device="cuda", generator=g).bfloat16() for _ in range(2))
    rkc = (torch.randn(B, L + 1, H, R, device="cuda", generator=g) * 0.25).bfloat16()
    q, kn, vn = (torch.randn(B, H, D, device="cuda", generator=g).bfloat16() for _ in range(3))
    rq, rkn = ((torch.randn(B, H, R, device="cuda", generator=g) * 0.25).bfloat16() for _ in range(2))
    gs = torch.ones(H, device="cuda")
    seq = torch.full((B,), L, dtype=torch.int32, device="cuda")
    for _ in range(a.reps):
        flash_naylis_decode(q, kc, vc, seq, rq, rkc, gs, kn, vn, rkn)
    torch.cuda.synchronize()
    print("ok")


if __name__ == "__main__":
    main()
