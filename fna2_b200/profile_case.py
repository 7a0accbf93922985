"""Run forward + backward of one dense causal problem a few times, for profilers.

    python -m fna2_b200.profile_case --batch 1 --heads 16 --seqlen 4096 --head-dim 128 --rank 16 --reps 2

Inputs are seeded synthetic tensors (q, k, v, dO ~ N(0, 1); r_q, r_k ~ N(0, 1)/4;
graph_scale = 1, all heads graph heads).  Each repetition launches the forward kernel
and the three backward kernels once, in that order, so a profiler can skip the first
repetition's launches (e.g. ``ncu -k regex:fna2_... -s 3 -c 3``).
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
    a = ap.parse_args(argv)
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


if __name__ == "__main__":
    main()
