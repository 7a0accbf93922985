"""Load a committed golden fixture and regenerate its (bf16-exact) inputs."""
import hashlib
import os

import torch

from oracle import fna2_oracle as O

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
CASES = ["cfg1_sdpa", "gqa_vanilla_sdpa", "interp_dense_causal_d64", "interp_dense_noncausal_d64",
         "interp_dense_causal_d128", "interp_varlen_d64", "interp_varlen_d128"]


def _hash(*ts):
    h = hashlib.sha256()
    for t in ts:
        h.update(t.detach().to(torch.float32).contiguous().numpy().tobytes())
    return h.hexdigest()


def load(name):
    rec = torch.load(os.path.join(GOLDEN, name + ".pt"), weights_only=False)
    if rec["kind"] == "dense":
        q, k, v, rq, rk, gs, do = O.make_dense_inputs(rec["B"], rec["H"], rec["S"], rec["D"], rec["r"],
                                                      rec["H_KV"], rec["H_G"], rec["seed"], rec["gs_value"])
        cu = None
    else:
        q, k, v, rq, rk, gs, do, cu = O.make_varlen_inputs(rec["lengths"], rec["H"], rec["D"], rec["r"],
                                                           rec["H_KV"], rec["H_G"], rec["seed"],
                                                           rec["gs_value"])
    q, k, v, rq, rk, do = O.bf16_round(q, k, v, rq, rk, do)
    assert _hash(q, k, v, rq, rk, do, gs) == rec["input_sha256"], "RNG drift: regenerated inputs differ"
    return rec, (q, k, v, rq, rk, gs, do, cu)
