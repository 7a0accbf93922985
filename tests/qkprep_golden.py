"""Load a committed QK-norm/RoPE golden fixture and regenerate its inputs."""
import hashlib
import os

import torch

from oracle import qk_prep_oracle as Q

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
CASES = ["qkprep_f32_d128", "qkprep_f32_d64_yarn_tail", "qkprep_bf16_d128_long", "qkprep_bf16_in_f32_weights_d128"]
_DT = {"torch.float32": torch.float32, "torch.bfloat16": torch.bfloat16}


def _hash(*ts):
    h = hashlib.sha256()
    for t in ts:
        h.update(t.detach().to(torch.float32).contiguous().numpy().tobytes())
    return h.hexdigest()


def load(name):
    rec = torch.load(os.path.join(GOLDEN, name + ".pt"), weights_only=False)
    wdt = _DT[rec["weights_dtype"]] if rec["weights_dtype"] else None
    inputs = Q.make_inputs(rec["lengths"], rec["H"], rec["H_KV"], rec["D"], rec["seed"], _DT[rec["dtype"]],
                           rec["lead"], rec["tail"], rec["yarn_scale"], wdt)
    assert _hash(*inputs) == rec["input_sha256"], "RNG drift: regenerated inputs differ"
    return rec, inputs
