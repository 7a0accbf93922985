"""Generate the golden fixtures under ``tests/golden/`` from the REFERENCE itself.

Run in a container that has the reference source mounted (it is imported from
``$FNA2_REFERENCE``, required: the reference checkout's FNA2 directory); the fixtures it writes
are committed, so nothing else ever needs the reference at run time.

Two witnesses of the reference are recorded:

* ``sdpa``   -- ``validate_fna2._sdpa_reference`` (validate_fna2.py:84-112),
  the reference's own eager validation path, run in fp32 on the CPU by setting
  its module globals ``DTYPE=float32`` and ``DEVICE="cpu"`` (read at
  validate_fna2.py:101,103,106).  Gradients via autograd, as its T2 test does
  (validate_fna2.py:150-159).
* ``interp`` -- the reference's Triton kernels (flash_naylis_attn.py) run in
  fp32 by the Triton CPU interpreter (``TRITON_INTERPRET=1``), with the module
  global ``BLOCK_R`` set to the case's rank (flash_naylis_attn.py:51 locks the
  rank to ``BLOCK_R``).  This records the kernels' exact semantics: the
  ``+1e-6`` normalisation, the LSE, ragged tiles, GQA, vanilla heads, non-causal
  dense and varlen packing.

Inputs are regenerated from seeds by ``oracle.fna2_oracle.make_*_inputs`` and
rounded to bf16-representable values, so a bf16 GPU kernel sees exactly the
same numbers; a SHA-256 of the rounded inputs is stored to catch RNG drift.
"""
from __future__ import annotations

import hashlib
import math
import os
import sys

os.environ.setdefault("TRITON_INTERPRET", "1")

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

import torch  # noqa: E402

from oracle import fna2_oracle as O  # noqa: E402

REF = os.environ.get("FNA2_REFERENCE")
if not REF:
    raise SystemExit("set FNA2_REFERENCE to the reference checkout's FNA2 directory "
                     "(the directory holding flash_naylis_attn.py)")


def _hash(*ts):
    h = hashlib.sha256()
    for t in ts:
        h.update(t.detach().to(torch.float32).contiguous().numpy().tobytes())
    return h.hexdigest()


def _leaf(*ts):
    return [t.detach().clone().requires_grad_(True) for t in ts]


def dense_case(name, B, H, S, D, r, H_KV, H_G, seed, gs_value, causal, witness):
    q, k, v, rq, rk, gs, do = O.make_dense_inputs(B, H, S, D, r, H_KV, H_G, seed, gs_value)
    q, k, v, rq, rk, do = O.bf16_round(q, k, v, rq, rk, do)
    scale = 1.0 / math.sqrt(D)
    rec = dict(kind="dense", B=B, H=H, S=S, D=D, r=r, H_KV=H_KV, H_G=H_G, seed=seed,
               gs_value=gs_value, causal=causal, scale=scale, witness=witness,
               input_sha256=_hash(q, k, v, rq, rk, do, gs))
    lq, lk, lv, lrq, lrk, lgs = _leaf(q, k, v, rq, rk, gs)
    if witness == "sdpa":
        import validate_fna2 as V
        V.DTYPE = torch.float32
        V.DEVICE = "cpu"
        assert causal
        cfg = dict(B=B, H=H, S=S, D=D, H_KV=H_KV, H_G=H_G)
        out = V._sdpa_reference(lq, lk, lv, lrq, lrk, lgs, cfg)
        lse = None
    else:
        import flash_naylis_attn as FN
        FN.BLOCK_R = r
        out = FN.FlashNaylisAttnFunc.apply(lq, lk, lv, lrq, lrk, lgs, scale, causal,
                                           None, None, 0, 0)
        lse = FN._fna2_forward(q, k, v, rq, rk, gs, scale, causal)[1]
    out.backward(do)
    rec.update(out=out.detach(), dq=lq.grad, dk=lk.grad, dv=lv.grad, drq=lrq.grad,
               drk=lrk.grad, dgs=lgs.grad)
    if lse is not None:
        rec["lse"] = lse.detach()
    torch.save(rec, os.path.join(HERE, f"{name}.pt"))
    print("wrote", name, {k2: tuple(v2.shape) for k2, v2 in rec.items() if torch.is_tensor(v2)})


def varlen_case(name, lengths, H, D, r, H_KV, H_G, seed, gs_value):
    q, k, v, rq, rk, gs, do, cu = O.make_varlen_inputs(lengths, H, D, r, H_KV, H_G, seed, gs_value)
    q, k, v, rq, rk, do = O.bf16_round(q, k, v, rq, rk, do)
    scale = 1.0 / math.sqrt(D)
    import flash_naylis_attn as FN
    FN.BLOCK_R = r
    cu_t = torch.tensor(cu, dtype=torch.int32)
    msl = max(lengths)
    lq, lk, lv, lrq, lrk, lgs = _leaf(q, k, v, rq, rk, gs)
    out = FN.FlashNaylisAttnFunc.apply(lq, lk, lv, lrq, lrk, lgs, scale, True, cu_t, cu_t, msl, msl)
    out.backward(do)
    lse = FN._fna2_forward_varlen(q, k, v, rq, rk, gs, cu_t, cu_t, msl, msl, scale)[1]
    rec = dict(kind="varlen", lengths=list(lengths), cu=cu, H=H, D=D, r=r, H_KV=H_KV, H_G=H_G,
               seed=seed, gs_value=gs_value, causal=True, scale=scale, witness="interp",
               input_sha256=_hash(q, k, v, rq, rk, do, gs),
               out=out.detach(), lse=lse.detach(), dq=lq.grad, dk=lk.grad, dv=lv.grad,
               drq=lrq.grad, drk=lrk.grad, dgs=lgs.grad)
    torch.save(rec, os.path.join(HERE, f"{name}.pt"))
    print("wrote", name, {k2: tuple(v2.shape) for k2, v2 in rec.items() if torch.is_tensor(v2)})


def main():
    sys.path.insert(0, REF)
    torch.set_num_threads(os.cpu_count() or 1)
    # B2 H4 L256 D64 r8 causal, seed 0, gs = 1 (the reference's eager path).
    dense_case("cfg1_sdpa", 2, 4, 256, 64, 8, 4, 4, 0, None, True, "sdpa")
    # validate_fna2 "60m" shape: GQA 2:1, 4 graph + 4 vanilla heads, R=32, gs ~ N(0,1).
    dense_case("gqa_vanilla_sdpa", 2, 8, 128, 64, 32, 4, 4, 42, "randn", True, "sdpa")
    # Reference kernels under the Triton interpreter: ragged S, GQA, vanilla heads.
    dense_case("interp_dense_causal_d64", 1, 4, 200, 64, 16, 2, 2, 1, "randn", True, "interp")
    dense_case("interp_dense_noncausal_d64", 1, 4, 200, 64, 16, 2, 2, 2, "randn", False, "interp")
    dense_case("interp_dense_causal_d128", 1, 2, 160, 128, 32, 1, 2, 3, "randn", True, "interp")
    varlen_case("interp_varlen_d64", [1, 63, 130, 64, 200], 4, 64, 16, 2, 2, 4, "randn")
    varlen_case("interp_varlen_d128", [129, 17, 256], 2, 128, 16, 2, 1, 5, "randn")


if __name__ == "__main__":
    main()
