"""Golden fixtures for the varlen QK-RMSNorm + RoPE transform, produced by the
REFERENCE's own classes (FNA2/attention_fna2.py: RMSNorm :94-102,
RotaryPositionalEmbedding :108-170, NaylisAttention._apply_rope_varlen
:620-647) on the CPU.  Run where the reference source is mounted
(``$FNA2_REFERENCE``, required: the reference checkout's FNA2 directory); the .pt files it writes
are committed.  Inputs are regenerated from seeds by
``oracle.qk_prep_oracle.make_inputs``; a SHA-256 of them is stored.

Every case has cu_seqlens[0] = 0: the reference's per-sequence loop starts at
token 0 whatever cu_seqlens[0] is (attention_fna2.py:634-646), while the
attention kernels (and this build) read cu_seqlens as absolute offsets, so a
leading gap is not a case the two agree on."""
from __future__ import annotations

import hashlib
import os
import sys
import types

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

import torch  # noqa: E402

from oracle import qk_prep_oracle as Q  # noqa: E402

REF = os.environ.get("FNA2_REFERENCE")
if not REF:
    raise SystemExit("set FNA2_REFERENCE to the reference checkout's FNA2 directory "
                     "(the directory holding flash_naylis_attn.py)")

CASES = {
    # name: (lengths, H, H_KV, D, seed, dtype, lead, tail, yarn_scale, weights dtype)
    "qkprep_f32_d128": ([37, 1, 200, 64], 4, 2, 128, 11, torch.float32, 0, 0, 1.0, None),
    "qkprep_f32_d64_yarn_tail": ([5, 250, 17], 3, 3, 64, 12, torch.float32, 0, 4, 2.0, None),
    "qkprep_bf16_d128_long": ([700, 12], 2, 1, 128, 13, torch.bfloat16, 0, 0, 1.0, None),
    "qkprep_bf16_in_f32_weights_d128": ([90, 33], 2, 2, 128, 14, torch.bfloat16, 0, 0, 1.0, torch.float32),
}


def _hash(*ts):
    h = hashlib.sha256()
    for t in ts:
        h.update(t.detach().to(torch.float32).contiguous().numpy().tobytes())
    return h.hexdigest()


def run_reference(A, q, k, wq, wk, inv_freq, cu, dqo, dko, D, yarn_scale):
    norm_q, norm_k = A.RMSNorm(D), A.RMSNorm(D)
    with torch.no_grad():
        norm_q.weight.copy_(wq.float())
        norm_k.weight.copy_(wk.float())
    norm_q.weight.data = norm_q.weight.data.to(wq.dtype)
    norm_k.weight.data = norm_k.weight.data.to(wk.dtype)
    rope = A.RotaryPositionalEmbedding(D, 4096, use_yarn=yarn_scale != 1.0, yarn_scale=yarn_scale)
    assert torch.equal(rope.inv_freq, inv_freq)
    self_like = types.SimpleNamespace(rope=rope)
    ql, kl = q.detach().clone().requires_grad_(True), k.detach().clone().requires_grad_(True)
    qn, kn = norm_q(ql), norm_k(kl)                                     # attention_fna2.py:558-561
    qr, kr = A.NaylisAttention._apply_rope_varlen(self_like, qn, kn, cu)  # :563-566
    if qr.dtype == torch.float32:                                        # :568-572
        qr, kr = qr.to(torch.bfloat16), kr.to(torch.bfloat16)
    lo, hi = int(cu[0]), int(cu[-1])
    loss = (qr[lo:hi].float() * dqo[lo:hi].float()).sum() + (kr[lo:hi].float() * dko[lo:hi].float()).sum()
    loss.backward()
    return qr.detach(), kr.detach(), ql.grad, kl.grad, norm_q.weight.grad, norm_k.weight.grad


def main():
    sys.path.insert(0, REF)
    import attention_fna2 as A  # noqa: E402
    for name, (lengths, H, H_KV, D, seed, dtype, lead, tail, ys, wdt) in CASES.items():
        q, k, wq, wk, inv_freq, cu, dqo, dko = Q.make_inputs(lengths, H, H_KV, D, seed, dtype, lead, tail, ys, wdt)
        qo, ko, gq, gk, gwq, gwk = run_reference(A, q, k, wq, wk, inv_freq, cu, dqo, dko, D, ys)
        rec = dict(kind="qkprep", lengths=lengths, H=H, H_KV=H_KV, D=D, seed=seed, dtype=str(dtype), lead=lead,
                   tail=tail, yarn_scale=ys, weights_dtype=str(wdt) if wdt else None, eps=1e-6,
                   input_sha256=_hash(q, k, wq, wk, inv_freq, cu, dqo, dko),
                   q_out=qo, k_out=ko, dq=gq, dk=gk, dwq=gwq, dwk=gwk)
        torch.save(rec, os.path.join(HERE, name + ".pt"))
        print(name, "T", q.shape[0], "saved")


if __name__ == "__main__":
    main()
