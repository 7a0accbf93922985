"""CPU: the QK-RMSNorm + RoPE oracle reproduces the reference's own classes
(fixtures from tests/golden/make_golden_qkprep.py) on outputs and gradients."""
import pytest
import torch

from oracle import qk_prep_oracle as Q
from tests.qkprep_golden import CASES, load


def _rel(a, b):
    a, b = a.float(), b.float()
    return ((a - b).norm() / b.norm().clamp_min(1e-30)).item()


@pytest.mark.parametrize("name", CASES)
def test_oracle_matches_reference_fixture(name):
    rec, (q, k, wq, wk, inv, cu, dqo, dko) = load(name)
    qo, ko, (gq, gk, gwq, gwk) = Q.qk_prep_with_grads(q, k, cu, wq, wk, rec["eps"], inv, dqo, dko)
    lo, hi = int(cu[0]), int(cu[-1])
    assert _rel(qo[lo:hi], rec["q_out"][lo:hi]) < 1e-6
    assert _rel(ko[lo:hi], rec["k_out"][lo:hi]) < 1e-6
    for got, want in ((gq, rec["dq"]), (gk, rec["dk"]), (gwq, rec["dwq"]), (gwk, rec["dwk"])):
        assert _rel(got, want) < 1e-6


def test_positions_restart_per_sequence():
    # a single token at the start of each sequence is never rotated (cos 0 = 1, sin 0 = 0)
    q, k, wq, wk, inv, cu, _, _ = Q.make_inputs([1, 1, 1], 2, 1, 64, 3)
    qo, ko = Q.qk_prep(q, k, cu, None, None, 1e-6, inv)
    assert torch.equal(qo, q.to(torch.bfloat16)) and torch.equal(ko, k.to(torch.bfloat16))


def test_inv_freq_matches_reference_formula():
    inv = Q.rope_inv_freq(128)
    assert torch.allclose(inv, 1.0 / (10000 ** (torch.arange(0, 128, 2).float() / 128)))
    yarn = Q.rope_inv_freq(128, yarn_scale=4.0)
    assert torch.equal(yarn[:33], inv[:33]) and (yarn[33:] < inv[33:]).all()  # dims >= D/2 scaled, dim D/2 by 1
