"""The bounded mbarrier waits: a wait that runs out records its site code,
the kernel exits cleanly (tensor memory released, no fault) and the next call
works.  The failure is made on purpose without any GPU fault: the forward
kernel withholds one hand-off arrival (a flag that nothing sets) under a 50 ms
wait budget, through the fna2_debug_watchdog testing hook."""
import math

import pytest
import torch

from oracle import fna2_oracle as O
from tests import parity

pytestmark = pytest.mark.gpu

SITE_FWD_P = 204  # the forward MMA thread's wait for the first P hand-off
# With that hand-off withheld, the first wait of the CTA to run out is either
# the MMA thread's (204) or the softmax warps' wait for the end of the tile,
# which can no longer come (304); both are sites of the forward kernel.
EXPECTED = {SITE_FWD_P, 304}


def test_wait_that_runs_out_reports_and_recovers():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from fna2_b200 import _lib, flash_naylis_attn
    lib = _lib.load()
    q, k, v, rq, rk, gs, do = O.make_dense_inputs(1, 2, 64, 64, 16, seed=1, gs_value="randn")
    q, k, v, rq, rk, do = O.bf16_round(q, k, v, rq, rk, do)
    dev = lambda t: t.cuda().bfloat16()
    assert lib.fna2_device_status(1) == 0
    try:
        _lib.check(lib.fna2_debug_watchdog(SITE_FWD_P, 50_000_000), "fna2_debug_watchdog")
        with torch.no_grad():
            flash_naylis_attn(dev(q), dev(k), dev(v), dev(rq), dev(rk), gs.cuda(), is_causal=True)
        torch.cuda.synchronize()  # the kernel returned: no hang, no fault
        assert lib.fna2_device_status(1) in EXPECTED
    finally:
        _lib.check(lib.fna2_debug_watchdog(0, 0), "fna2_debug_watchdog")
    # the context is intact and the next call is exact again
    got = parity.run_cuda(q, k, v, rq, rk, gs, do, 1 / math.sqrt(64), True)
    ref = parity.run_oracle(q, k, v, rq, rk, gs, do, 1 / math.sqrt(64), True)
    parity.compare(ref, got, label="after watchdog ")
    assert lib.fna2_device_status(1) == 0


def test_debug_hook_rejects_unknown_sites():
    from fna2_b200 import _lib
    lib = _lib.load()
    assert lib.fna2_debug_watchdog(999, 0) == _lib.FNA2_ERR_INVALID
