"""fna2_bwd_noalloc: the backward entry point for callers that cannot allocate.

Callers such as a process whose device memory is owned entirely by another
allocator (a fixed arena or a framework's caching pool), or a thin cgo / JNI /
ctypes binding with no allocator of its own, cannot hand fna2_bwd the scratch
workspace it needs.  fna2_bwd_noalloc takes that scratch from a static device
array instead.  These tests call it through the C ABI and check it against
fna2_bwd (same kernels, caller-provided workspace) on two calls in a row, so a
second call that reuses the array's stale contents is covered too.

The file name sorts last so that a run stopping at the first failure has run
every other test before this one.
"""
import ctypes
import math
import threading

import pytest
import torch

from fna2_b200 import _lib
from fna2_b200.flash_naylis_attn import _desc, _problem
from oracle import fna2_oracle as O
from tests import parity


def _bwd_args(prob, t, varlen):
    a = _lib.Fna2BwdArgs()
    a.prob = prob
    a.q, a.k, a.v = _desc(t["q"], varlen), _desc(t["k"], varlen), _desc(t["v"], varlen)
    a.r_q, a.r_k = _desc(t["rq"], varlen), _desc(t["rk"], varlen)
    a.graph_scale = t["gs"].data_ptr()
    a.out, a.dout = _desc(t["out"], varlen), _desc(t["do"], varlen)
    a.lse = t["lse"].data_ptr()
    a.dq, a.dk, a.dv = _desc(t["dq"], varlen), _desc(t["dk"], varlen), _desc(t["dv"], varlen)
    a.dr_q, a.dr_k = _desc(t["drq"], varlen), _desc(t["drk"], varlen)
    a.d_graph_scale = t["dgs"].data_ptr()
    return a


def _fresh_grads(t):
    nan = float("nan")
    for n, src in (("dq", "q"), ("dk", "k"), ("dv", "v"), ("drq", "rq"), ("drk", "rk")):
        t[n] = torch.full_like(t[src], nan)
    t["dgs"] = torch.full_like(t["gs"], nan)


@pytest.mark.gpu
def test_noalloc_backward_matches_workspace_backward_twice():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    lib = _lib.load()
    lengths = [200, 77, 300]
    H, HKV, HG, D, r = 4, 2, 3, 128, 16
    q, k, v, rq, rk, gs, do, cu = O.make_varlen_inputs(lengths, H, D, r, HKV, HG, seed=21, gs_value="randn")
    dev = torch.device("cuda", 0)
    t = {n: x.to(dev, torch.bfloat16).contiguous() for n, x in
         (("q", q), ("k", k), ("v", v), ("rq", rq), ("rk", rk), ("do", do))}
    t["gs"] = gs.to(dev)
    cu_t = torch.tensor(cu, dtype=torch.int32, device=dev)
    scale = 1.0 / math.sqrt(D)
    prob = _problem(t["q"], t["k"], t["rq"], scale, True, cu_t, cu_t, max(lengths), max(lengths))
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)

    # forward through the C ABI
    t["out"] = torch.empty_like(t["q"])
    t["lse"] = torch.empty(H, t["q"].shape[0], dtype=torch.float32, device=dev)
    fa = _lib.Fna2FwdArgs()
    fa.prob = prob
    fa.q, fa.k, fa.v = _desc(t["q"], True), _desc(t["k"], True), _desc(t["v"], True)
    fa.r_q, fa.r_k = _desc(t["rq"], True), _desc(t["rk"], True)
    fa.graph_scale = t["gs"].data_ptr()
    fa.out = _desc(t["out"], True)
    fa.lse = t["lse"].data_ptr()
    fws = torch.empty(lib.fna2_fwd_workspace_size(ctypes.byref(prob)), dtype=torch.uint8, device=dev)
    fa.workspace, fa.workspace_bytes = fws.data_ptr(), fws.numel()
    _lib.check(lib.fna2_fwd(ctypes.byref(fa), stream), "fna2_fwd")

    # existing entry point with a caller-provided workspace
    _fresh_grads(t)
    ws = torch.empty(lib.fna2_bwd_workspace_size(ctypes.byref(prob)), dtype=torch.uint8, device=dev)
    a = _bwd_args(prob, t, True)
    a.workspace, a.workspace_bytes = ws.data_ptr(), ws.numel()
    _lib.check(lib.fna2_bwd(ctypes.byref(a), stream), "fna2_bwd")
    torch.cuda.synchronize()
    ref = {n: t[n].float().cpu() for n in ("dq", "dk", "dv", "drq", "drk", "dgs")}

    # the no-allocation entry point, twice in a row (the second reuses the scratch)
    for call in range(2):
        _fresh_grads(t)
        b = _bwd_args(prob, t, True)
        b.workspace, b.workspace_bytes = None, 0
        _lib.check(lib.fna2_bwd_noalloc(ctypes.byref(b), stream), "fna2_bwd_noalloc")
        torch.cuda.synchronize()
        for n in ref:
            parity.check(f"noalloc call {call + 1} {n}", ref[n], t[n])

    # and once more from a host thread that has made no CUDA call yet: the
    # scratch address is cached from the calls above, and the tensor maps
    # still need the device's context bound on this new thread
    _fresh_grads(t)
    b = _bwd_args(prob, t, True)
    b.workspace, b.workspace_bytes = None, 0
    torch.cuda.synchronize()
    rc = []
    def call():  # fna2_last_error is per host thread: read it on the calling thread
        rc.append((lib.fna2_bwd_noalloc(ctypes.byref(b), None), lib.fna2_last_error()))

    th = threading.Thread(target=call)
    th.start()
    th.join()
    assert rc and rc[0][0] == _lib.FNA2_OK, rc
    torch.cuda.synchronize()
    for n in ref:
        parity.check(f"noalloc fresh-thread call {n}", ref[n], t[n])
    assert lib.fna2_device_status(1) == 0


def test_noalloc_rejects_problems_beyond_the_static_scratch():
    """Oversized problems fail on the host with FNA2_ERR_WORKSPACE, before any
    CUDA call (runs without a GPU)."""
    lib = _lib.load()
    a = _lib.Fna2BwdArgs()
    p = a.prob
    p.batch, p.seqlen_q, p.seqlen_k = 1, 262144, 262144  # 32 heads x 262144 rows x 8 B = 64 MiB > 32 MiB
    p.heads, p.heads_kv, p.heads_graph, p.head_dim, p.rank = 32, 32, 0, 128, 16
    p.softmax_scale, p.causal = 0.088, 1
    for name in ("q", "k", "v", "out", "dout", "dq", "dk", "dv"):
        d = getattr(a, name)
        d.ptr = 0x10000
        d.stride[:] = (32 * 262144 * 128, 262144 * 128, 128, 1)
    a.lse = 0x10000
    rc = lib.fna2_bwd_noalloc(ctypes.byref(a), None)
    assert rc == _lib.FNA2_ERR_WORKSPACE
    msg = lib.fna2_last_error().decode()
    assert "static scratch" in msg and str(_lib.NOALLOC_SCRATCH_BYTES) in msg
