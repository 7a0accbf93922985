"""Drop-in replacement for the reference module ``FNA2/flash_naylis_attn.py``.

Public surface kept verbatim (myAiByMe/FNA2):

* ``flash_naylis_attn(q, k, v, r_q, r_k, graph_scale, softmax_scale=None,
  is_causal=True, cu_seqlens_q=None, cu_seqlens_k=None, max_seqlen_q=0,
  max_seqlen_k=0)`` -- flash_naylis_attn.py:1380-1434;
* ``FlashNaylisAttnFunc`` -- the autograd Function, flash_naylis_attn.py:1307-1373
  (saves q,k,v,r_q,r_k,gs,out,lse; backward makes dout contiguous and returns
  six gradients plus six ``None``);
* module constants ``BLOCK_M``, ``BLOCK_N``, ``BLOCK_R`` (:49-51).  ``BLOCK_R``
  stays 32 so that ``NaylisAttention`` (attention_fna2.py:225-228), which
  enables FNA2 only when ``rel_rank == BLOCK_R``, keeps working unchanged; the
  op itself accepts any rank r in {8, 16, 24, 32} (the reference asserts
  ``r == BLOCK_R``, :1423-1427).

Behind it, the op is registered with PyTorch as the custom ops ``fna2::fwd``
and ``fna2::bwd`` (torch.library; fake kernels for shape inference, the
backward as the forward's autograd formula), whose CUDA implementations call
the C ABI of ``libfna2_b200.so`` (include/fna2.h) to hand-written sm_100a
kernels; there is no Triton, no eager fallback and no CPU path.  Tensors must
live on a CUDA device.
"""
from __future__ import annotations

import ctypes
import math
from typing import Optional, Tuple

import torch

from . import _lib

BLOCK_M = 128  # query rows per tile
BLOCK_N = 128  # key rows per tile
BLOCK_R = 32   # rank advertised to NaylisAttention (attention_fna2.py:51,225)

SUPPORTED_RANKS = (8, 16, 24, 32)
SUPPORTED_HEAD_DIMS = (64, 128)


# ---------------------------------------------------------------------------
# descriptors
# ---------------------------------------------------------------------------

def _tma_ok(t: torch.Tensor) -> bool:
    """Column stride 1, other strides multiples of 8 elements, 16-B aligned base."""
    if t.numel() == 0:
        return True
    if t.stride(-1) != 1 or t.data_ptr() % 16:
        return False
    return all(s % 8 == 0 for d, s in zip(t.shape[:-1], t.stride()[:-1]) if d > 1)


def _prep(t: torch.Tensor) -> torch.Tensor:
    return t if _tma_ok(t) else t.clone(memory_format=torch.contiguous_format)


def _desc(t: Optional[torch.Tensor], varlen: bool) -> _lib.Fna2Tensor:
    d = _lib.Fna2Tensor()
    if t is None or t.numel() == 0:
        d.ptr = None
        d.stride[:] = (0, 0, 0, 1)
        return d
    d.ptr = t.data_ptr()
    s = t.stride()
    d.stride[:] = (0, s[1], s[0], s[2]) if varlen else (s[0], s[1], s[2], s[3])
    return d


def _problem(q, k, r_q, softmax_scale, is_causal, cu_q, cu_k, max_q, max_k) -> _lib.Fna2Problem:
    p = _lib.Fna2Problem()
    varlen = cu_q is not None
    if varlen:
        tq, h, d = q.shape
        tk, hkv = k.shape[0], k.shape[1]
        p.batch = cu_q.shape[0] - 1
        # max_seqlen bounds the grid; 0 (the signature default) means "unknown",
        # which the total token count safely bounds without a host sync
        p.seqlen_q = int(max_q) if max_q and max_q > 0 else tq
        p.seqlen_k = int(max_k) if max_k and max_k > 0 else tk
        p.total_q, p.total_k = tq, tk
        hg, r = r_q.shape[1], r_q.shape[2]
    else:
        b, h, s, d = q.shape
        hkv = k.shape[1]
        p.batch, p.seqlen_q, p.seqlen_k = b, s, k.shape[2]
        p.total_q = p.total_k = 0
        hg, r = r_q.shape[1], r_q.shape[3]
    p.heads, p.heads_kv, p.heads_graph, p.head_dim = h, hkv, hg, d
    p.rank = r if hg > 0 else 16
    p.softmax_scale = float(softmax_scale)
    p.causal = 1 if (is_causal or varlen) else 0
    p.cu_seqlens_q = cu_q.data_ptr() if varlen else None
    p.cu_seqlens_k = cu_k.data_ptr() if varlen else None
    return p


def _stream() -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _validate(q, k, v, r_q, r_k, graph_scale, cu_q, cu_k):
    # meta tensors carry shapes only (tracing, shape inference); data must be on a CUDA device
    if q.device.type not in ("cuda", "meta"):
        raise RuntimeError("flash_naylis_attn: tensors must be on a CUDA device (no CPU implementation)")
    dev = q.device
    for name, t in (("k", k), ("v", v), ("r_q", r_q), ("r_k", r_k), ("graph_scale", graph_scale)):
        if t.device != dev:
            raise RuntimeError(f"flash_naylis_attn: {name} is on {t.device}, q on {dev}")
    for name, t in (("q", q), ("k", k), ("v", v)):
        if t.dtype != torch.bfloat16:
            raise AssertionError(f"{name} must be bfloat16 (got {t.dtype})")
    varlen = cu_q is not None
    nd = 3 if varlen else 4
    for name, t in (("q", q), ("k", k), ("v", v), ("r_q", r_q), ("r_k", r_k)):
        if t.dim() != nd:
            raise AssertionError(f"{name} must be {nd}-D for {'varlen' if varlen else 'dense'} mode")
    d = q.shape[-1]
    if d not in SUPPORTED_HEAD_DIMS:
        raise AssertionError(f"head_dim must be 64 or 128 (got {d})")
    hg = r_q.shape[1]
    if hg > 0 and r_q.shape[-1] not in SUPPORTED_RANKS:
        raise AssertionError(f"rel_rank must be one of {SUPPORTED_RANKS} (got {r_q.shape[-1]})")
    if r_k.shape[1] != hg:
        raise AssertionError("r_q and r_k must have the same number of graph heads")
    if graph_scale.numel() != hg:
        raise AssertionError(f"graph_scale must have H_G={hg} entries (got {graph_scale.numel()})")
    if varlen:
        if cu_k is None or cu_q.dtype != torch.int32 or cu_k.dtype != torch.int32:
            raise AssertionError("cu_seqlens_q/cu_seqlens_k must both be int32 tensors")
        if cu_q.shape != cu_k.shape:
            raise AssertionError("cu_seqlens_q and cu_seqlens_k must have the same length")


# ---------------------------------------------------------------------------
# launchers (the C-ABI calls)
# ---------------------------------------------------------------------------

def _events_arg(events):
    """ctypes array of raw cudaEvent_t handles (torch.cuda.Event, already created)."""
    if not events:
        return None, None
    arr = (ctypes.c_void_p * len(events))(*[e.cuda_event for e in events])
    return ctypes.cast(arr, ctypes.c_void_p), arr


def _fna2_forward(q, k, v, r_q, r_k, gs, softmax_scale, is_causal, cu_q=None, cu_k=None, max_q=0, max_k=0,
                  launch_events=None, out=None) -> Tuple[torch.Tensor, torch.Tensor]:
    """Forward launcher; replaces _fna2_forward / _fna2_forward_varlen
    (flash_naylis_attn.py:700-804).  Inputs must be TMA-addressable
    (``_prep``), ``gs`` fp32.  Returns (out, lse); lse is [B,H,S] dense or
    [H,T] packed (fp32).  ``out`` may be given (a TMA-addressable buffer)."""
    lib = _lib.load()
    varlen = cu_q is not None
    if out is None:
        out = torch.empty_like(q)
        if not _tma_ok(out):
            out = torch.empty(q.shape, dtype=q.dtype, device=q.device)
    if varlen:
        lse = torch.empty(q.shape[1], q.shape[0], dtype=torch.float32, device=q.device)
    else:
        lse = torch.empty(q.shape[0], q.shape[1], q.shape[2], dtype=torch.float32, device=q.device)
    a = _lib.Fna2FwdArgs()
    a.prob = _problem(q, k, r_q, softmax_scale, is_causal, cu_q, cu_k, max_q, max_k)
    a.q, a.k, a.v = _desc(q, varlen), _desc(k, varlen), _desc(v, varlen)
    a.r_q, a.r_k = _desc(r_q, varlen), _desc(r_k, varlen)
    a.graph_scale = gs.data_ptr() if gs.numel() else None
    a.out = _desc(out, varlen)
    a.lse = lse.data_ptr()
    a.launch_events, keep = _events_arg(launch_events)
    ws = None
    if varlen:  # the table of real query-tile pairs (caching allocator)
        ws_bytes = lib.fna2_fwd_workspace_size(ctypes.byref(a.prob))
        ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=q.device)
        a.workspace, a.workspace_bytes = ws.data_ptr(), ws.numel()
    _lib.check(lib.fna2_fwd(ctypes.byref(a), _stream()), "fna2_fwd")
    return out, lse


def _fna2_backward(dout, q, k, v, r_q, r_k, gs, out, lse, softmax_scale, is_causal, cu_q=None, cu_k=None,
                   max_q=0, max_k=0, launch_events=None, grads=None):
    """Backward launcher; replaces _fna2_backward / _fna2_backward_varlen
    (flash_naylis_attn.py:807-892, :1215-1300).  Inputs must be
    TMA-addressable, ``gs`` fp32.  Returns (dq, dk, dv, dr_q, dr_k, d_gs);
    ``grads`` may give the five bf16 gradient buffers."""
    lib = _lib.load()
    varlen = cu_q is not None
    dout = _prep(dout)
    if grads is None:
        grads = [torch.empty_like(t) for t in (q, k, v, r_q, r_k)]
    dq, dk, dv, dr_q, dr_k = grads
    hg = r_q.shape[1]
    d_gs = torch.empty(hg, dtype=torch.float32, device=q.device)
    a = _lib.Fna2BwdArgs()
    a.prob = _problem(q, k, r_q, softmax_scale, is_causal, cu_q, cu_k, max_q, max_k)
    ws_bytes = lib.fna2_bwd_workspace_size(ctypes.byref(a.prob))
    ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=q.device)
    a.q, a.k, a.v = _desc(q, varlen), _desc(k, varlen), _desc(v, varlen)
    a.r_q, a.r_k = _desc(r_q, varlen), _desc(r_k, varlen)
    a.graph_scale = gs.data_ptr() if gs.numel() else None
    a.out, a.dout = _desc(out, varlen), _desc(dout, varlen)
    a.lse = lse.data_ptr()
    a.dq, a.dk, a.dv = _desc(dq, varlen), _desc(dk, varlen), _desc(dv, varlen)
    a.dr_q, a.dr_k = _desc(dr_q, varlen), _desc(dr_k, varlen)
    a.d_graph_scale = d_gs.data_ptr() if hg else None
    a.workspace = ws.data_ptr()
    a.workspace_bytes = ws.numel()
    a.launch_events, keep = _events_arg(launch_events)
    _lib.check(lib.fna2_bwd(ctypes.byref(a), _stream()), "fna2_bwd")
    return dq, dk, dv, dr_q, dr_k, d_gs


# ---------------------------------------------------------------------------
# PyTorch custom ops fna2::fwd / fna2::bwd over the C ABI
# ---------------------------------------------------------------------------
# Registered with torch.library so that the op is a node of its own in
# torch.compile / export graphs (no graph break at the call), with fake
# (meta) kernels for shape inference and the backward registered as its
# autograd formula.  The real kernels run on CUDA devices only.

def _out_like(t: torch.Tensor) -> torch.Tensor:
    """Output buffer with ``t``'s layout (``empty_like``, as the reference's
    launchers allocate, flash_naylis_attn.py:722-723,835-840)."""
    return torch.empty_like(t)


def _kernel_view(buf: torch.Tensor) -> torch.Tensor:
    """The buffer itself when TMA can address it, else a contiguous stand-in
    whose result is copied back by _finish."""
    return buf if _tma_ok(buf) else torch.empty(buf.shape, dtype=buf.dtype, device=buf.device)


def _finish(buf: torch.Tensor, k: torch.Tensor) -> torch.Tensor:
    if k is not buf:
        buf.copy_(k)
    return buf


def _lse_shape(q: torch.Tensor, varlen: bool):
    return (q.shape[1], q.shape[0]) if varlen else (q.shape[0], q.shape[1], q.shape[2])


@torch.library.custom_op("fna2::fwd", mutates_args=(), device_types="cuda")
def fna2_fwd_op(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, r_q: torch.Tensor, r_k: torch.Tensor,
                graph_scale: torch.Tensor, softmax_scale: float, is_causal: bool,
                cu_seqlens_q: Optional[torch.Tensor], cu_seqlens_k: Optional[torch.Tensor],
                max_seqlen_q: int, max_seqlen_k: int) -> Tuple[torch.Tensor, torch.Tensor]:
    """Forward (flash_naylis_attn.py:700-804): returns (out, lse); out has q's
    shape, dtype and layout, lse is fp32 [B,H,S] dense or [H,T] packed."""
    gs = graph_scale.to(torch.float32).contiguous()
    qp, kp, vp, rqp, rkp = (_prep(t) for t in (q, k, v, r_q, r_k))
    out = _out_like(q)
    ko = _kernel_view(out)
    lse = _fna2_forward(qp, kp, vp, rqp, rkp, gs, softmax_scale, is_causal, cu_seqlens_q, cu_seqlens_k,
                        max_seqlen_q, max_seqlen_k, out=ko)[1]
    return _finish(out, ko), lse


@fna2_fwd_op.register_fake
def _fna2_fwd_fake(q, k, v, r_q, r_k, graph_scale, softmax_scale, is_causal, cu_seqlens_q, cu_seqlens_k,
                   max_seqlen_q, max_seqlen_k):
    return torch.empty_like(q), q.new_empty(_lse_shape(q, cu_seqlens_q is not None), dtype=torch.float32)


@torch.library.custom_op("fna2::bwd", mutates_args=(), device_types="cuda")
def fna2_bwd_op(dout: torch.Tensor, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, r_q: torch.Tensor,
                r_k: torch.Tensor, graph_scale: torch.Tensor, out: torch.Tensor, lse: torch.Tensor,
                softmax_scale: float, is_causal: bool, cu_seqlens_q: Optional[torch.Tensor],
                cu_seqlens_k: Optional[torch.Tensor], max_seqlen_q: int, max_seqlen_k: int
                ) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    """Backward (flash_naylis_attn.py:807-892, :1215-1300): returns
    (dq, dk, dv, dr_q, dr_k, d_graph_scale), each in its input's dtype and
    layout."""
    gs = graph_scale.to(torch.float32).contiguous()
    # dout.contiguous() in the reference (:1355); here only when TMA cannot read it
    dp, qp, kp, vp, rqp, rkp, op = (_prep(t) for t in (dout, q, k, v, r_q, r_k, out))
    bufs = [_out_like(t) for t in (q, k, v, r_q, r_k)]
    kv = [_kernel_view(b) for b in bufs]
    d_gs = _fna2_backward(dp, qp, kp, vp, rqp, rkp, gs, op, lse.contiguous(), softmax_scale, is_causal,
                          cu_seqlens_q, cu_seqlens_k, max_seqlen_q, max_seqlen_k, grads=kv)[5]
    dq, dk, dv, dr_q, dr_k = (_finish(b, x) for b, x in zip(bufs, kv))
    return dq, dk, dv, dr_q, dr_k, d_gs.to(graph_scale.dtype)


@fna2_bwd_op.register_fake
def _fna2_bwd_fake(dout, q, k, v, r_q, r_k, graph_scale, out, lse, softmax_scale, is_causal, cu_seqlens_q,
                   cu_seqlens_k, max_seqlen_q, max_seqlen_k):
    return (torch.empty_like(q), torch.empty_like(k), torch.empty_like(v), torch.empty_like(r_q),
            torch.empty_like(r_k), torch.empty_like(graph_scale))


def _fwd_setup_context(ctx, inputs, output):
    (q, k, v, r_q, r_k, graph_scale, softmax_scale, is_causal, cu_q, cu_k, max_q, max_k) = inputs
    out, lse = output
    ctx.save_for_backward(q, k, v, r_q, r_k, graph_scale, out, lse, cu_q, cu_k)
    ctx.softmax_scale = softmax_scale
    ctx.is_causal = is_causal
    ctx.max_seqlen_q = max_q
    ctx.max_seqlen_k = max_k


def _fwd_backward(ctx, dout, dlse):
    # lse is an auxiliary output; its gradient is not propagated (the
    # reference's autograd Function returns out only, :1340)
    q, k, v, r_q, r_k, graph_scale, out, lse, cu_q, cu_k = ctx.saved_tensors
    grads = torch.ops.fna2.bwd(dout, q, k, v, r_q, r_k, graph_scale, out, lse, ctx.softmax_scale, ctx.is_causal,
                               cu_q, cu_k, ctx.max_seqlen_q, ctx.max_seqlen_k)
    return tuple(grads) + (None,) * 6


fna2_fwd_op.register_autograd(_fwd_backward, setup_context=_fwd_setup_context)


# ---------------------------------------------------------------------------
# autograd Function and public op
# ---------------------------------------------------------------------------

class FlashNaylisAttnFunc(torch.autograd.Function):
    """Autograd wrapper with the reference's name and call signature
    (flash_naylis_attn.py:1307-1373): ``apply(q, k, v, r_q, r_k, graph_scale,
    softmax_scale, is_causal, cu_seqlens_q, cu_seqlens_k, max_seqlen_q,
    max_seqlen_k)`` returns ``out``; backward returns six gradients and six
    ``None``.  Both directions run the fna2::fwd / fna2::bwd custom ops."""

    @staticmethod
    def forward(ctx, q, k, v, r_q, r_k, graph_scale, softmax_scale: float, is_causal: bool,
                cu_seqlens_q=None, cu_seqlens_k=None, max_seqlen_q: int = 0, max_seqlen_k: int = 0):
        out, lse = torch.ops.fna2.fwd(q, k, v, r_q, r_k, graph_scale, softmax_scale, is_causal,
                                      cu_seqlens_q, cu_seqlens_k, max_seqlen_q, max_seqlen_k)
        ctx.save_for_backward(q, k, v, r_q, r_k, graph_scale, out, lse)
        ctx.args = (softmax_scale, is_causal, cu_seqlens_q, cu_seqlens_k, max_seqlen_q, max_seqlen_k)
        return out

    @staticmethod
    def backward(ctx, dout):
        q, k, v, r_q, r_k, graph_scale, out, lse = ctx.saved_tensors
        grads = torch.ops.fna2.bwd(dout, q, k, v, r_q, r_k, graph_scale, out, lse, *ctx.args)
        return tuple(grads) + (None,) * 6


def flash_naylis_attn(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    r_q: torch.Tensor,
    r_k: torch.Tensor,
    graph_scale: torch.Tensor,
    softmax_scale: Optional[float] = None,
    is_causal: bool = True,
    cu_seqlens_q: Optional[torch.Tensor] = None,
    cu_seqlens_k: Optional[torch.Tensor] = None,
    max_seqlen_q: int = 0,
    max_seqlen_k: int = 0,
) -> torch.Tensor:
    """FlashNaylisAttention-2 public op (flash_naylis_attn.py:1380-1434).

    q, k, v      : dense [B,H,S,D] / [B,H_KV,S,D], or packed [T,H,D] / [T,H_KV,D]
    r_q, r_k     : dense [B,H_G,S,r] or packed [T,H_G,r], bfloat16
    graph_scale  : [H_G] (fp32; gradients are returned in its dtype)
    softmax_scale: 1/sqrt(head_dim) when None (:1415-1416)
    is_causal    : dense only; packed (varlen) calls are always causal
    cu_seqlens_* : int32 [N+1] cumulative lengths (varlen mode when given)
    max_seqlen_* : upper bounds of the packed lengths (0 = unknown)

    Returns ``out`` with q's shape and dtype.  Runs the fna2::fwd custom op
    (autograd: fna2::bwd), so it traces into torch.compile graphs without a
    break.
    """
    if softmax_scale is None:
        softmax_scale = 1.0 / math.sqrt(q.shape[-1])
    # the graph bias must stay in bf16 (flash_naylis_attn.py:1419-1420)
    assert r_q.dtype == torch.bfloat16, "r_q must be bfloat16"
    assert r_k.dtype == torch.bfloat16, "r_k must be bfloat16"
    _validate(q, k, v, r_q, r_k, graph_scale, cu_seqlens_q, cu_seqlens_k)
    out, _ = torch.ops.fna2.fwd(q, k, v, r_q, r_k, graph_scale, float(softmax_scale), bool(is_causal),
                                cu_seqlens_q, cu_seqlens_k, int(max_seqlen_q or 0), int(max_seqlen_k or 0))
    return out
