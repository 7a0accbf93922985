"""The drop-in boundary is registered with PyTorch as the custom ops
fna2::fwd and fna2::bwd: schemas, shape inference through their fake kernels
(meta tensors, no GPU needed), the registered autograd formula and
torch.compile(fullgraph=True) tracing without a graph break."""
import torch

import fna2_b200  # noqa: F401  (registers the ops)
from fna2_b200 import flash_naylis_attn


def _meta(*shape, dtype=torch.bfloat16):
    return torch.empty(*shape, device="meta", dtype=dtype).requires_grad_(True)


def test_schemas():
    f = str(torch.ops.fna2.fwd.default._schema)
    b = str(torch.ops.fna2.bwd.default._schema)
    assert f.startswith("fna2::fwd(Tensor q, Tensor k, Tensor v, Tensor r_q, Tensor r_k, Tensor graph_scale, "
                        "float softmax_scale, bool is_causal, Tensor? cu_seqlens_q, Tensor? cu_seqlens_k, "
                        "SymInt max_seqlen_q, SymInt max_seqlen_k) -> (Tensor, Tensor)"), f
    assert b.startswith("fna2::bwd(Tensor dout, Tensor q, Tensor k, Tensor v"), b
    assert b.endswith("-> (Tensor, Tensor, Tensor, Tensor, Tensor, Tensor)"), b


def test_fake_shapes_dense_and_grads():
    q, k, v = _meta(2, 4, 64, 128), _meta(2, 2, 64, 128), _meta(2, 2, 64, 128)
    rq, rk = _meta(2, 3, 64, 16), _meta(2, 3, 64, 16)
    gs = _meta(3, dtype=torch.float32)
    out = flash_naylis_attn(q, k, v, rq, rk, gs)
    assert out.shape == q.shape and out.dtype == torch.bfloat16
    _, lse = torch.ops.fna2.fwd(q, k, v, rq, rk, gs, 0.1, True, None, None, 0, 0)
    assert lse.shape == (2, 4, 64) and lse.dtype == torch.float32
    out.sum().backward()
    for t in (q, k, v, rq, rk, gs):
        assert t.grad.shape == t.shape and t.grad.dtype == t.dtype


def test_fake_shapes_packed_lse_layout():
    q, k, v = _meta(300, 4, 64), _meta(300, 4, 64), _meta(300, 4, 64)
    rq, rk = _meta(300, 4, 16), _meta(300, 4, 16)
    gs = _meta(4, dtype=torch.bfloat16)
    cu = torch.empty(3, device="meta", dtype=torch.int32)
    out, lse = torch.ops.fna2.fwd(q, k, v, rq, rk, gs, 0.125, True, cu, cu, 200, 200)
    assert out.shape == q.shape and lse.shape == (4, 300)
    out.float().sum().backward()
    assert gs.grad.dtype == torch.bfloat16  # d_graph_scale in graph_scale's dtype (:1373)


def test_compile_fullgraph_without_graph_break():
    q, k, v = _meta(256, 4, 128), _meta(256, 2, 128), _meta(256, 2, 128)
    rq, rk = _meta(256, 4, 16), _meta(256, 4, 16)
    gs = _meta(4, dtype=torch.float32)
    cu = torch.empty(5, device="meta", dtype=torch.int32)

    def f(q, k, v, rq, rk, gs, cu):
        o = flash_naylis_attn(q, k, v, rq, rk, gs, cu_seqlens_q=cu, cu_seqlens_k=cu, max_seqlen_q=128,
                              max_seqlen_k=128)
        return o.float().square().mean()

    ex = torch._dynamo.explain(f)(q, k, v, rq, rk, gs, cu)
    assert ex.graph_break_count == 0 and ex.graph_count == 1
    torch._dynamo.reset()
    loss = torch.compile(f, fullgraph=True, backend="aot_eager")(q, k, v, rq, rk, gs, cu)
    loss.backward()
    assert q.grad.shape == q.shape and gs.grad.shape == gs.shape
