"""Host-side logic of the multi-GPU path on CPU: LPT partition, per-rank
scatter of packed sequences, gather of results and the d_gs sum, run as two
gloo ranks with the CPU oracle standing in for the per-rank kernel."""
import os

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from fna2_b200 import partition as PT


def test_lpt_balances_config5():
    L = PT.loguniform_lengths(512, 128, 16384, seed=0)
    for w in (1, 2, 4, 8):
        parts = PT.lpt_partition(L, w)
        assert sorted(i for p in parts for i in p) == list(range(512))
        assert PT.imbalance(L, parts) < 1.01


def test_scatter_gather_roundtrip():
    L = [5, 1, 9, 3, 7]
    x = torch.arange(sum(L) * 2).view(-1, 2)
    parts = PT.lpt_partition(L, 3)
    locs = [PT.scatter_rows(x, L, parts, r) for r in range(3)]
    assert sum(t.shape[0] for t in locs) == sum(L)
    assert torch.equal(PT.gather_rows(locs, L, parts), x)


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from oracle import fna2_oracle as O
        L = [17, 3, 40, 9, 25]
        H, D, r = 2, 16, 8
        qq, k, v, rq, rk, gs, do, cu = O.make_varlen_inputs(L, H, D, r, seed=5, gs_value="randn")
        parts = PT.lpt_partition(L, world)
        mine = [L[i] for i in parts[rank]]
        cu_l = PT.cu_seqlens(mine)
        loc = [PT.scatter_rows(t.double(), L, parts, rank) for t in (qq, k, v, rq, rk, do)]
        out, lse = O.varlen_fwd(*loc[:5], gs.double(), cu_l, cu_l, 0.25)
        grads = O.varlen_bwd(*loc[:5], gs.double(), out, lse, loc[5], cu_l, cu_l, 0.25)
        dgs = grads[5].clone()
        dist.all_reduce(dgs)
        # gather variable-size shards: pad to the largest token count
        n = torch.tensor([out.shape[0]])
        ns = [torch.zeros(1, dtype=torch.long) for _ in range(world)]
        dist.all_gather(ns, n)
        mx = int(max(x.item() for x in ns))
        pad = lambda t: torch.cat([t, t.new_zeros((mx - t.shape[0],) + tuple(t.shape[1:]))])
        res = {}
        for name, t in (("out", out), ("dq", grads[0]), ("dk", grads[1])):
            bufs = [torch.zeros((mx,) + tuple(t.shape[1:]), dtype=t.dtype) for _ in range(world)]
            dist.all_gather(bufs, pad(t))
            res[name] = PT.gather_rows([b[: int(c.item())] for b, c in zip(bufs, ns)], L, parts)
        if rank == 0:
            full_out, full_lse = O.varlen_fwd(qq.double(), k.double(), v.double(), rq.double(), rk.double(),
                                              gs.double(), cu, cu, 0.25)
            fg = O.varlen_bwd(qq.double(), k.double(), v.double(), rq.double(), rk.double(), gs.double(),
                              full_out, full_lse, do.double(), cu, cu, 0.25)
            ok = (torch.allclose(res["out"], full_out) and torch.allclose(res["dq"], fg[0])
                  and torch.allclose(res["dk"], fg[1]) and torch.allclose(dgs, fg[5]))
            q.put(bool(ok))
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_reassemble_the_single_process_result():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29500 + os.getpid() % 1000
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert q.get(timeout=5) is True


def _oracle_fwd_bwd(ins, cu_g, msl, scale):
    """The CPU oracle in the role of one GPU's fwd + bwd, with the kernels'
    output dtypes (bf16 tensors, fp32 d_gs)."""
    from oracle import fna2_oracle as O
    cu = cu_g.tolist()
    q, k, v, rq, rk, do = (t.double() for t in ins)
    gs = torch.ones(q.shape[1], dtype=torch.float64)
    out, lse = O.varlen_fwd(q, k, v, rq, rk, gs, cu, cu, scale)
    g = O.varlen_bwd(q, k, v, rq, rk, gs, out, lse, do, cu, cu, scale)
    return tuple(t.to(torch.bfloat16) for t in (out,) + g[:5]) + (g[5].float(),)


def _dataplane_worker(rank, world, port, q, plant):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import bench
        L = [17, 3, 40, 9, 25, 1, 12]
        H, D, r = 2, 16, 8
        parts = PT.lpt_partition(L, world)
        mine = [L[i] for i in parts[rank]]
        shard = bench.scatter_batch(dist, L, parts, rank, world, H, D, r, "cpu")
        # the shard is exactly the global batch's rows of this rank's sequences
        assert all(torch.equal(a, b) for a, b in zip(shard, bench.build_rows(L, parts[rank], H, D, r, "cpu")))
        cu_l = torch.tensor(PT.cu_seqlens(mine), dtype=torch.int32)
        res = _oracle_fwd_bwd(shard, cu_l, max(mine), 0.25)
        results = list(res[:6])
        if plant and rank == 1:  # a mistake planted in one rank's result must be caught
            results[2] = results[2].clone()
            results[2][0, 0, 0] += 1.0
        chk = bench.check_sharding(dist, results, res[6], L, parts, rank, world, H, D, r, "cpu", 0.25, n_groups=3,
                                   compute=_oracle_fwd_bwd)
        if rank == 0:
            q.put(chk)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("plant", [False, True])
def test_bench_dataplane_scatter_gather_check(plant):
    """bench.py's multi-GPU data plane on two gloo ranks: rank 0 builds the
    seeded global batch and sends each rank its shard; the gathered results
    equal one process's results for the global packing bit for bit, and
    d_gs's all-reduce equals the single-process sum; a planted mistake is
    reported."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29600 + os.getpid() % 1000 + (7 if plant else 0)
    procs = [ctx.Process(target=_dataplane_worker, args=(r, 2, port, q, plant)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=180)
        assert p.exitcode == 0
    chk = q.get(timeout=5)
    assert chk["per_sequence_bitwise"] is (not plant), chk
    assert chk["d_gs_max_rel_err"] < 1e-5, chk
