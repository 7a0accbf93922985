#!/usr/bin/env python3
"""Benchmark of the FNA2 hot path: varlen causal fwd+bwd TFLOP/s on B200.

Default workload (the metric's 1/2/4/8-GPU case): 512 packed
sequences with lengths log-uniform in [128, 16384] (seeded), H = 32 heads (all
graph heads), head_dim 128, rank 16, bf16, causal, gs = 1.  At N GPUs the
sequences are LPT-partitioned by FLOPs across ranks (whole sequences per rank,
no collective on the data path): total work is fixed, so scaling is "strong".

One step = forward + backward of every sequence a rank owns.  ``value`` is
total algorithmic FLOPs of the whole batch / max-over-ranks step time (device
resident inputs); ``e2e`` is the same metric through the public API
(``flash_naylis_attn`` + ``backward``) with the step's inputs copied from
pinned host memory and d_graph_scale read back every step; the sequences go
through in 8 groups so that one group's host-to-device copy (PCIe) overlaps
the previous group's compute.

``--impl reference`` times the reference's eager path restated on the CPU
(oracle/fna2_oracle.py: materialised bias + SDPA + autograd, fp32, all host
threads) on a bounded sample of the same workload.

``--op qk_prep`` instead measures the fused varlen QK-RMSNorm + RoPE transform
(fna2_b200/qk_prep.py) forward + backward on the workload's q and k (bf16,
H_KV = H), as HBM GB/s against the measured copy bandwidth, with the
reference's per-sequence CPU path (oracle/qk_prep_oracle.py) timed beside it.

``--op decode`` measures one KV-cache decode step with the relational bias
(fna2_b200/decode.py) for every sequence of the workload at once: each
sequence's cache holds its L tokens (packed caches, K/V/R_k), one new token
per sequence is appended and attends to L + 1 keys; HBM GB/s of the step
against the measured copy bandwidth, with the decode oracle
(oracle/decode_oracle.py) timed on the host beside it.

``--op rel_proj`` measures the fused R_q/R_k projection (fna2_b200/rel_proj.py:
the library's tcgen05 GEMM over the stacked weights for Y, dX and dW, strided
views out) forward + backward on the workload's tokens (x [T, H*D] bf16), with
the reference's two-Linear composition timed on the same GPU beside it.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

from fna2_b200 import flops as FL  # noqa: E402
from fna2_b200 import partition as PT  # noqa: E402

METRIC = "fwd+bwd TFLOP/s (bf16, varlen causal, d=128, r=16)"


# ---------------------------------------------------------------------------
# workloads
# ---------------------------------------------------------------------------

def workload(name: str):
    if name == "cfg5":
        return dict(name="cfg5", lengths=PT.loguniform_lengths(512, 128, 16384, seed=0), H=32, D=128, r=16,
                    desc="BASELINE config 5: 512 packed seqs, L log-uniform [128,16384] (seed 0), H32 D128 r16, "
                         "causal bf16, gs=1")
    if name == "cfg3":
        return dict(name="cfg3", lengths=PT.uniform_int_lengths(16, 64, 4096, seed=0), H=16, D=128, r=16,
                    desc="BASELINE config 3: 16 packed seqs, L uniform-int [64,4096] (seed 0), H16 D128 r16")
    if name == "cfg2":
        return dict(name="cfg2", lengths=[2048] * 8, H=16, D=128, r=16,
                    desc="BASELINE config 2 as 8 packed sequences of 2048: H16 D128 r16")
    if name == "cfg4":
        return dict(name="cfg4", lengths=[32768], H=32, D=128, r=32,
                    desc="BASELINE config 4: one sequence of 32768, H32 D128 r32")
    if name == "cfg5short":
        lengths = [L for L in PT.loguniform_lengths(512, 128, 16384, seed=0) if L <= 512]
        return dict(name="cfg5short", lengths=lengths, H=32, D=128, r=16,
                    desc=f"BASELINE config 5's sequences with L <= 512 ({len(lengths)} seqs): the short-sequence "
                         "regime, H32 D128 r16")
    if name.startswith("seqs:"):
        # seqs:N:L:H:r -- N packed sequences of L tokens (profiling and small cases)
        n, L, H, r = (int(x) for x in name.split(":")[1:])
        return dict(name=name, lengths=[L] * n, H=H, D=128, r=r,
                    desc=f"{n} packed sequences of {L}, H{H} D128 r{r}, causal bf16, gs=1")
    raise ValueError(name)


# ---------------------------------------------------------------------------
# clocks sampled during the timed region
# ---------------------------------------------------------------------------

class ClockSampler:
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def start(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        rows = []
        with open(self.path) as f:
            for line in f:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) >= 9:
                    rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = max(float(r[2]) for r in rows if r[2].replace(".", "").isdigit())
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        load = [s for s in sm if s > 0.5 * mx] or sm
        return {"sm_mhz": statistics.median(load), "sm_max_mhz": mx, "reasons": reasons, "samples": len(rows)}


# ---------------------------------------------------------------------------
# CPU baseline: the reference's eager path (restated) on the host cores
# ---------------------------------------------------------------------------

def cpu_sample(w, budget_s: float, max_len: int = 2048):
    """Time the fp32 eager oracle (fwd + autograd bwd) on whole sequences of the
    workload (those with L <= max_len, in order) until ``budget_s`` is spent."""
    from oracle import fna2_oracle as O
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    H, D, r = w["H"], w["D"], w["r"]
    scale = 1.0 / math.sqrt(D)

    def one(L, seed):
        q, k, v, rq, rk, gs, do = O.make_dense_inputs(1, H, L, D, r, seed=seed)
        ts = [t.requires_grad_(True) for t in (q, k, v, rq, rk, gs)]
        out = O.sdpa_reference(*ts, scale, True)
        out.backward(do)

    one(128, 0)  # warm-up
    done, flops, t0 = [], 0.0, time.perf_counter()
    for i, L in enumerate(w["lengths"]):
        if L > max_len:
            continue
        one(L, i)
        done.append(L)
        flops += FL.total_flops([L], H, H, D, r)
        if time.perf_counter() - t0 > budget_s:
            break
    dt = time.perf_counter() - t0
    return {"value": flops / dt / 1e12, "unit": "TFLOP/s", "cores": threads, "kind": "port",
            "sample": f"{len(done)} whole sequences of the workload with L<=2048 (sum L={sum(done)}), "
                      f"fp32 eager fwd+bwd (materialised bias + SDPA + autograd), {dt:.1f} s"}


def run_reference(args, w):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    budget = 4.0
    vals = []
    for _ in range(args.warmup):
        cpu_sample(w, 1.0)
    for _ in range(args.steps):
        vals.append(cpu_sample(w, budget))
    v = statistics.median([x["value"] for x in vals])
    last = vals[-1]
    line = {
        "impl": "reference", "metric": METRIC, "value": v, "unit": "TFLOP/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": None, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": w["desc"], "sample": last["sample"]},
        "cpu_baseline": {"value": v, "unit": "TFLOP/s", "cores": last["cores"], "kind": "port",
                         "sample": last["sample"]},
        "e2e": {"value": v, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------

def build_rows(lengths, seqs, H, D, r, dev, seed=1000):
    """Packed inputs (q, k, v, r_q, r_k, dO) of the sequences ``seqs`` in that
    order.  Sequence i is drawn from its own generator (seed + i), so the
    global batch and any subset of it (a rank's shard, a check group) hold
    identical rows: Q, K, V, dO ~ N(0, 1), R ~ N(0, 1/r), bf16."""
    n = sum(int(lengths[i]) for i in seqs)
    ts = [torch.empty(n, H, D, device=dev, dtype=torch.bfloat16) for _ in range(3)]
    ts += [torch.empty(n, H, r, device=dev, dtype=torch.bfloat16) for _ in range(2)]
    ts += [torch.empty(n, H, D, device=dev, dtype=torch.bfloat16)]
    off = 0
    for i in seqs:
        L = int(lengths[i])
        g = torch.Generator(device=torch.device(dev).type).manual_seed(seed + i)
        for j, t in enumerate(ts):
            t[off:off + L].normal_(0.0, r ** -0.5 if j in (3, 4) else 1.0, generator=g)
        off += L
    return ts


def scatter_batch(dist, lengths, parts, rank, world, H, D, r, dev):
    """Rank 0 builds the seeded global batch and sends every rank its packed
    shard over NCCL (outside the timed region); returns this rank's shard."""
    if world == 1:
        return build_rows(lengths, parts[0], H, D, r, dev)
    n_me = sum(int(lengths[i]) for i in parts[rank])
    if rank == 0:
        glob = build_rows(lengths, range(len(lengths)), H, D, r, dev)
        for dst in range(1, world):
            idx = torch.tensor(PT.shard_token_index(lengths, parts[dst]), dtype=torch.long, device=dev)
            for t in glob:
                stage = t.index_select(0, idx)
                dist.send(stage, dst)
                del stage
        idx = torch.tensor(PT.shard_token_index(lengths, parts[0]), dtype=torch.long, device=dev)
        mine = [t.index_select(0, idx) for t in glob]
        del glob
        torch.cuda.empty_cache()
        return mine
    mine = [torch.empty((n_me, H, X), device=dev, dtype=torch.bfloat16) for X in (D, D, D, r, r, D)]
    for t in mine:
        dist.recv(t, 0)
    return mine


def cuda_fwd_bwd(ins, cu_g, msl, scale):
    """Forward + backward of one packed batch through the library's launchers:
    (out, dq, dk, dv, dr_q, dr_k, d_gs)."""
    from fna2_b200.flash_naylis_attn import _fna2_backward, _fna2_forward
    gs = torch.ones(ins[0].shape[1], device=ins[0].device)
    out, lse = _fna2_forward(*ins[:5], gs, scale, True, cu_g, cu_g, msl, msl)
    return (out,) + tuple(_fna2_backward(ins[5], *ins[:5], gs, out, lse, scale, True, cu_g, cu_g, msl, msl))


def check_sharding(dist, results, dgs_local, lengths, parts, rank, world, H, D, r, dev, scale, n_groups=16,
                   compute=cuda_fwd_bwd):
    """Gather every rank's O and gradients to rank 0, group by group of
    sequences in the global packing, and compare them with one GPU's result
    for the same rows: the group recomputed on rank 0 from the seeded global
    batch (``compute``).  Per-sequence tensors must agree bit for bit (a
    sequence's tiles do not depend on where it is packed); the all-reduced
    d_graph_scale must equal the single-GPU sum up to fp32 summation order."""
    own = PT.owner_of(parts)
    cu = PT.cu_seqlens(lengths)
    widths = [D, D, D, D, r, r]  # out, dq, dk, dv, dr_q, dr_k
    dgs_all = dgs_local.clone()
    if world > 1:
        dist.all_reduce(dgs_all)
    dgs_ref = torch.zeros(H, dtype=torch.float64, device=dev)
    bitwise, worst = True, 0.0
    for a, b in PT.sequence_groups(lengths, n_groups):
        seqs = list(range(a, b))
        mine = [i for i in seqs if own[i] == rank]
        if rank != 0:
            if mine:
                rows = torch.tensor(PT.local_rows_of(lengths, parts[rank], mine), dtype=torch.long, device=dev)
                flat = torch.cat([t.index_select(0, rows).reshape(-1) for t in results])
                dist.send(flat, 0)
                del flat
            continue
        ins = build_rows(lengths, seqs, H, D, r, dev)
        cu_g = torch.tensor([c - cu[a] for c in cu[a:b + 1]], dtype=torch.int32, device=dev)
        msl = max(int(lengths[i]) for i in seqs)
        res_g = compute(ins, cu_g, msl, scale)
        ref = list(res_g[:6])
        dgs_ref += res_g[6].double()
        got = [torch.empty_like(x) for x in ref]
        for src in range(world):
            rs = [i for i in seqs if own[i] == src]
            if not rs:
                continue
            g_rows = torch.tensor([j for i in rs for j in range(cu[i] - cu[a], cu[i + 1] - cu[a])],
                                  dtype=torch.long, device=dev)
            n = g_rows.numel()
            if src == 0:
                loc = torch.tensor(PT.local_rows_of(lengths, parts[0], rs), dtype=torch.long, device=dev)
                pieces = [t.index_select(0, loc) for t in results]
            else:
                flat = torch.empty(n * H * sum(widths), device=dev, dtype=torch.bfloat16)
                dist.recv(flat, src)
                pieces, o = [], 0
                for wd in widths:
                    pieces.append(flat[o:o + n * H * wd].view(n, H, wd))
                    o += n * H * wd
            for gt, pc in zip(got, pieces):
                gt.index_copy_(0, g_rows, pc)
        for x, y in zip(ref, got):
            if not torch.equal(x, y):
                bitwise = False
                worst = max(worst, (x.float() - y.float()).abs().max().item())
        del ins, res_g, ref, got
    if world > 1:
        dist.barrier()
    res = None
    if rank == 0:
        rel = ((dgs_all.double() - dgs_ref).abs().max() / dgs_ref.abs().max().clamp_min(1e-30)).item()
        res = {"ranks": world, "groups": n_groups, "per_sequence_bitwise": bitwise,
               "max_abs_diff": worst, "d_gs_max_rel_err": rel,
               "scatter": "rank 0 builds the seeded global batch, NCCL send/recv of each rank's packed shard",
               "gather": "NCCL send/recv of every rank's O and gradients to rank 0 by sequence group, compared "
                         "with rank 0's single-GPU result for the same rows; d_gs all_reduce(sum)"}
    return res


def run_gpu(args, w):
    import torch.distributed as dist
    from fna2_b200 import flash_naylis_attn
    from fna2_b200.flash_naylis_attn import _fna2_backward, _fna2_forward

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)

    H, D, r = w["H"], w["D"], w["r"]
    lengths = w["lengths"]
    parts = PT.lpt_partition(lengths, world)
    mine = [lengths[i] for i in parts[rank]]
    cu = PT.cu_seqlens(mine)
    T = cu[-1]
    flops_all = FL.total_flops(lengths, H, H, D, r)
    scale = 1.0 / math.sqrt(D)

    q, k, v, rq, rk, do = scatter_batch(dist, lengths, parts, rank, world, H, D, r, dev)
    gs = torch.ones(H, device=dev, dtype=torch.float32)
    cu_t = torch.tensor(cu, dtype=torch.int32, device=dev)
    msl = max(mine)
    stream = torch.cuda.current_stream()

    def mk_events(n):
        evs = [torch.cuda.Event(enable_timing=True) for _ in range(n)]
        for e in evs:
            e.record(stream)
        return evs

    def step(evf=None, evb=None):
        out, lse = _fna2_forward(q, k, v, rq, rk, gs, scale, True, cu_t, cu_t, msl, msl, launch_events=evf)
        grads = _fna2_backward(do, q, k, v, rq, rk, gs, out, lse, scale, True, cu_t, cu_t, msl, msl,
                               launch_events=evb)
        return out, grads

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])

    K, W = args.steps, args.warmup
    for _ in range(W):
        step()
    ev_f = [mk_events(2) for _ in range(K)]
    ev_b = [mk_events(4) for _ in range(K)]
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clocks = ClockSampler(local)
    barrier()
    torch.cuda.synchronize()
    clocks.start()
    t0.record(stream)
    for i in range(K):
        step()
    t1.record(stream)
    torch.cuda.synchronize()
    clk = clocks.stop()
    barrier()
    ms = t0.elapsed_time(t1) / K
    # per-kernel breakdown: K more steps with events recorded between the kernels
    # (kept out of the timed region, where they would add their own gaps)
    for i in range(K):
        step(ev_f[i], ev_b[i])
    torch.cuda.synchronize()
    ms_t = torch.tensor([ms], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(ms_t, op=dist.ReduceOp.MAX)
    ms_max = float(ms_t.item())
    value = flops_all / (ms_max / 1e3) / 1e12

    kern = {
        "fwd": statistics.mean(ev_f[i][0].elapsed_time(ev_f[i][1]) for i in range(K)),
        "bwd_pre": statistics.mean(ev_b[i][0].elapsed_time(ev_b[i][1]) for i in range(K)),
        "bwd_dkdv": statistics.mean(ev_b[i][1].elapsed_time(ev_b[i][2]) for i in range(K)),
        "bwd_dq": statistics.mean(ev_b[i][2].elapsed_time(ev_b[i][3]) for i in range(K)),
    }
    algo = {
        "fwd": FL.fwd_flops(mine, H, H, D, r),
        "bwd_dkdv": FL.dkdv_flops(mine, H, H, D, r),
        "bwd_dq": FL.dq_flops(mine, H, H, D, r),
    }
    dom = max(algo, key=lambda n: kern[n])
    peaks = {}
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            peaks = json.load(f)
    except Exception:
        pass
    peak = peaks.get("bf16_tflops_sustained")
    peak_src = "measured sustained"
    if peak is None:
        peak, peak_src = 1400.0, "fallback sustained"
    achieved = algo[dom] / (kern[dom] / 1e3) / 1e12
    traffic = None
    try:
        with open(os.path.join(ROOT, "profiles", "ncu_traffic.json")) as f:
            tr = json.load(f)
        per_tok = tr.get("per_token_head", {}).get(dom.replace("bwd_", ""))
        if per_tok is not None:
            traffic = per_tok * T * H
    except Exception:
        pass
    del ev_f, ev_b

    # ---------------- e2e through the public API with host buffers
    e2e, ceiling = None, None
    if not args.no_e2e:
        e2e, ceiling = run_e2e(args, dist, world, rank, local, dev, stream, q, k, v, rq, rk, do, gs, mine, cu,
                               H, D, r, scale, flops_all, barrier)

    # ---------------- the shards add up: gather, compare with one GPU's result
    check = None
    if not args.no_check:
        out, grads = step()
        results = [out] + list(grads[:5])
        dgs_local = grads[5]
        del q, k, v, rq, rk, do
        torch.cuda.synchronize()
        torch.cuda.empty_cache()
        check = check_sharding(dist, results, dgs_local, lengths, parts, rank, world, H, D, r, dev, scale)
        del results, out, grads

    from fna2_b200 import _lib
    status = _lib.load().fna2_device_status(0)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu = cpu_sample(w, args.cpu_budget)

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": K, "warmup": W,
            "ms_per_step": ms_max, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "bf16", "data": "synthetic",
            "config": {"workload": w["desc"], "total_tokens": sum(lengths), "sequences": len(lengths),
                       "parallelism": f"sequence-sharded LPT x{world} (no data-path collective)",
                       "l2": "inputs larger than L2 (no flush needed)" if sum(lengths) * H * D * 2 > 126e6
                       else "inputs smaller than L2: not flushed"},
            "roofline": {"bound": "tensor", "kernel": dom, "achieved": achieved, "peak": peak,
                         "peak_source": peak_src, "unit": "TFLOP/s", "frac": achieved / peak,
                         "traffic": traffic},
            "kernels_ms": kern,
            "e2e": e2e,
            "copy_ceiling": ceiling,
            "sharding_check": check,
            "gpu_launches": 5 * K,  # per step: forward tile table, forward, backward pre-pass, dK/dV, dQ
            "clocks": clk,
            "cpu_baseline": cpu,
            "device_status": status,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()


def run_e2e(args, dist, world, rank, local, dev, stream, q, k, v, rq, rk, do, gs, mine, cu, H, D, r, scale,
            flops_all, barrier):
    """The metric through the public API (flash_naylis_attn + backward) with
    host buffers: every step copies its inputs from pinned host memory and
    copies O and the five gradients (and d_graph_scale) back to pinned host
    memory.  The sequences go through in G groups on three streams, so that
    group g+1's inputs cross PCIe to the GPU while group g computes and group
    g-1's results cross back.  Also measures the copy ceiling of this host
    link alone: the same bytes in, out, and in and out at once, no compute."""
    from fna2_b200 import flash_naylis_attn
    K, W = args.steps, args.warmup
    T = cu[-1]
    torch.cuda.synchronize()
    # inputs (q, k, v, r_q, r_k, dO) and results (O, dq, dk, dv, dr_q, dr_k) in
    # page-locked host memory: one exact-size buffer per direction, registered
    # with cudaHostRegister (PyTorch's pinned allocator rounds every tensor up
    # to a power of two, ~10 GB more at config 5)
    pinned = []

    def host_tensors(like):
        nbytes = [t.numel() * t.element_size() for t in like]
        buf = torch.empty(sum(nbytes), dtype=torch.uint8)
        rc = torch.cuda.cudart().cudaHostRegister(buf.data_ptr(), buf.numel(), 0)
        if int(rc) != 0:
            raise RuntimeError(f"cudaHostRegister of {buf.numel()} bytes failed ({rc})")
        pinned.append(buf)
        views, off = [], 0
        for t, nb in zip(like, nbytes):
            views.append(buf[off:off + nb].view(t.dtype).view(t.shape))
            off += nb
        return views

    host_in = host_tensors([q, k, v, rq, rk, do])
    for h, t in zip(host_in, (q, k, v, rq, rk, do)):
        h.copy_(t)
    host_out = host_tensors([q, q, k, v, rq, rk])  # O, dq, dk, dv, dr_q, dr_k
    host_dgs = torch.empty(H, dtype=torch.float32, pin_memory=True)
    assert all(t.is_pinned() for t in host_in + host_out)
    h2d = sum(t.numel() * t.element_size() for t in host_in)
    d2h = sum(t.numel() * t.element_size() for t in host_out) + host_dgs.numel() * 4
    leaves = [q, k, v, rq, rk]   # device buffers the host inputs are copied into each step
    gsl = gs.clone().requires_grad_(True)
    G = 8
    bounds, acc_t = [0], 0
    for i, L in enumerate(mine):
        acc_t += L
        if acc_t >= T * len(bounds) / G and len(bounds) < G:
            bounds.append(i + 1)
    if bounds[-1] != len(mine):
        bounds.append(len(mine))
    groups = []
    for a, b in zip(bounds[:-1], bounds[1:]):
        t0g, t1g = cu[a], cu[b]
        cu_g = torch.tensor([c - t0g for c in cu[a:b + 1]], dtype=torch.int32, device=dev)
        groups.append((t0g, t1g, cu_g, max(mine[a:b])))
    copy_in = torch.cuda.Stream(device=dev)
    copy_out = torch.cuda.Stream(device=dev)
    done = [torch.cuda.Event() for _ in groups]
    for e in done:
        e.record(stream)

    def e2e_step():
        start = torch.cuda.Event()
        start.record(stream)
        copied = []
        with torch.cuda.stream(copy_in):
            copy_in.wait_event(start)
            for gi, (t0g, t1g, _, _) in enumerate(groups):
                copy_in.wait_event(done[gi])  # group gi's previous compute has read these buffers
                for dst, src in zip(leaves + [do], host_in):
                    dst[t0g:t1g].copy_(src[t0g:t1g], non_blocking=True)
                ev = torch.cuda.Event()
                ev.record(copy_in)
                copied.append(ev)
        gsl.grad = None
        keep = []
        for gi, (t0g, t1g, cu_g, msl_g) in enumerate(groups):
            stream.wait_event(copied[gi])
            ins = [t[t0g:t1g].detach().requires_grad_(True) for t in leaves]
            out = flash_naylis_attn(*ins, gsl, softmax_scale=scale, is_causal=True, cu_seqlens_q=cu_g,
                                    cu_seqlens_k=cu_g, max_seqlen_q=msl_g, max_seqlen_k=msl_g)
            out.backward(do[t0g:t1g])
            done[gi].record(stream)
            res = [out.detach()] + [x.grad for x in ins]
            with torch.cuda.stream(copy_out):
                copy_out.wait_event(done[gi])
                for dst, src in zip(host_out, res):
                    dst[t0g:t1g].copy_(src, non_blocking=True)
            keep.append(res)
        finish = torch.cuda.Event()
        with torch.cuda.stream(copy_out):
            copy_out.wait_event(done[-1])  # d_graph_scale is complete after the last group
            host_dgs.copy_(gsl.grad, non_blocking=True)
            finish.record(copy_out)
        stream.wait_event(finish)  # the step ends when its results are on the host
        return keep

    def timed(fn, n):
        barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(n):
            keep = fn()
            del keep
        e1.record(stream)
        torch.cuda.synchronize()
        barrier()
        t = torch.tensor([e0.elapsed_time(e1) / n], device=dev, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    for _ in range(W):
        del_keep = e2e_step()
        del del_keep
    ems = timed(e2e_step, K)
    nbytes = torch.tensor([h2d, d2h], device=dev, dtype=torch.float64)
    if world > 1:  # every rank copies its own shard: sum the bytes
        dist.all_reduce(nbytes)
    h2d_all, d2h_all = int(nbytes[0].item()), int(nbytes[1].item())
    e2e = {"value": flops_all / (ems / 1e3) / 1e12, "unit": "TFLOP/s",
           "h2d_bytes_per_step": h2d_all, "d2h_bytes_per_step": d2h_all, "ms_per_step": ems}

    # copy ceiling of the host link: the same bytes, the same group copies, no compute
    dev_out = [torch.empty(t.shape, dtype=t.dtype, device=dev) for t in host_out]

    def copies(inp, outp):
        def fn():
            ev = torch.cuda.Event()
            ev.record(stream)
            ends = []
            if inp:
                with torch.cuda.stream(copy_in):
                    copy_in.wait_event(ev)
                    for t0g, t1g, _, _ in groups:
                        for dst, src in zip(leaves + [do], host_in):
                            dst[t0g:t1g].copy_(src[t0g:t1g], non_blocking=True)
                    e = torch.cuda.Event()
                    e.record(copy_in)
                    ends.append(e)
            if outp:
                with torch.cuda.stream(copy_out):
                    copy_out.wait_event(ev)
                    for t0g, t1g, _, _ in groups:
                        for dst, src in zip(host_out, dev_out):
                            dst[t0g:t1g].copy_(src[t0g:t1g], non_blocking=True)
                    e = torch.cuda.Event()
                    e.record(copy_out)
                    ends.append(e)
            for e in ends:
                stream.wait_event(e)
            return None
        return fn

    n_c = max(1, min(K, 3))
    ms_in = timed(copies(True, False), n_c)
    ms_out = timed(copies(False, True), n_c)
    ms_both = timed(copies(True, True), n_c)
    ceiling = {"h2d_gbs": h2d_all / (ms_in / 1e3) / 1e9, "d2h_gbs": d2h_all / (ms_out / 1e3) / 1e9,
               "both_ms_per_step": ms_both, "both_gbs": (h2d_all + d2h_all) / (ms_both / 1e3) / 1e9,
               "e2e_over_ceiling_ms": ems / ms_both,
               "note": "the same bytes and group copies as e2e without compute, all ranks together "
                       "(time = max over ranks): the host link's ceiling for e2e"}
    e2e["copy_ceiling_fraction"] = ms_both / ems
    torch.cuda.synchronize()
    del dev_out, host_in, host_out
    for buf in pinned:
        torch.cuda.cudart().cudaHostUnregister(buf.data_ptr())
    return e2e, ceiling


def run_qk_prep(args, w):
    """Fused varlen QK-RMSNorm + RoPE, forward + backward, one GPU."""
    import types
    from fna2_b200.qk_prep import apply_qk_norm_rope_varlen
    from oracle import qk_prep_oracle as QO
    dev = "cuda"
    lengths, H, D = w["lengths"], w["H"], w["D"]
    T = sum(lengths)
    cu = torch.tensor([0] + list(torch.tensor(lengths).cumsum(0).tolist()), dtype=torch.int32, device=dev)
    g = torch.Generator(device=dev).manual_seed(0)
    q = torch.randn(T, H, D, device=dev, generator=g).bfloat16().requires_grad_(True)
    k = torch.randn(T, H, D, device=dev, generator=g).bfloat16().requires_grad_(True)
    norms = [types.SimpleNamespace(weight=torch.ones(D, device=dev, dtype=torch.bfloat16).requires_grad_(True),
                                   eps=1e-6) for _ in range(2)]
    rope = types.SimpleNamespace(inv_freq=QO.rope_inv_freq(D).to(dev))
    gq = torch.randn(T, H, D, device=dev, generator=g).bfloat16()
    gk = torch.randn(T, H, D, device=dev, generator=g).bfloat16()

    def step():
        # gradients set to None between steps (zero_grad(set_to_none=True)), so
        # autograd hands over dq/dk instead of adding them into earlier ones
        q.grad = k.grad = norms[0].weight.grad = norms[1].weight.grad = None
        qo, ko = apply_qk_norm_rope_varlen(q, k, cu, norms[0], norms[1], rope)
        torch.autograd.backward([qo, ko], [gq, gk])

    for _ in range(args.warmup):
        step()
    st = torch.cuda.current_stream()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clocks = ClockSampler(0)
    torch.cuda.synchronize()
    clocks.start()
    t0.record(st)
    for _ in range(args.steps):
        step()
    t1.record(st)
    torch.cuda.synchronize()
    clk = clocks.stop()
    ms = t0.elapsed_time(t1) / args.steps
    rows = T * 2 * H * D  # elements of q and k together
    # forward reads x (bf16) and writes y (bf16); backward reads x and dy, writes dx (all bf16)
    algo_bytes = rows * (2 + 2) + rows * (2 + 2 + 2)
    gbs = algo_bytes / (ms / 1e3) / 1e9
    peak = None
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            peak = json.load(f).get("hbm_gbs")
    except Exception:
        pass
    peak_src = "measured"
    if peak is None:
        peak, peak_src = 6650.0, "fallback"
    # CPU: the reference path restated (norm + per-sequence RoPE loop + autograd), fp32, sample of sequences
    cpu = None
    if not args.no_cpu:
        torch.set_num_threads(os.cpu_count())
        sample = []
        for L in lengths:  # whole short sequences of the workload, about 16k tokens
            if L <= 1024 and sum(sample) + L <= 16384:
                sample.append(L)
        qc, kc, wq, wk, inv, cuc, dqo, dko = QO.make_inputs(sample, H, H, D, 0)
        t_c = time.perf_counter()
        QO.qk_prep_with_grads(qc, kc, cuc, wq, wk, 1e-6, inv, dqo, dko)
        dt = time.perf_counter() - t_c
        cb = sum(sample) * 2 * H * D * (4 + 2 + 4 + 2 + 4)
        cpu = {"value": cb / dt / 1e9, "unit": "GB/s", "cores": os.cpu_count(), "kind": "port",
               "sample": f"{len(sample)} sequences of the workload with L<=1024 (sum L={sum(sample)}), fp32, "
                         f"{dt:.2f} s"}
    print(json.dumps({
        "metric": "qk_prep fwd+bwd GB/s (varlen QK-RMSNorm + RoPE, bf16)", "value": gbs, "unit": "GB/s",
        "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "dtype": "bf16", "data": "synthetic",
        "config": {"workload": w["desc"] + "; q and k of every token, H_KV = H", "tokens": T},
        "roofline": {"bound": "hbm", "achieved": gbs, "peak": peak, "unit": "GB/s", "frac": gbs / peak,
                     "peak_source": peak_src, "algorithmic_bytes_per_step": algo_bytes},
        "cpu_baseline": cpu, "clocks": clk,
    }))


def run_decode(args, w):
    """KV-cache decode (one new token per sequence, bias on), one GPU."""
    from fna2_b200.decode import flash_naylis_decode
    from oracle import decode_oracle as DO
    dev = "cuda"
    lengths, H, D, R = w["lengths"], w["H"], w["D"], w["r"]
    H_KV = H
    B = len(lengths)
    cap = max(lengths) + 1
    offs = [0]
    for n in lengths:
        offs.append(offs[-1] + n + 1)  # each sequence owns L + 1 slots
    rows = offs[-1]
    g = torch.Generator(device=dev).manual_seed(0)
    kc = torch.randn(rows, H_KV, D, device=dev, generator=g, dtype=torch.bfloat16)
    vc = torch.randn(rows, H_KV, D, device=dev, generator=g, dtype=torch.bfloat16)
    rkc = (torch.randn(rows, H, R, device=dev, generator=g) * 0.25).bfloat16()
    q = torch.randn(B, H, D, device=dev, generator=g, dtype=torch.bfloat16)
    rq = (torch.randn(B, H, R, device=dev, generator=g) * 0.25).bfloat16()
    kn = torch.randn(B, H_KV, D, device=dev, generator=g, dtype=torch.bfloat16)
    vn = torch.randn(B, H_KV, D, device=dev, generator=g, dtype=torch.bfloat16)
    rkn = (torch.randn(B, H, R, device=dev, generator=g) * 0.25).bfloat16()
    gs = torch.ones(H, device=dev)
    seq = torch.tensor(lengths, dtype=torch.int32, device=dev)
    offsets = torch.tensor(offs[:-1], dtype=torch.int32, device=dev)

    def step():
        return flash_naylis_decode(q, kc, vc, seq, rq, rkc, gs, kn, vn, rkn, cache_offsets=offsets, capacity=cap)

    for _ in range(max(args.warmup, 3)):
        step()
    st = torch.cuda.current_stream()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clocks = ClockSampler(0)
    torch.cuda.synchronize()
    clocks.start()
    t0.record(st)
    for _ in range(args.steps):
        step()
    t1.record(st)
    torch.cuda.synchronize()
    clk = clocks.stop()
    ms = t0.elapsed_time(t1) / args.steps
    keys = sum(lengths)
    # reads: cached K, V, R_k of every key, q, r_q, the new rows; writes: the new rows, out
    algo_bytes = keys * (2 * H_KV * D + H * R) * 2 + B * (H * D + H * R) * 2 + 2 * B * (2 * H_KV * D + H * R) * 2 \
        + B * H * D * 2
    gbs = algo_bytes / (ms / 1e3) / 1e9
    peak, peak_src = None, "measured"
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            peak = json.load(f).get("hbm_gbs")
    except Exception:
        pass
    if peak is None:
        peak, peak_src = 6650.0, "fallback"
    cpu = None
    if not args.no_cpu:
        torch.set_num_threads(os.cpu_count())
        sample = [b for b in range(B) if lengths[b] <= 2048][:8]
        qs, rqs = q[sample].cpu(), rq[sample].cpu()
        kcs = [kc[offs[b]:offs[b] + lengths[b]].cpu() for b in sample]
        vcs = [vc[offs[b]:offs[b] + lengths[b]].cpu() for b in sample]
        rks = [rkc[offs[b]:offs[b] + lengths[b]].cpu() for b in sample]
        Lm = max(lengths[b] for b in sample)
        pad = lambda ts: torch.stack([torch.nn.functional.pad(t, (0, 0, 0, 0, 0, Lm - t.shape[0])) for t in ts])
        t_c = time.perf_counter()
        DO.decode(qs, pad(kcs), pad(vcs), [lengths[b] for b in sample], rqs, pad(rks), gs.cpu(),
                  kn[sample].cpu(), vn[sample].cpu(), rkn[sample].cpu())
        dt = time.perf_counter() - t_c
        cb = sum(lengths[b] for b in sample) * (2 * H_KV * D + H * R) * 2
        cpu = {"value": cb / dt / 1e9, "unit": "GB/s", "cores": os.cpu_count(), "kind": "port",
               "sample": f"{len(sample)} sequences of the workload with L<=2048 (sum L="
                         f"{sum(lengths[b] for b in sample)}), fp64 per-head loop, {dt:.2f} s"}
    print(json.dumps({
        "metric": "decode step GB/s (KV cache + relational bias, bf16, one new token per sequence)",
        "value": gbs, "unit": "GB/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": w["desc"] + f"; decode of one token per sequence against caches of its L tokens, "
                                           f"H_KV = H = {H}, packed caches", "cached_keys": keys, "sequences": B,
                   "tokens_per_s": B / (ms / 1e3), "inputs_vs_l2": "caches far larger than L2"},
        "roofline": {"bound": "hbm", "achieved": gbs, "peak": peak, "unit": "GB/s", "frac": gbs / peak,
                     "peak_source": peak_src, "algorithmic_bytes_per_step": algo_bytes},
        "cpu_baseline": cpu, "clocks": clk,
    }))


def run_rel_proj(args, w):
    """Fused R_q/R_k projection (fna2_gemm over the stacked weights) fwd + bwd, one GPU."""
    import torch.nn.functional as F
    from fna2_b200.rel_proj import compute_rq_rk
    dev = "cuda"
    lengths, H, D, R = w["lengths"], w["H"], w["D"], w["r"]
    T, E, n = sum(lengths), H * D, H * R
    g = torch.Generator(device=dev).manual_seed(0)
    x = torch.randn(T, E, device=dev, generator=g, dtype=torch.bfloat16).requires_grad_(True)
    wq = (torch.randn(n, E, device=dev, generator=g) * 0.01).bfloat16().requires_grad_(True)
    wk = (torch.randn(n, E, device=dev, generator=g) * 0.01).bfloat16().requires_grad_(True)
    w_st = torch.cat([wq.detach(), wk.detach()]).requires_grad_(True)
    gq = torch.randn(T, H, R, device=dev, generator=g, dtype=torch.bfloat16)
    gk = torch.randn(T, H, R, device=dev, generator=g, dtype=torch.bfloat16)

    def fused():
        x.grad = w_st.grad = None
        rq, rk = compute_rq_rk(x, w_st, H, R)
        torch.autograd.backward([rq, rk], [gq, gk])

    def reference():  # attention_fna2.py:332-333: two Linear layers, view, cast, contiguous
        x.grad = wq.grad = wk.grad = None
        rq = F.linear(x, wq).view(T, H, R).to(torch.bfloat16).contiguous()
        rk = F.linear(x, wk).view(T, H, R).to(torch.bfloat16).contiguous()
        torch.autograd.backward([rq, rk], [gq, gk])

    def timeit(fn):
        for _ in range(max(args.warmup, 3)):
            fn()
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        t0.record()
        for _ in range(args.steps):
            fn()
        t1.record()
        torch.cuda.synchronize()
        return t0.elapsed_time(t1) / args.steps

    clocks = ClockSampler(0)
    clocks.start()
    ms = timeit(fused)
    clk = clocks.stop()
    ms_ref = timeit(reference)
    flops = 6.0 * T * E * 2 * n  # forward, dX and dW GEMMs over N = 2 * H_G * R
    tf = flops / (ms / 1e3) / 1e12
    peak, peak_src = None, "measured"
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            peak = json.load(f).get("bf16_tflops")
    except Exception:
        pass
    if peak is None:
        peak, peak_src = 1590.0, "fallback"
    print(json.dumps({
        "metric": "R_q/R_k projection fwd+bwd TFLOP/s (bf16, fna2_gemm over the stacked weights)",
        "value": tf, "unit": "TFLOP/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": w["desc"] + f"; x [T, {E}] bf16, H_G = {H}, R = {R}", "tokens": T,
                   "reference_two_linears_ms": ms_ref, "speedup_vs_reference_composition": ms_ref / ms,
                   "gemm": "fna2_gemm (tcgen05, 128 x 256 tiles, persistent; Y, dX and dW)",
                   "gpu_launches_per_step": 3},
        "roofline": {"bound": "tensor", "achieved": tf, "peak": peak, "unit": "TFLOP/s", "frac": tf / peak,
                     "peak_source": peak_src},
        "clocks": clk,
    }))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="fna2", choices=["fna2", "reference"])
    ap.add_argument("--workload", default="cfg5",
                    help="cfg5 (default), cfg3, cfg2, cfg4, cfg5short, or seqs:N:L:H:r")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-check", action="store_true", help="skip the gather-and-compare check of the shards")
    ap.add_argument("--cpu-budget", type=float, default=15.0)
    ap.add_argument("--op", default="attention", choices=["attention", "qk_prep", "decode", "rel_proj"])
    args = ap.parse_args()
    w = workload(args.workload)
    if args.op == "qk_prep":
        run_qk_prep(args, w)
    elif args.op == "decode":
        run_decode(args, w)
    elif args.op == "rel_proj":
        run_rel_proj(args, w)
    elif args.impl == "reference":
        run_reference(args, w)
    else:
        run_gpu(args, w)


if __name__ == "__main__":
    main()
