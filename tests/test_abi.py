"""CPU tests of the C ABI: the library loads, exports every symbol include/fna2.h
declares, the ctypes structs match the C layout, and invalid arguments are
rejected on the host (no GPU needed: validation precedes any CUDA call)."""
import ctypes
import os
import re
import subprocess

import pytest

from fna2_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "fna2.h")


def _declared():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"^\s*(?:int|size_t|const char\*)\s+(fna2_\w+)\s*\(", text, re.M)))


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    declared = _declared()
    assert declared, "no declarations parsed"
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True, text=True).stdout
    exported = set(re.findall(r"\sT\s(fna2_\w+)", out))
    for name in declared:
        assert name in exported, name
        assert hasattr(lib, name)
    assert set(_lib.EXPORTED) <= set(declared)


def test_struct_layout_matches_c(tmp_path):
    src = tmp_path / "sz.c"
    src.write_text('#include <stdio.h>\n#include <stddef.h>\n#include "fna2.h"\n'
                   'int main(){printf("%zu %zu %zu %zu %zu %zu\\n", sizeof(Fna2Tensor), sizeof(Fna2Problem),'
                   ' sizeof(Fna2FwdArgs), sizeof(Fna2BwdArgs), offsetof(Fna2BwdArgs, workspace_bytes),'
                   ' offsetof(Fna2FwdArgs, launch_events));}\n')
    exe = tmp_path / "sz"
    subprocess.check_call(["gcc", "-I", os.path.join(ROOT, "include"), str(src), "-o", str(exe)])
    got = [int(x) for x in subprocess.check_output([str(exe)]).split()]
    want = [ctypes.sizeof(_lib.Fna2Tensor), ctypes.sizeof(_lib.Fna2Problem), ctypes.sizeof(_lib.Fna2FwdArgs),
            ctypes.sizeof(_lib.Fna2BwdArgs), _lib.Fna2BwdArgs.workspace_bytes.offset,
            _lib.Fna2FwdArgs.launch_events.offset]
    assert got == want


def test_qkprep_struct_layout_matches_c(tmp_path):
    src = tmp_path / "sz2.c"
    src.write_text('#include <stdio.h>\n#include <stddef.h>\n#include "fna2.h"\n'
                   'int main(){printf("%zu %zu %zu %zu %zu %zu\\n", sizeof(Fna2Rows), sizeof(Fna2QkPrepArgs),'
                   ' sizeof(Fna2QkPrepBwdArgs), offsetof(Fna2QkPrepArgs, inv_freq), offsetof(Fna2QkPrepArgs, q_in),'
                   ' offsetof(Fna2QkPrepBwdArgs, dk_weight));}\n')
    exe = tmp_path / "sz2"
    subprocess.check_call(["gcc", "-I", os.path.join(ROOT, "include"), str(src), "-o", str(exe)])
    got = [int(x) for x in subprocess.check_output([str(exe)]).split()]
    want = [ctypes.sizeof(_lib.Fna2Rows), ctypes.sizeof(_lib.Fna2QkPrepArgs), ctypes.sizeof(_lib.Fna2QkPrepBwdArgs),
            _lib.Fna2QkPrepArgs.inv_freq.offset, _lib.Fna2QkPrepArgs.q_in.offset,
            _lib.Fna2QkPrepBwdArgs.dk_weight.offset]
    assert got == want


def _qk_args(**over):
    a = _lib.Fna2QkPrepArgs()
    a.total_tokens, a.num_seqs, a.heads_q, a.heads_k, a.head_dim = 8, 1, 2, 1, 128
    a.in_dtype = a.weight_dtype = a.rope_dtype = _lib.FNA2_DTYPE_BF16
    buf = ctypes.create_string_buffer(1 << 16)
    base = (ctypes.addressof(buf) + 255) // 256 * 256
    for name in ("q_in", "k_in", "q_out", "k_out"):
        setattr(a, name, _lib.Fna2Rows(base, 256, 128))
    for k, v in over.items():
        setattr(a, k, v)
    return a, buf


@pytest.mark.parametrize("field,value,msg", [
    ("head_dim", 96, "head_dim"),
    ("in_dtype", 7, "in_dtype"),
    ("rope_dtype", -1, "rope_dtype"),
    ("total_tokens", -1, "negative"),
])
def test_qkprep_invalid_arguments_rejected(field, value, msg):
    lib = _lib.load()
    a, _buf = _qk_args(**{field: value})
    assert lib.fna2_qk_prep_fwd(a, None) == _lib.FNA2_ERR_INVALID
    assert msg in lib.fna2_last_error().decode()


def test_qkprep_rope_needs_cu_and_alignment():
    lib = _lib.load()
    inv = (ctypes.c_float * 64)()
    a, _buf = _qk_args(inv_freq=ctypes.addressof(inv))
    assert lib.fna2_qk_prep_fwd(a, None) == _lib.FNA2_ERR_INVALID
    assert "cu_seqlens" in lib.fna2_last_error().decode()
    a, _buf = _qk_args()
    a.q_in = _lib.Fna2Rows(a.q_in.ptr + 2, 256, 128)
    assert lib.fna2_qk_prep_fwd(a, None) == _lib.FNA2_ERR_INVALID
    assert "aligned" in lib.fna2_last_error().decode()


def test_qkprep_empty_is_a_no_op():
    lib = _lib.load()
    a, _buf = _qk_args(total_tokens=0)
    assert lib.fna2_qk_prep_fwd(a, None) == _lib.FNA2_OK


def _fwd_args(**over):
    a = _lib.Fna2FwdArgs()
    p = a.prob
    p.batch, p.seqlen_q, p.seqlen_k = 1, 128, 128
    p.heads, p.heads_kv, p.heads_graph, p.head_dim, p.rank = 2, 2, 2, 128, 16
    p.softmax_scale, p.causal = 0.088, 1
    for k, v in over.items():
        setattr(p, k, v)
    return a


@pytest.mark.parametrize("field,value,msg", [
    ("head_dim", 96, "head_dim"),
    ("heads_kv", 3, "heads_kv"),
    ("heads_graph", 5, "heads_graph"),
    ("rank", 12, "rank"),
    ("softmax_scale", 0.0, "softmax_scale"),
])
def test_invalid_problem_rejected_on_host(field, value, msg):
    lib = _lib.load()
    a = _fwd_args(**{field: value})
    rc = lib.fna2_fwd(ctypes.byref(a), None)
    assert rc == _lib.FNA2_ERR_INVALID
    assert msg in lib.fna2_last_error().decode()


def test_null_and_misaligned_tensors_rejected():
    lib = _lib.load()
    a = _fwd_args()
    rc = lib.fna2_fwd(ctypes.byref(a), None)  # q.ptr is NULL
    assert rc == _lib.FNA2_ERR_INVALID and "q: null pointer" in lib.fna2_last_error().decode()
    a.q.ptr = 0x1008  # not 16-byte aligned
    a.q.stride[:] = (256 * 128, 128 * 128, 128, 1)
    rc = lib.fna2_fwd(ctypes.byref(a), None)
    assert rc == _lib.FNA2_ERR_INVALID and "16-byte" in lib.fna2_last_error().decode()
    a.q.ptr = 0x1000
    a.q.stride[:] = (256 * 128, 128 * 128, 128, 2)
    rc = lib.fna2_fwd(ctypes.byref(a), None)
    assert rc == _lib.FNA2_ERR_INVALID and "column stride" in lib.fna2_last_error().decode()


def test_empty_problem_is_a_no_op():
    lib = _lib.load()
    a = _fwd_args(batch=0)
    assert lib.fna2_fwd(ctypes.byref(a), None) == _lib.FNA2_OK


def test_forward_workspace_size_and_check():
    """Packed forwards need the tile table (32 B per entry, ceil(T/256) + N
    entries); dense ones need none.  A packed call without it fails on the host."""
    lib = _lib.load()
    dense = _fwd_args()
    assert lib.fna2_fwd_workspace_size(ctypes.byref(dense.prob)) == 0
    a = _fwd_args(batch=3, seqlen_q=300, seqlen_k=300, total_q=700, total_k=700)
    a.prob.cu_seqlens_q = a.prob.cu_seqlens_k = 0x2000  # device pointers are not read on the host
    n = lib.fna2_fwd_workspace_size(ctypes.byref(a.prob))
    assert n == ((700 + 255) // 256 + 3) * 32
    for name in ("q", "k", "v", "out", "r_q", "r_k"):
        d = getattr(a, name)
        d.ptr = 0x10000
        d.stride[:] = (0, 128, 2 * 128, 1) if name not in ("r_q", "r_k") else (0, 16, 2 * 16, 1)
    a.graph_scale = 0x10000
    a.lse = 0x10000
    rc = lib.fna2_fwd(ctypes.byref(a), None)
    assert rc == _lib.FNA2_ERR_WORKSPACE and "forward workspace" in lib.fna2_last_error().decode()


def test_workspace_size():
    lib = _lib.load()
    a = _fwd_args()
    n = lib.fna2_bwd_workspace_size(ctypes.byref(a.prob))
    assert n >= 2 * 1 * 2 * 128 * 4 and n % 256 == 0
    bad = _fwd_args(head_dim=80)
    assert lib.fna2_bwd_workspace_size(ctypes.byref(bad.prob)) == 0


def test_python_entry_refuses_cpu_tensors():
    import torch
    from fna2_b200 import flash_naylis_attn
    q = torch.zeros(1, 2, 8, 64, dtype=torch.bfloat16)
    r = torch.zeros(1, 2, 8, 16, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="CUDA"):
        flash_naylis_attn(q, q, q, r, r, torch.ones(2))
    with pytest.raises(AssertionError):
        flash_naylis_attn(q, q, q, r.float(), r, torch.ones(2))


def test_module_constants_keep_reference_contract():
    import fna2_b200
    assert fna2_b200.BLOCK_R == 32  # NaylisAttention requires rel_rank == BLOCK_R (attention_fna2.py:225)
    assert fna2_b200.BLOCK_M == 128


def test_decode_struct_layout_matches_c(tmp_path):
    src = tmp_path / "dec.c"
    src.write_text('#include <stdio.h>\n#include <stddef.h>\n#include "fna2.h"\n'
                   'int main(){printf("%zu %zu %zu %zu %zu\\n", sizeof(Fna2DecodeArgs),'
                   ' offsetof(Fna2DecodeArgs, q), offsetof(Fna2DecodeArgs, cache_offsets),'
                   ' offsetof(Fna2DecodeArgs, rk_new), offsetof(Fna2DecodeArgs, num_splits));}\n')
    exe = tmp_path / "dec"
    subprocess.check_call(["gcc", "-I", os.path.join(ROOT, "include"), str(src), "-o", str(exe)])
    got = [int(x) for x in subprocess.check_output([str(exe)]).split()]
    D = _lib.Fna2DecodeArgs
    assert got == [ctypes.sizeof(D), D.q.offset, D.cache_offsets.offset, D.rk_new.offset, D.num_splits.offset]


def _dec_args(**over):
    a = _lib.Fna2DecodeArgs()
    a.batch, a.heads, a.kv_heads, a.graph_heads, a.head_dim, a.rank = 2, 4, 2, 4, 128, 16
    a.capacity, a.softmax_scale = 64, 0.088
    buf = ctypes.create_string_buffer(1 << 16)
    base = (ctypes.addressof(buf) + 255) // 256 * 256
    for name in ("q", "r_q", "k_cache", "v_cache", "rk_cache", "graph_scale", "cache_seqlens", "out"):
        setattr(a, name, base)
    a.q_batch_stride, a.q_head_stride = 512, 128
    a.k_batch_stride, a.k_token_stride, a.k_head_stride = 64 * 256, 256, 128
    a.v_batch_stride, a.v_token_stride, a.v_head_stride = 64 * 256, 256, 128
    a.rk_batch_stride, a.rk_token_stride, a.rk_head_stride = 64 * 64, 64, 16
    a.rq_batch_stride, a.rq_head_stride = 64, 16
    a.out_batch_stride, a.out_head_stride = 512, 128
    for k, v in over.items():
        setattr(a, k, v)
    return a, buf


@pytest.mark.parametrize("field,value,msg", [
    ("head_dim", 96, "head_dim"),
    ("kv_heads", 3, "multiple of kv_heads"),
    ("rank", 24, "rank"),
    ("graph_heads", 5, "graph_heads"),
    ("q_head_stride", 100, "strides"),
    ("softmax_scale", 0.0, "softmax_scale"),
])
def test_decode_invalid_arguments_rejected(field, value, msg):
    lib = _lib.load()
    a, _buf = _dec_args(**{field: value})
    assert lib.fna2_decode(a, None, 0, None) == _lib.FNA2_ERR_INVALID
    assert msg in lib.fna2_last_error().decode()


def test_decode_pairs_and_alignment_checked():
    lib = _lib.load()
    a, buf = _dec_args()
    a.k_new = a.q  # without v_new
    assert lib.fna2_decode(a, None, 0, None) == _lib.FNA2_ERR_INVALID
    assert "k_new and v_new" in lib.fna2_last_error().decode()
    a, buf = _dec_args()
    a.k_cache = a.k_cache + 8
    assert lib.fna2_decode(a, None, 0, None) == _lib.FNA2_ERR_INVALID
    assert "aligned" in lib.fna2_last_error().decode()


def test_decode_workspace_size_and_empty_batch():
    lib = _lib.load()
    a, _buf = _dec_args(num_splits=4)
    assert lib.fna2_decode_workspace_size(a) == 2 * 4 * 4 * (128 + 2) * 4
    a, _buf = _dec_args(num_splits=1)
    assert lib.fna2_decode_workspace_size(a) == 0
    a, _buf = _dec_args(num_splits=4)
    assert lib.fna2_decode(a, None, 0, None) == _lib.FNA2_ERR_WORKSPACE
    a, _buf = _dec_args(batch=0)
    assert lib.fna2_decode(a, None, 0, None) == _lib.FNA2_OK
