"""Producers of the packed varlen format that flash_naylis_attn consumes:
tokens of all sequences concatenated along dim 0, int32 cu_seqlens of N+1
offsets, and max_seqlen.

pack_batch follows the reference helper of the same name
(FNA2/INTEGRATION.md:133-151): x_packed = the sequences concatenated,
cu_seqlens[0] = 0 and cu_seqlens[i+1] = cu_seqlens[i] + len(sequences[i])
(int32, on `device`), max_seqlen = the longest length as a Python int.  As in
the reference, an empty list is an error (the reference's torch.cat raises).
Here the lengths and offsets are formed on the host, so nothing waits for the
device, and a host batch bound for a GPU is concatenated into pinned memory
and crosses PCIe as one non-blocking copy (two with cu_seqlens) instead of one
copy per intermediate.

pack_documents follows the reference's greedy document-aware packing
(FNA2/INTEGRATION.md:236-257): each document gets eos_id appended; a document
that does not fit in the current bin (len(bin) + len(doc) + 1 > max_seq_len)
closes the bin and starts a new one, truncated to max_seq_len tokens (the
truncated tail, EOS included, is dropped); empty bins are never emitted.
pack_documents_batch chains the two.
"""
from typing import List, Sequence, Tuple

import torch


def _offsets(lengths: Sequence[int]) -> List[int]:
    cu = [0]
    for n in lengths:
        cu.append(cu[-1] + int(n))
    return cu


def pack_batch(sequences: Sequence[torch.Tensor], device) -> Tuple[torch.Tensor, torch.Tensor, int]:
    """Concatenate `sequences` ([s_i, ...] each) into ([sum s_i, ...], cu_seqlens [N+1] int32, max_seqlen)."""
    if len(sequences) == 0:
        raise RuntimeError("pack_batch: expected a non-empty list of sequences")
    device = torch.device(device)
    lengths = [int(s.shape[0]) for s in sequences]
    cu = _offsets(lengths)
    if cu[-1] >= 2 ** 31:
        raise ValueError(f"pack_batch: {cu[-1]} tokens do not fit int32 cu_seqlens")
    on_host = all(s.device.type == "cpu" for s in sequences)
    if device.type == "cuda" and on_host:
        first = sequences[0]
        staged = torch.empty((cu[-1],) + tuple(first.shape[1:]), dtype=first.dtype, pin_memory=True)
        torch.cat(list(sequences), dim=0, out=staged)
        x_packed = staged.to(device, non_blocking=True)
        cu_host = torch.tensor(cu, dtype=torch.int32).pin_memory()
        cu_seqlens = cu_host.to(device, non_blocking=True)
    else:
        x_packed = torch.cat([s.to(device) for s in sequences], dim=0)
        cu_seqlens = torch.tensor(cu, dtype=torch.int32, device=device)
    return x_packed, cu_seqlens, max(lengths)


def pack_documents(docs: Sequence[Sequence[int]], max_seq_len: int, eos_id: int = 2) -> List[List[int]]:
    """Greedy packing of token-id documents into bins of at most max_seq_len tokens."""
    bins: List[List[int]] = []
    cur: List[int] = []
    for doc in docs:
        need = len(doc) + 1  # the document and its EOS
        if len(cur) + need > max_seq_len:
            if cur:
                bins.append(cur)
            cur = (list(doc) + [eos_id])[:max_seq_len]  # plain slice, as the reference's
        else:
            cur.extend(doc)
            cur.append(eos_id)
    if cur:
        bins.append(cur)
    return bins


def pack_documents_batch(docs: Sequence[Sequence[int]], max_seq_len: int, device, eos_id: int = 2,
                         dtype=torch.int64) -> Tuple[torch.Tensor, torch.Tensor, int]:
    """pack_documents, then pack_batch of the bins: (tokens, cu_seqlens, max_seqlen) on `device`."""
    bins = pack_documents(docs, max_seq_len, eos_id)
    return pack_batch([torch.tensor(b, dtype=dtype) for b in bins], device)
