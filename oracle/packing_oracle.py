"""CPU restatement of the reference's packing helpers.

TEST INFRASTRUCTURE ONLY: imported by tests/ (as the checker of
fna2_b200/packing.py); never by the product path.

  pack_batch      FNA2/INTEGRATION.md:133-151  concatenation, int32 cu_seqlens
                                               (cumulative sum with a leading 0),
                                               max_seqlen = longest sequence
  pack_documents  FNA2/INTEGRATION.md:236-257  greedy bins: doc + EOS appended to
                                               the open bin if it fits, else the
                                               bin closes and the doc (sliced to
                                               max_seq_len) opens the next one
Pinned against fixtures produced by executing the reference's own code blocks
(tests/golden/make_golden_packing.py).
"""
from __future__ import annotations

import itertools

import torch


def pack_batch(sequences, device="cpu"):
    if not sequences:
        raise RuntimeError("no sequences")
    lengths = [s.shape[0] for s in sequences]
    cu = torch.tensor([0] + list(itertools.accumulate(lengths)), dtype=torch.int32, device=device)
    return torch.cat(list(sequences), 0).to(device), cu, max(lengths)


def pack_documents(docs, max_seq_len, eos_id=2):
    out, open_bin = [], []
    for d in docs:
        toks = list(d) + [eos_id]
        if len(open_bin) + len(toks) <= max_seq_len:
            open_bin = open_bin + toks
            continue
        if open_bin:
            out.append(open_bin)
        open_bin = toks[:max_seq_len]
    return out + ([open_bin] if open_bin else [])
