"""Generate tests/golden/packing_cases.json from the reference's own packing
helpers.

The reference ships pack_batch and pack_documents as Python code blocks in
FNA2/INTEGRATION.md (:133-151 and :236-257).  This script takes each block's
source text from that file, executes it, and records its outputs on seeded
inputs and edge cases.  It needs the reference tree (FNA2_REFERENCE, required:
the reference checkout's FNA2 directory) and runs on CPU; the JSON it writes is what the tests
read.

    python tests/golden/make_golden_packing.py
"""
import json
import os
import random

import torch

REF = os.environ.get("FNA2_REFERENCE")
if not REF:
    raise SystemExit("set FNA2_REFERENCE to the reference checkout's FNA2 directory "
                     "(the directory holding flash_naylis_attn.py)")
OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "packing_cases.json")


def _block(lines, name):
    """Source of the fenced code block that defines `name` (from its def to the fence)."""
    start = next(i for i, l in enumerate(lines) if l.startswith(f"def {name}("))
    end = next(i for i in range(start, len(lines)) if lines[i].startswith("```"))
    body = []
    for l in lines[start:end]:
        if body and l and not l[0].isspace() and not l.startswith("def "):
            break  # module-level code after the function (usage examples)
        body.append(l)
    return "\n".join(body), start + 1


def load_reference():
    with open(os.path.join(REF, "INTEGRATION.md"), encoding="utf-8") as f:
        lines = f.read().splitlines()
    ns = {"torch": torch}
    where = {}
    for name in ("pack_batch", "pack_documents"):
        src, line = _block(lines, name)
        exec(compile(src, f"INTEGRATION.md:{line}", "exec"), ns)
        where[name] = f"FNA2/INTEGRATION.md:{line}"
    return ns["pack_batch"], ns["pack_documents"], where


def doc_cases():
    rng = random.Random(7)
    cases = [
        dict(docs=[], max_seq_len=16, eos_id=2),
        dict(docs=[[]], max_seq_len=16, eos_id=2),
        dict(docs=[[5] * 15], max_seq_len=16, eos_id=2),          # doc + EOS fills the bin exactly
        dict(docs=[[5] * 15, [6]], max_seq_len=16, eos_id=2),
        dict(docs=[[7] * 40, [8, 9]], max_seq_len=16, eos_id=2),   # truncated, EOS dropped
        dict(docs=[[1, 2], [3]], max_seq_len=0, eos_id=2),
        dict(docs=[[1, 2, 3], [4]], max_seq_len=-1, eos_id=2),
        dict(docs=[[1], [2], [3]], max_seq_len=1, eos_id=0),
    ]
    for n_docs, max_len in ((20, 64), (50, 128), (80, 512)):
        docs = [[rng.randrange(3, 1000) for _ in range(rng.choice([0, 1, 5, 17, 60, 200, 600]))]
                for _ in range(n_docs)]
        cases.append(dict(docs=docs, max_seq_len=max_len, eos_id=2))
    return cases


def batch_cases():
    rng = random.Random(8)
    cases = [dict(lengths=[7], feat=[]), dict(lengths=[3, 0, 5, 1], feat=[]), dict(lengths=[4, 2], feat=[3])]
    cases.append(dict(lengths=[rng.randrange(0, 100) for _ in range(30)], feat=[]))
    return cases


def main():
    pack_batch, pack_documents, where = load_reference()
    out = {"source": where, "pack_documents": [], "pack_batch": []}
    for c in doc_cases():
        bins = pack_documents([list(d) for d in c["docs"]], c["max_seq_len"], c["eos_id"])
        out["pack_documents"].append(dict(c, bins=bins))
    g = torch.Generator().manual_seed(9)
    for c in batch_cases():
        seqs = [torch.randint(0, 1000, [n] + c["feat"], generator=g) for n in c["lengths"]]
        x, cu, mx = pack_batch(seqs, torch.device("cpu"))
        out["pack_batch"].append(dict(c, sequences=[s.tolist() for s in seqs], x_packed=x.tolist(),
                                      cu_seqlens=cu.tolist(), cu_dtype=str(cu.dtype), max_seqlen=mx))
    with open(OUT, "w") as f:
        json.dump(out, f, separators=(",", ":"))
    print("wrote", OUT, {k: len(v) for k, v in out.items() if isinstance(v, list)})


if __name__ == "__main__":
    main()
