"""Times the reference's own PyTorch CPU forward: ``fastexec.Executor(c, "cpu", B, sparse)``
(``ERV/chipformer/rv/fastexec.py:88-218``), teacher-forced the way the reference's harness
``fastexec.timed`` (``fastexec.py:343-396``) times it on a GPU: every batch row loaded from the
same snapshot, the trace's embeddings computed before the timed region, one ``step`` per token.

Measurement infrastructure, not product code: it imports the reference tree, so it runs only
where that tree is present (argument or ``QX_REFERENCE_ROOT``)::

    python oracle/time_reference_cpu.py /path/to/reference/experimental/riscv [--batches 1 64 256]

Prints one JSON line per (batch, dense / sparse) with trace tokens/s = B * steps / seconds on
``torch.get_num_threads()`` host threads.  The program is one of the bignum-mix programs of the
executor's bench (seed 1000).
"""

from __future__ import annotations

import argparse
import json
import os
import sys
import time
from pathlib import Path
from types import SimpleNamespace

sys.dont_write_bytecode = True  # the reference tree is read-only
REPO = Path(__file__).resolve().parents[1]


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("ref_root", nargs="?", default=os.environ.get("QX_REFERENCE_ROOT"))
    ap.add_argument("--batches", type=int, nargs="+", default=[1, 64, 256])
    ap.add_argument("--steps", type=int, default=40)
    ap.add_argument("--seconds", type=float, default=20.0, help="cap on each timed region")
    a = ap.parse_args()
    if not a.ref_root:
        ap.error("give the reference's experimental/riscv directory or set QX_REFERENCE_ROOT")
    sys.path.insert(0, a.ref_root)
    sys.path.insert(0, str(REPO))
    import torch
    from chipformer.rv import core, fastexec, ref

    from qwenputer_b200 import workload

    torch.set_num_threads(os.cpu_count() or 1)
    c = core.build()
    p = workload.workload_programs("bignum", 1, 1000)[0]
    prog = SimpleNamespace(text=[int(w) for w in p.text], data=bytes(p.data), data_base=int(p.data_base),
                           entry=int(p.entry), rodata=bytes(p.rodata))  # plain ints for the reference
    core.snapshot(c, ref.Machine.from_program(prog))
    toks = ref.Machine.from_program(prog).run(a.steps + 30)
    for B in a.batches:
        for sparse in (False, True):
            ex = fastexec.Executor(c, "cpu", B, sparse)
            for b in range(B):
                ex.load_init(b)
            emb = ex.embed(toks[:a.steps + 5])
            xin = torch.zeros(B, ex.D)
            with torch.no_grad():
                for t in range(3):  # warm-up
                    xin.copy_(emb[t].expand(B, -1))
                    ex.step(xin)
                n, t0 = 0, time.perf_counter()
                for t in range(3, 3 + a.steps):
                    xin.copy_(emb[t].expand(B, -1))
                    ex.step(xin)
                    n += 1
                    if time.perf_counter() - t0 > a.seconds:
                        break
                dt = time.perf_counter() - t0
            print(json.dumps({"impl": "reference fastexec.Executor (PyTorch CPU)", "batch": B,
                              "sparse": sparse, "steps": n, "seconds": round(dt, 3),
                              "tokens_per_s": B * n / dt, "threads": torch.get_num_threads(),
                              "cpu": os.cpu_count()}), flush=True)
            del ex


if __name__ == "__main__":
    main()
