"""Writes ``rv32im_graph.npz``: the reference's standalone RV32IM (+Zba, bignum) compiled stack
(``ERV/chipformer/rv/core.py:299 build()``, target Qwen3.5-4B layer shapes ``core.T4B``) in the
executor's file format (``qwenputer_b200/graphfile.py``).

Needs the reference tree importable (``ERV`` = ``experimental/riscv``), given as the argument
or as ``QX_REFERENCE_ROOT``::

    python qwenputer_b200/plans/export_rv32im.py /path/to/reference/experimental/riscv
"""

import os
import sys
import time
from pathlib import Path

sys.dont_write_bytecode = True  # the reference tree is read-only


def main(ref_root: str) -> None:
    sys.path.insert(0, ref_root)
    sys.path.insert(0, str(Path(__file__).resolve().parents[2]))
    from chipformer.rv import core

    from qwenputer_b200.graphfile import default_graph_path, export_graph, save_graph

    t0 = time.time()
    c = core.build()
    g = export_graph(c)
    save_graph(g, default_graph_path())
    print(f"exported {c.stats()} in {time.time() - t0:.1f} s -> {default_graph_path()} "
          f"({default_graph_path().stat().st_size} bytes)")


if __name__ == "__main__":
    root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("QX_REFERENCE_ROOT")
    if not root:
        sys.exit("usage: export_rv32im.py REFERENCE/experimental/riscv (or set QX_REFERENCE_ROOT)")
    main(root)
