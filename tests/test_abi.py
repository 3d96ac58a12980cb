"""libqx.so builds, loads without a GPU and exports every entry point of include/qx.h; the plan
compiler's output is self-consistent (CPU only: no compute call is made)."""

import ctypes as C
import re
from pathlib import Path

import numpy as np

from conftest import REPO


def declared_symbols() -> list[str]:
    text = (REPO / "include" / "qx.h").read_text()
    return sorted(set(re.findall(r"^\s*(?:QX_API\s+)?(?:qx_status|size_t|const char \*)\s*(qx_\w+)\s*\(", text, re.M)))


def test_library_exports_every_declared_symbol():
    from qwenputer_b200 import build

    lib = C.CDLL(str(build.build()))
    names = declared_symbols()
    assert len(names) == 14, names
    for n in names:
        assert hasattr(lib, n), n


def test_no_device_gives_an_error_not_a_crash():
    """Without a usable device qx_create returns a status (never a CPU fallback)."""
    from qwenputer_b200 import build
    from qwenputer_b200.graphfile import default_graph_path, load_graph
    from qwenputer_b200.plan import compile_plan

    lib = C.CDLL(str(build.build()))
    lib.qx_last_error.restype = C.c_char_p
    blob = compile_plan(load_graph(default_graph_path())).blob()
    h = C.c_void_p()
    st = lib.qx_create(blob, C.c_size_t(len(blob)), 4, 0, C.byref(h))
    import torch

    if not torch.cuda.is_available():
        assert st != 0 and h.value is None
    else:
        lib.qx_destroy(h)


def test_bad_plans_are_rejected():
    from qwenputer_b200 import build
    from qwenputer_b200.graphfile import default_graph_path, load_graph
    from qwenputer_b200.plan import compile_plan

    lib = C.CDLL(str(build.build()))
    blob = bytearray(compile_plan(load_graph(default_graph_path())).blob())
    h = C.c_void_p()
    bad = bytearray(blob)
    bad[0] ^= 0xFF  # magic
    assert lib.qx_create(bytes(bad), C.c_size_t(len(bad)), 4, 0, C.byref(h)) == 1
    assert lib.qx_create(bytes(blob[:1000]), C.c_size_t(1000), 4, 0, C.byref(h)) == 1


def test_plan_is_consistent(graph):
    from qwenputer_b200.plan import PH, compile_plan

    P = compile_plan(graph)
    s = P.sec
    rows = P.hdr["n_slots"] + P.hdr["n_scratch"]
    # every packed entry and destination addresses a shared-memory row
    assert int((s["NNZ"] & 0xFFFF).max()) < rows
    assert int(s["FORMS"]["dst"].max()) < rows
    assert int(s["NODES"]["out"].max()) < rows
    assert all(r < rows or r == 0xFFFF for r in s["UNITS"]["a"]) and all(r < rows or r == 0xFFFF for r in s["UNITS"]["b"])
    # forms' entries lie inside the packed array and are 16-byte aligned
    assert np.all(s["FORMS"]["nnz0"] % 4 == 0)
    assert np.all(s["FORMS"]["nnz0"] + 4 * s["FORMS"]["nnz4"].astype(np.int64) <= len(s["NNZ"]))
    # each run program ends with the decode and END, warp ranges are monotone
    kinds = list(s["RUN_PROG"]["kind"])
    assert kinds[-2:] == [PH["DECODE"], PH["END"]] and kinds.count(PH["END"]) == 1
    wp = s["WARP_PTR"].astype(np.int64)
    for ph in s["RUN_PROG"]:
        if ph["kind"] in (PH["FORMS"], PH["UNITS"]):
            seg = wp[ph["c"]:ph["c"] + P.hdr["nw"] + 1]
            assert np.all(np.diff(seg) >= 0) and seg[0] == ph["a"] and seg[-1] == ph["b"]
    # 99 snapshot tables, the plan fits the shared memory of one CTA
    assert len(s["TABLES"]) == 198
    smem = rows * 33 * 4 + P.hdr["n_ksel_slots"] * 32 * (1 + P.hdr["qhot_max"]) * 4 + 32 * 18 * 4 + 64
    assert smem <= 232448, smem
    assert P.hdr["n_born0"] == P.hdr["n_feat"]
    assert list(s["PAIRS"][:P.hdr["n_born0"], 1]) == [int(d) for d in graph.feat_dims]


def test_plan_residual_slots_never_collide(graph):
    """Two dims sharing a residual row never live in the same sublayer."""
    from qwenputer_b200.plan import compile_plan

    P = compile_plan(graph)
    assert P.hdr["n_slots"] < 1500
    assert P.stats["form_nnz"] < 400_000
