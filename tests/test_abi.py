"""libqx.so builds, loads without a GPU and exports every entry point of include/qx.h; the plan
compiler's output is self-consistent (CPU only: no compute call is made)."""

import ctypes as C
import re
from pathlib import Path

import numpy as np
import pytest

from conftest import REPO


def declared_symbols() -> list[str]:
    text = (REPO / "include" / "qx.h").read_text()
    return sorted(set(re.findall(r"^\s*(?:QX_API\s+)?(?:qx_status|size_t|const char \*)\s*(qx_\w+)\s*\(", text, re.M)))


def test_library_exports_every_declared_symbol():
    from qwenputer_b200 import build

    lib = C.CDLL(str(build.build()))
    names = declared_symbols()
    assert len(names) == 18, names
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


@pytest.mark.parametrize("cluster,tc,group", [(1, False, 32), (4, False, 32), (1, True, 32), (4, True, 32),
                                              (1, False, 16), (1, False, 8), (1, False, 4)])
def test_plan_is_consistent(graph, cluster, tc, group):
    from qwenputer_b200.plan import PH, RING_QUADS, SMEM_MAX, compile_plan, smem_extra_bytes

    P = compile_plan(graph, cluster=cluster, tc=tc, group=group)
    s = P.sec
    R = 32 // group  # record slots a warp: the stream comes in lines of R quads
    rb = (group + 1) * 4  # bytes per residual row
    rows = (P.hdr["n_slots"] + P.hdr["n_scratch"] + 1) * rb  # byte offsets, zero row included
    assert P.hdr["cluster"] == cluster and P.hdr["group"] == group
    nw = P.hdr["nw"] * cluster  # the warps of a machine group's cluster
    st = s["STREAM"].astype(np.int64)
    wp = s["WARP_PTR"].astype(np.int64)
    # walk every stream piece of every phase: rows in range, pieces inside one ring chunk,
    # records complete, a bundle's records of one shape, ranges end on their warp's range
    from qwenputer_b200.plan import PIECE_MAX, R_FIRST, R_LAST, R_NOP, R_QUERY, R_SKIP, R_SPLIT

    chunk = RING_QUADS * R
    for ph in s["RUN_PROG"]:
        k = int(ph["kind"]) & 0xFF
        if k not in (PH["FORMS"], PH["UNITS"], PH["KSEL"]):
            continue
        seg = wp[ph["c"]:ph["c"] + nw + 1]
        assert np.all(np.diff(seg) >= 0) and np.all(seg % R == 0)
        for w in range(nw):
            i, end, start = seg[w], seg[w + 1], seg[w]
            open_rec = False
            while i < end:
                hs = st[i:i + R]
                n, fl = int(hs[0][3]) & 0xFFFFFF, int(hs[0][3]) >> 24
                if fl & R_SKIP:
                    assert all(int(h[3]) >> 24 & R_SKIP for h in hs)
                    i = start + ((i - start) // chunk + 1) * chunk
                    continue
                assert 1 + n <= PIECE_MAX
                assert (i - start) // chunk == (i + R * (1 + n) - 1 - start) // chunk, "piece crosses a chunk"
                assert bool(fl & R_FIRST) != open_rec
                body = st[i + R:i + R * (1 + n)].reshape(n, R, 4)
                for sl in range(R):
                    h, b = hs[sl], body[:, sl]
                    fs = int(h[3]) >> 24
                    assert int(h[3]) & 0xFFFFFF == n and fs & 3 == fl & 3, "a bundle's pieces differ"
                    assert (fs ^ fl) & R_SPLIT == 0 and (not fs & R_SPLIT or (k == PH["FORMS"] and R > 1))
                    if k == PH["FORMS"]:
                        assert h[0] < rows and h[0] % rb == 0 and h[1] < rows and h[1] % rb == 0
                        assert np.all(b[:, 0] < rows) and np.all(b[:, 2] < rows)
                    elif k == PH["UNITS"]:
                        nc = int(h[1])
                        assert nc == int(hs[0][1]), "a bundle's constant-gate counts differ"
                        assert h[0] < rows and nc <= n and (n - nc) % 2 == 0
                        assert np.all(b[:nc, 0] < rows)
                        assert np.all(b[nc::2, 0] < rows) and np.all(b[nc::2, 1] < rows)
                    else:
                        assert fs & R_QUERY == fl & R_QUERY, "a bundle mixes keys and queries"
                        assert (h[0] & 0xFFFF) < P.hdr["n_ksel_slots"] and h[1] < rows and h[2] < rows
                        assert np.all(b[:, 0] < rows)
                    if fs & R_NOP:  # a padding record: zero weights only
                        assert not (b[:, 1] | (b[:, 3] if k == PH["FORMS"] else 0)).any()
                open_rec = not (fl & R_LAST)
                i += R * (1 + n)
            assert not open_rec
            assert i == end
    kinds = [int(k) & 0xFF for k in s["RUN_PROG"]["kind"]]
    assert kinds[-2:] == [PH["DECODE"], PH["END"]] and kinds.count(PH["END"]) == 1
    # tensor-core phases: staged rows and destinations inside the rows, blocks within the
    # staging area and accumulator columns, every tile inside its phase, the first tile of each
    # form block starting its accumulator, and the commit counts behind the barrier parity
    from qwenputer_b200.plan import MMA_MAX_FB, MMA_MAX_KB

    assert (PH["FORMS"] in kinds) != tc and (PH["MMA"] in kinds) == tc
    if tc:
        assert P.hdr["flags"] & 1 and bool(P.hdr["flags"] & 4) == (cluster == 1)
        tiles, n_tiles = s["MMA_TILES"], len(s["TILEDATA"]) // (128 * 16)
        commits = 0
        for mp in s["MMA_PHASES"]:
            n_kb, kr0, n_fb, dst0, t0, t1 = (int(mp[f]) for f in ("n_kb", "kr0", "n_fb", "dst0", "t0", "t1"))
            assert 1 <= n_kb <= MMA_MAX_KB and 1 <= n_fb <= MMA_MAX_FB and kr0 % 4 == 0 and t0 < t1
            src = s["ROWS"][kr0:kr0 + 16 * n_kb]
            assert np.all(src < rows) and np.all(src % 132 == 0)
            dst = s["ROWS"][dst0:dst0 + 128 * n_fb]
            real = dst[dst != 0xFFFFFFFF]
            assert np.all(real < rows - 132) and len(set(real.tolist())) == len(real)
            seen = set()
            for t in tiles[t0:t1]:
                assert int(t["data"]) < n_tiles and int(t["fb"]) < n_fb and int(t["kb"]) < n_kb
                assert int(t["acc"]) == (int(t["fb"]) in seen)
                seen.add(int(t["fb"]))
            assert seen == set(range(n_fb))
            assert int(mp["pad0"]) == commits
            commits += -(-(t1 - t0) // 16)
        assert all(int(mp["pad1"]) == commits for mp in s["MMA_PHASES"])
    assert len(s["TABLES"]) == 198
    smem = (P.hdr["n_slots"] + P.hdr["n_scratch"]) * rb + smem_extra_bytes(P.hdr["n_ksel_slots"], P.hdr["qhot_max"], P.hdr["nw"], group)
    assert smem <= SMEM_MAX, smem
    assert RING_QUADS == 32
    assert P.hdr["n_born0"] == P.hdr["n_feat"]
    assert list(s["PAIRS"][:P.hdr["n_born0"], 1]) == [int(d) for d in graph.feat_dims]


def test_plan_residual_slots_never_collide(graph):
    """Two dims sharing a residual row never live in the same sublayer."""
    from qwenputer_b200.plan import compile_plan

    P = compile_plan(graph)
    assert P.hdr["n_slots"] < 1500
    assert P.stats["form_nnz"] < 150_000


def test_gdn_step_rejects_bad_shapes_before_any_launch():
    """gdn_step validates every tensor's shape, dtype and device (and the work buffer's size)
    on the host, so a wrong shape raises instead of reaching the kernels."""
    import torch

    from qwenputer_b200.executor import gdn_check_args

    BH = 4
    ok = dict(S=torch.zeros(BH, 128, 128), q=torch.zeros(BH, 128), k=torch.zeros(BH, 128),
              v=torch.zeros(BH, 128), alpha=torch.ones(BH), beta=torch.ones(BH))
    bad = [("S", torch.zeros(BH, 128, 64)), ("S", torch.zeros(BH * 128, 128)), ("q", torch.zeros(BH + 1, 128)),
           ("k", torch.zeros(BH, 127)), ("v", torch.zeros(BH, 128, 1)), ("alpha", torch.ones(BH, 1)),
           ("beta", torch.ones(BH + 1)), ("q", torch.zeros(BH, 128, dtype=torch.float64)),
           ("k", torch.zeros(128, BH).t())]
    for name, t in bad:
        args = dict(ok, **{name: t})
        with pytest.raises(ValueError, match=name):
            gdn_check_args(**args)
    with pytest.raises(ValueError, match="o must"):
        gdn_check_args(**ok, o=torch.zeros(BH, 64))
    # right shapes, but no CUDA device holds them: still rejected on the host
    with pytest.raises(ValueError, match="CUDA device"):
        gdn_check_args(**ok)


@pytest.mark.parametrize("merged,tc,cluster,group", [(False, False, 1, 32), (False, True, 1, 32), (True, False, 1, 32),
                                                     (True, True, 4, 32), (False, False, 8, 32), (False, False, 1, 4),
                                                     (True, False, 1, 8), (False, False, 1, 16)])
def test_library_accepts_every_plan_variant(graph, merged, tc, cluster, group):
    """qx_create validates a plan before it touches a device: every plan the compiler emits
    (standalone or merged graph, CUDA-core or tensor-core forms, cluster sizes) passes the
    library's validation (without a GPU the call then fails on the device, status 3)."""
    import torch

    from qwenputer_b200 import build
    from qwenputer_b200.graphfile import load_graph, merged_graph_path
    from qwenputer_b200.plan import compile_plan

    if torch.cuda.is_available():
        pytest.skip("checks the validation path that runs before the device is touched")
    lib = C.CDLL(str(build.build()))
    lib.qx_last_error.restype = C.c_char_p
    g = load_graph(merged_graph_path()) if merged else graph
    blob = compile_plan(g, cluster=cluster, tc=tc, group=group).blob()
    h = C.c_void_p()
    st = lib.qx_create(blob, C.c_size_t(len(blob)), 4, 0, C.byref(h))
    assert st == 3, (st, lib.qx_last_error())
