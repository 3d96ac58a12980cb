"""The drop-in boundary with a live graph: the reference's own ``core.build()`` graph, exported on
the fly, equals the graph file the package ships, ``load_init``'s host buffers equal the reference
snapshot hashes, and the ``Executor2`` binding of the integration notes constructs from the live
graph.

These tests import the reference tree (``experimental/riscv``), given by ``QX_REFERENCE_ROOT`` or
found as a ``reference`` checkout beside this repository; they skip where it is absent.  CPU
only: nothing here launches a kernel unless a CUDA device is present.
"""

from __future__ import annotations

import dataclasses
import os
import sys
from pathlib import Path
from types import SimpleNamespace

import numpy as np
import pytest

from conftest import GOLDEN, REPO


def _reference_root() -> Path | None:
    env = os.environ.get("QX_REFERENCE_ROOT")
    for cand in ([Path(env)] if env else []) + [REPO.parent / "reference" / "experimental" / "riscv"]:
        if (cand / "chipformer" / "rv" / "core.py").exists():
            return cand
    return None


ROOT = _reference_root()
pytestmark = pytest.mark.skipif(ROOT is None, reason="the reference tree is not available")


@pytest.fixture(scope="module")
def live():
    sys.dont_write_bytecode = True  # the reference tree is read-only
    sys.path.insert(0, str(ROOT))
    from chipformer.rv import core

    return core.build()


def _equal(a, b, path=""):
    if dataclasses.is_dataclass(a):
        assert type(a) is type(b), path
        for f in dataclasses.fields(a):
            _equal(getattr(a, f.name), getattr(b, f.name), f"{path}.{f.name}")
    elif isinstance(a, np.ndarray):
        b = np.asarray(b)
        assert a.shape == b.shape and a.dtype.kind == b.dtype.kind, path
        assert np.array_equal(a, b), path
    else:
        assert a == b, path


def test_export_of_live_graph_equals_shipped_file(live):
    """graphfile.export_graph(core.build()) == qwenputer_b200/plans/rv32im_graph.npz, field by field."""
    from qwenputer_b200.graphfile import default_graph_path, export_graph, load_graph

    _equal(export_graph(live), load_graph(default_graph_path()), "GraphData")


def test_live_graph_compiles_to_the_shipped_plan(live):
    """The plan blob compiled from the live graph is the one compiled from the shipped file."""
    from qwenputer_b200.executor import load_graph as ex_load_graph
    from qwenputer_b200.graphfile import default_graph_path, load_graph
    from qwenputer_b200.plan import compile_plan

    assert compile_plan(ex_load_graph(live)).blob() == compile_plan(load_graph(default_graph_path())).blob()


def test_load_init_buffers_match_reference_snapshot_hashes(live, programs):
    """core.snapshot(c, m) then Executor.load_init's host buffers (snapshot_states): every head
    sublayer's [V, 128, 128] state hashes to the value the reference's own Executor2.load_init
    buffers hashed to (tests/golden/snapshot.npz)."""
    from chipformer.rv import core, ref

    from qwenputer_b200.executor import snapshot_states
    from qwenputer_b200.graphfile import default_graph_path, load_graph

    sys.path.insert(0, str(REPO / "tests" / "golden"))
    from make_golden import fnv1a_bytes

    z = np.load(GOLDEN / "snapshot.npz")
    levels = load_graph(default_graph_path()).head_sublayers()
    for name in ["gen_base_0", "digit_file", "zba_rodata", "fault_ecall", "div_fuzz_1"]:
        p = programs[name]["prog"]
        p = SimpleNamespace(text=[int(w) for w in p.text], data=bytes(p.data), data_base=int(p.data_base),
                            entry=int(p.entry), rodata=bytes(p.rodata))  # plain ints, as the reference expects
        core.snapshot(live, ref.Machine.from_program(p))
        bufs = snapshot_states(live, levels)
        got = [fnv1a_bytes(b.tobytes()) for b in bufs]
        assert got == [int(h) for h in z[name]], name


def test_executor2_binding_constructs_from_live_graph(live):
    """The binding the integration notes add to tritonexec.py: Executor2(c, batch, device) as a
    subclass of the shim.  With a CUDA device it constructs from the live graph, loads the
    snapshot with load_init and steps; without one it raises the shim's error (no CPU path)."""
    import torch

    from qwenputer_b200.executor import Executor as _QxExecutor
    from qwenputer_b200.executor import QxError

    class Executor2(_QxExecutor):
        pass

    if not torch.cuda.is_available():
        with pytest.raises(QxError, match="CUDA"):
            Executor2(live, 2, "cuda")
        return
    ex = Executor2(live, 2, "cuda")
    assert ex.D == live.dims
    ex.load_init(0)
    x = ex.embed([0, 0])
    ex.step(x)
    torch.cuda.synchronize()


def test_export_of_live_merged_graph_equals_shipped_file():
    """graphfile.export_graph(core.build(text=ByteVocab())) == plans/rv32im_merged_graph.npz, field
    by field: the merged readout (code dims, keep dims, the Q family) and every text token's
    bits, which the export checks against the graph's own feature functions."""
    from chipformer.rv import core

    from qwenputer_b200.graphfile import export_graph, load_graph, merged_graph_path
    from qwenputer_b200.plans.export_rv32im import ByteVocab

    _equal(export_graph(core.build(text=ByteVocab())), load_graph(merged_graph_path()), "GraphData")
