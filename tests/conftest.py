"""Shared fixtures. Tests marked ``gpu`` need a B200; everything else runs on CPU."""

import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(REPO))
sys.path.insert(0, str(REPO / "oracle"))
GOLDEN = REPO / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


@pytest.fixture(scope="session")
def graph():
    from qwenputer_b200.graphfile import default_graph_path, load_graph

    return load_graph(default_graph_path())


@pytest.fixture(scope="session")
def oracle_(graph):
    import oracle

    return oracle.Oracle(graph)


@pytest.fixture(scope="session")
def programs():
    import numpy as np

    from qwenputer_b200.workload import Program

    z = np.load(GOLDEN / "programs.npz")
    out = {}
    for n in z["names"]:
        n = str(n)
        out[n] = {
            "prog": Program(z[f"{n}.text"], z[f"{n}.data"].tobytes(), int(z[f"{n}.data_base"]),
                            z[f"{n}.rodata"].tobytes(), int(z[f"{n}.entry"])),
            "trace": z[f"{n}.trace"].astype(np.int64), "x": z[f"{n}.x"],
            "anchor_n": z[f"{n}.anchor_n"], "ram": z[f"{n}.ram"], "halted": bool(z[f"{n}.halted"]),
        }
    return out
