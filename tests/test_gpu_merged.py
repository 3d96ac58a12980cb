"""The machine with the text bridge (the merged graph) on the device, against the oracle and the
reference's bridge sessions (tests/golden/merged.npz): teacher-forced steps on every dim, text
tokens embedded on the device, and free-running generation through a tool call's run, whose
echoes (text tokens) and chip tokens the device decodes and embeds itself, until the circuit
hands the stream back."""

import numpy as np
import pytest

import oracle
from conftest import GOLDEN

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
SESSIONS = ["echo_short", "echo_words"]


@pytest.fixture(scope="module")
def qx():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from qwenputer_b200 import build

    build.build()
    from qwenputer_b200 import executor

    return executor


@pytest.fixture(scope="module")
def mgraph():
    from qwenputer_b200.graphfile import load_graph, merged_graph_path

    return load_graph(merged_graph_path())


@pytest.fixture(scope="module")
def z():
    return np.load(GOLDEN / "merged.npz")


def _prog(z):
    from qwenputer_b200.workload import Program

    return Program(z["text"], z["data"].tobytes(), int(z["data_base"]), b"", int(z["entry"]))


def _state(z, name):
    return (z[f"{name}.x"], int(z[f"{name}.anchor_n"][0]), int(z[f"{name}.anchor_n"][1]), z[f"{name}.ram"])


def _loaded(qx, mgraph, z, names, tc=False, cluster=None):
    ex = qx.Executor(mgraph, batch=len(names), tc=tc, cluster=cluster)
    ex.load_machines(0, [_prog(z)] * len(names), states=[_state(z, n) for n in names])
    return ex


@pytest.mark.parametrize("tc,cluster", [(False, None), (False, 1), (True, 1)])
def test_merged_steps_match_oracle(qx, mgraph, z, tc, cluster):
    """Both sessions as a batch, teacher-forced through the short one's length: every dim equals
    the oracle's step, and the residual hashes to the reference evaluator's."""
    from test_merged import fnv1a, parked_machine

    ex = _loaded(qx, mgraph, z, SESSIONS, tc, cluster)
    o = oracle.Oracle(mgraph)
    ost = o.new_state(2)
    for r in range(2):
        o.snapshot(ost, r, parked_machine(z))
    streams = [z[f"{n}.tokens"] for n in SESSIONS]
    for t in range(len(streams[0])):
        emb = mgraph.embed([int(s[t]) for s in streams])
        x = torch.from_numpy(emb).cuda()
        ex.step(x)
        o.step(ost, emb)
        got = x.cpu().numpy()
        assert np.array_equal(got, emb), (t, np.argwhere(got != emb)[:5])
        for r, n in enumerate(SESSIONS):
            assert fnv1a(got[r].tobytes()) == int(z[f"{n}.hash"][t]), (n, t)
    assert ex.errors() == 0


def test_text_tokens_embedded_on_device(qx, mgraph):
    """qx_set_tokens of text tokens (bytes, the tool-call markers, multi-byte tokens) and chip
    tokens writes the embeddings the graph's tables give."""
    from qwenputer_b200.graphfile import TEXT_TOKEN

    toks = [TEXT_TOKEN + q for q in (0, 10, 65, 255, 256, 257, 258, 263, 300, 4359)] + [230322, 0, 65537]
    ex = qx.Executor(mgraph, batch=len(toks))
    ex.set_tokens(0, toks)
    torch.cuda.synchronize()
    assert np.array_equal(ex.x.cpu().numpy(), mgraph.embed(toks))
    assert ex.errors() == 0


@pytest.mark.parametrize("tc", [False, True])
def test_merged_free_run_through_a_tool_call(qx, mgraph, z, tc):
    """Each session teacher-forced up to its </tool_call>, then free running on the device: every
    token the circuit owns (GO, the run's records, each putchar's echo as a text token, the
    closing </tool_response>, the HALT's newline echo) equals the reference session's; after the
    newline the circuit predicts nothing (-1)."""
    from qwenputer_b200.graphfile import TEXT_TOKEN

    TCC = next(q for q in range(len(mgraph.text_words)) if mgraph.text_words[q, 4] >> (129 - 128) & 1)
    for name in SESSIONS:
        toks, own = z[f"{name}.tokens"], z[f"{name}.own"]
        i_tcc = int(np.flatnonzero(toks == TEXT_TOKEN + TCC)[0])
        ex = _loaded(qx, mgraph, z, [name], tc, 1)
        for t in range(i_tcc + 1):
            x = torch.from_numpy(mgraph.embed([int(toks[t])])).cuda()
            ex.step(x)
        go = mgraph.decode(x[0].cpu().numpy())
        assert go == int(toks[i_tcc + 1])
        want = [int(v) for v in toks[i_tcc + 2:]]
        n = len(want) + 1
        ex.set_tokens(0, [go])
        out = torch.empty(n, 1, dtype=torch.int32, device="cuda")
        ex.run(n, out)
        got = out[:, 0].cpu().numpy().astype(np.int64)
        assert list(got[:len(want)]) == want, (name, int(np.argmax(got[:len(want)] != want)))
        assert not own[-1] and got[len(want)] == -1
        assert sum(v >= TEXT_TOKEN for v in want) >= 3  # echoes were decoded as text tokens
        assert ex.errors() == 0
