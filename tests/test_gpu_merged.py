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


@pytest.mark.parametrize("batch", [2, 64])
def test_calc_tool_call_free_run(qx, mgraph, batch):
    """The calculator firmware through the bridge on the device (tests/golden/calc.npz): the
    session teacher-forced up to </tool_call>, then the device runs on its own; every token it
    generates equals the reference session's until the circuit hands the stream back, and the
    echoed text is A*B's tool response.  batch 64: the two sessions repeated over 64 machines
    (the merged workload's batch: two groups of 32 machines on clusters of CTAs)."""
    from qwenputer_b200.calc import calc_program, expected_response
    from qwenputer_b200.graphfile import TEXT_TOKEN

    zc = np.load(GOLDEN / "calc.npz")
    names = [str(n) for n in zc["names"]]
    rows = [names[i % len(names)] for i in range(batch)]
    p = calc_program()
    ex = qx.Executor(mgraph, batch=batch)
    ex.load_machines(0, [p] * batch, states=[(zc[f"{n}.x"], int(zc[f"{n}.anchor_n"][0]),
                                              int(zc[f"{n}.anchor_n"][1]), zc[f"{n}.ram"]) for n in rows])
    toks = {n: zc[f"{n}.tokens"] for n in names}
    # </tool_call>: the first text token the circuit owns (both sessions put it at one position)
    tcc = {n: int(next(i for i, v in enumerate(toks[n]) if v >= TEXT_TOKEN and zc[f"{n}.own"][i])) for n in names}
    assert len(set(tcc.values())) == 1
    for t in range(tcc[names[0]] + 1):  # teacher-forced through </tool_call>
        ex.set_tokens(0, [int(toks[n][t]) for n in rows])
        ex.step(ex.x)
    go = [mgraph.decode(v) for v in ex.x.cpu().numpy()]
    assert all(g == int(toks[n][tcc[n] + 1]) for g, n in zip(go, rows))
    n_run = max(len(toks[n]) - tcc[n] for n in names)
    ex.set_tokens(0, go)
    out = torch.empty(n_run, batch, dtype=torch.int32, device="cuda")
    ex.run(n_run, out)
    got = out.cpu().numpy().T.astype(np.int64)
    for r, n in enumerate(rows):
        want = toks[n][tcc[n] + 2:]
        assert np.array_equal(got[r, :len(want)], want), (r, n, int(np.argmax(got[r, :len(want)] != want)))
        echo = [int(v) - TEXT_TOKEN for v in want if v >= TEXT_TOKEN]
        a, b = (int(v) for v in zc[f"{n}.a_b"])
        assert b"".join(mgraph_bytes(mgraph, q) for q in echo[:-1]) == expected_response(a, b)
    assert ex.errors() == 0


def mgraph_bytes(g, q: int) -> bytes:
    """A text token's bytes, from its 128 text-row bits in the graph."""
    w = g.text_words[q]
    row = bytes(sum(((int(w[(8 * k + i) >> 5]) >> ((8 * k + i) & 31)) & 1) << i for i in range(8))
                for k in range(16))
    return row.rstrip(b"\0")


def test_park_matches_reference_parked_state(qx):
    """rvbatch.park (a standalone executor free running the firmware to its exit ecall, the state
    read back) gives the parked state the reference's bridge.park gave (tests/golden/calc.npz)."""
    from qwenputer_b200 import rvbatch
    from qwenputer_b200.calc import calc_program

    zc = np.load(GOLDEN / "calc.npz")
    (x, anchor, n, ram), = rvbatch.park([calc_program()])
    assert list(x)[1:] == [int(v) for v in zc["calc0.x"]][1:]
    assert (anchor, n) == tuple(int(v) for v in zc["calc0.anchor_n"])
    assert np.array_equal(ram, zc["calc0.ram"])


@pytest.mark.parametrize("fp8", [False, True])
def test_conversations_with_qwen_layers(qx, fp8):
    """The merged workload end to end on a small case: 2 conversations of 96 tokens ending in a
    calc tool call, Qwen3.5-4B-shaped layers (4 of them here, random weights; bf16 or fp8 e4m3)
    reading the text, the executor running the calls: both tool responses are A*B's."""
    from qwenputer_b200 import rvbatch

    r = rvbatch.run(batch=2, length=96, fp8=fp8, layers=4, seed=3, chunk=1024)
    assert r["rows_correct"] == 2 and r["device_errors"] == 0
    assert r["fp8_linears"] > 0 if fp8 else r["fp8_linears"] == 0
