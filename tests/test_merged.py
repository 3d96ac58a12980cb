"""The machine with the text bridge (the merged graph, ``rv32im_merged_graph.npz``) on the CPU:
the oracle against the reference's own evaluator on bridge sessions (tests/golden/merged.npz),
the merged readout (code-dim signs, Q codes naming text tokens) against the reference's
predictions at every position the circuit owns, and the compiled plan (deferred feature loads,
fewer key-select slots) against the oracle on every dim."""

import numpy as np
import pytest

import oracle
from conftest import GOLDEN

SESSIONS = ["echo_short", "echo_words"]


@pytest.fixture(scope="module")
def mgraph():
    from qwenputer_b200.graphfile import load_graph, merged_graph_path

    return load_graph(merged_graph_path())


@pytest.fixture(scope="module")
def moracle(mgraph):
    return oracle.Oracle(mgraph)


@pytest.fixture(scope="module")
def z():
    return np.load(GOLDEN / "merged.npz")


def parked_machine(z):
    """The firmware run to its first park (the reference's bridge.park), on the oracle machine."""
    m = oracle.Machine(z["text"], z["data"].tobytes(), int(z["data_base"]), b"", int(z["entry"]))
    m.run()
    return m


def fnv1a(b: bytes) -> int:
    h = 0xcbf29ce484222325
    for x in b:
        h = ((h ^ x) * 0x100000001b3) & 0xFFFFFFFFFFFFFFFF
    return h


def test_merged_graph_readout_tables(mgraph):
    """The merged graph reads its prediction from 21 code dims; Q names text tokens; every
    printable text token's embedding carries its own Q code on the code dims."""
    assert mgraph.merged and len(mgraph.code_dims) == 21 and len(mgraph.fam_dims) == 0
    col = {int(d): j for j, d in enumerate(mgraph.feat_dims)}
    for p in (0, 10, 65, 256, 259):
        row = mgraph.text_embedding(int(mgraph.printable[p]))
        bits = [int(row[col[int(d)]] > 0) for d in mgraph.code_dims]
        nf = 5
        assert sum(b << i for i, b in enumerate(bits[:nf])) == int(mgraph.q_fid[0])
        assert sum(b << i for i, b in enumerate(bits[nf:])) == p


@pytest.mark.parametrize("name", SESSIONS)
def test_oracle_parked_state_matches_reference(z, name):
    st = parked_machine(z).state()
    assert list(st.x)[1:] == [int(v) for v in z[f"{name}.x"]][1:]
    assert (st.anchor, st.n) == tuple(int(v) for v in z[f"{name}.anchor_n"])
    assert np.array_equal(np.ctypeslib.as_array(st.ram), z[f"{name}.ram"])


@pytest.mark.parametrize("name", SESSIONS)
def test_oracle_matches_reference_on_bridge_session(mgraph, moracle, z, name):
    """Teacher-forced through the session's stream (text, the tool call, the run and its
    echoes): the oracle's float32 residual hashes to the reference evaluator's at every
    position, and the merged readout predicts the stream's next token wherever the circuit owns
    it (the reference's own core.predictions elsewhere too)."""
    st = moracle.new_state(1)
    moracle.snapshot(st, 0, parked_machine(z))
    toks, own, pred = z[f"{name}.tokens"], z[f"{name}.own"], z[f"{name}.pred"]
    for t, tok in enumerate(toks):
        x = mgraph.embed([int(tok)])
        moracle.step(st, x, nthreads=1)
        assert fnv1a(x[0].tobytes()) == int(z[f"{name}.hash"][t]), t
        got = mgraph.decode(x[0])
        if not np.any(x[0, mgraph.code_dims] != 0):
            # no code: the circuit predicts nothing here (RvChat.code_token, chat.py:172-184);
            # core.predictions reads the all-zero bits as family 0, payload 0
            assert got == -1 and int(pred[t]) == 0, t
        else:
            assert got == int(pred[t]), (t, got, int(pred[t]))
        if own[t] and t + 1 < len(toks):
            assert got == int(toks[t + 1]), t


@pytest.mark.parametrize("cluster,tc", [(1, False), (2, True)])
def test_merged_plan_matches_oracle(mgraph, moracle, z, cluster, tc):
    """The compiled merged plan (493 features loaded where first used) through the interpreter
    equals the oracle on every dim for the short session, both sessions as a batch of two."""
    from plan_interp import PlanInterp

    from qwenputer_b200.plan import compile_plan

    P = compile_plan(mgraph, cluster=cluster, tc=tc)
    assert P.stats["deferred_features"] > 400
    it = PlanInterp(P, 2)
    ost = moracle.new_state(2)
    for r in range(2):
        moracle.snapshot(ost, r, parked_machine(z))
    for i in range(len(it.S)):
        it.S[i][...] = ost["S"][i]
    streams = [z[f"{n}.tokens"] for n in SESSIONS]
    for t in range(len(streams[0])):
        emb = mgraph.embed([int(s[t]) for s in streams])
        x = emb.copy()
        it.step(x)
        moracle.step(ost, emb, nthreads=1)
        bad = np.argwhere(x != emb)
        assert not len(bad), (t, bad[:5])


@pytest.mark.parametrize("case", ["calc0", "calc1"])
def test_oracle_runs_calc_tool_call(mgraph, moracle, case):
    """The calculator firmware (qwenputer_b200/calc.py) called through the bridge (tests/golden/
    calc.npz): the oracle's residual hashes to the reference evaluator's at every position of
    the session, and the merged readout predicts every token the circuit owns."""
    zc = np.load(GOLDEN / "calc.npz")
    from qwenputer_b200.calc import calc_program

    p = calc_program()
    assert np.array_equal(p.text, zc["text"])  # the firmware the goldens were made with
    m = oracle.Machine(p.text, b"", p.data_base, b"", p.entry)
    m.run()  # parked
    st = moracle.new_state(1)
    moracle.snapshot(st, 0, m)
    toks, own, hashes = zc[f"{case}.tokens"], zc[f"{case}.own"], zc[f"{case}.hash"]
    for t, tok in enumerate(toks):
        x = mgraph.embed([int(tok)])
        moracle.step(st, x, nthreads=1)
        assert oracle.fnv1a(x[0].view(np.uint32)) == int(hashes[t]), t
        if own[t] and t + 1 < len(toks):
            assert mgraph.decode(x[0]) == int(toks[t + 1]), t
