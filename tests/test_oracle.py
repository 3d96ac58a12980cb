"""The CPU oracle against golden vectors produced by the reference itself (tests/golden/)."""

import ctypes as C

import numpy as np
import pytest

import oracle
from conftest import GOLDEN


def fnv_rows(a: np.ndarray) -> np.ndarray:
    """FNV-1a 64 of every row's bytes (float32 rows seen as 32-bit words)."""
    return np.asarray([oracle.fnv1a(np.ascontiguousarray(r).view(np.uint32)) for r in a],
                      np.uint64)


def test_machine_traces_and_states(programs):
    """ref.Machine.run (ERV/chipformer/rv/ref.py:600-605) on every golden program."""
    for name, p in programs.items():
        m = oracle.Machine.from_program(p["prog"])
        toks = m.run(60000)
        assert np.array_equal(toks, p["trace"]), name
        st = m.state()
        assert list(st.x)[1:] == list(p["x"])[1:], name
        assert (st.anchor, st.n) == tuple(p["anchor_n"]), name
        assert np.array_equal(np.ctypeslib.as_array(st.ram), p["ram"]), name


def test_rom_words():
    z = np.load(GOLDEN / "romword.npz")
    got = np.asarray([oracle.rom_word(int(w), int(pc)) for w, pc in zip(z["w"], z["pc"])], np.uint32)
    assert np.array_equal(got, z["rom"])


def test_div_records():
    """DIV-class records (ERV/tests/test_rv_ref.py:97-110) on edge and random operands."""
    z = np.load(GOLDEN / "divrec.npz")
    buf = np.zeros(32, np.int32)
    for op, a, b, rec, n in zip(z["op"], z["a"], z["b"], z["rec"], z["len"]):
        ln = oracle.lib().qxo_div_record(C.c_int32(int(op)), C.c_uint32(int(a)), C.c_uint32(int(b)),
                                         buf.ctypes.data_as(C.POINTER(C.c_int32)), C.c_int64(32))
        assert ln == n and np.array_equal(buf[:n], rec[:n]), (op, a, b)


def test_snapshot_matches_load_init(oracle_, programs):
    """core.snapshot + Executor2.load_init (ERV/chipformer/rv/core.py:1218-1270,
    tritonexec.py:246-258): every head sublayer's state, bit for bit."""
    z = np.load(GOLDEN / "snapshot.npz")
    st = oracle_.new_state(1)
    for name in ["gen_base_0", "gen_bignum_5", "digit_file", "zba_rodata", "div_fuzz_1"]:
        oracle_.snapshot(st, 0, oracle.Machine.from_program(programs[name]["prog"]))
        got = np.asarray([oracle.fnv1a(s[0].reshape(-1).view(np.uint32)) for s in st["S"]], np.uint64)
        assert np.array_equal(got, z[name]), name


def test_readback_inverts_snapshot(oracle_, programs):
    st = oracle_.new_state(1)
    for name in ["gen_base_1", "zba_rodata"]:
        m = oracle.Machine.from_program(programs[name]["prog"])
        m.run(3000)
        oracle_.snapshot(st, 0, m)
        rb = oracle_.readback(st, 0)
        ms = m.state()
        assert list(rb.x)[1:] == list(ms.x)[1:]
        assert (rb.anchor, rb.n) == (ms.anchor, ms.n)
        assert np.array_equal(np.ctypeslib.as_array(rb.ram), np.ctypeslib.as_array(ms.ram))
        assert rb.checksum() == ms.checksum()


RESIDUAL_CASES = ["gen_small_7", "div_fuzz_0", "mul_fuzz_0", "zba_rodata", "digit_file",
                  "fault_bad_jump", "refresh_70", "csr_putchar", "gen_bignum_5", "gen_base_0"]


@pytest.mark.parametrize("name", RESIDUAL_CASES)
def test_step_matches_ir_evaluate(oracle_, graph, programs, name):
    """Teacher-forced: the oracle's Executor2 step equals ir.evaluate (fp64, exact) on every dim
    at every position (tritonexec.py:292-305 check), and the decoded code equals
    core.predictions."""
    z = np.load(GOLDEN / "residual.npz")
    toks = z[f"{name}.tokens"].astype(np.int64)
    n = min(len(toks), 250)
    st = oracle_.new_state(1)
    oracle_.snapshot(st, 0, oracle.Machine.from_program(programs[name]["prog"]))
    emb = graph.embed(toks[:n])
    for t in range(n):
        x = emb[t:t + 1].copy()
        oracle_.step(st, x, nthreads=1)
        if t < 8:
            assert np.array_equal(x[0], z[f"{name}.head"][t]), (name, t)
        assert fnv_rows(x)[0] == z[f"{name}.hash"][t], (name, t)
        tok, _, bad = oracle_.decode(x)
        want = int(z[f"{name}.pred"][t])
        if want >= 0:
            assert tok[0] == want and bad == 0, (name, t)


def test_free_run_matches_trace(oracle_, programs):
    """FreeRun (fastexec.py:298-340) on the oracle: each prediction is the next input."""
    p = programs["gen_small_7"]
    st = oracle_.new_state(1)
    oracle_.snapshot(st, 0, oracle.Machine.from_program(p["prog"]))
    n = 200
    got = oracle_.free_run(st, [int(p["trace"][0])], n)[0]
    assert np.array_equal(got, p["trace"][1:n + 1])


def test_gdn_one_hot_matches_transformers():
    """One-hot keys / queries: the oracle's state equals transformers'
    torch_recurrent_gated_delta_rule bit for bit; its read equals the scaled-back query's read."""
    z = np.load(GOLDEN / "gdn.npz")
    B, H, dk, dv = z["S"].shape
    S = np.ascontiguousarray(z["S"].reshape(B * H, dk, dv).astype(np.float32))
    o = oracle.gdn_step(S, z["q"].reshape(B * H, dk), z["k"].reshape(B * H, dk),
                        z["v"].reshape(B * H, dv), z["alpha"].reshape(-1), z["beta"].reshape(-1))
    assert np.array_equal(S, z["S_out"].reshape(B * H, dk, dv))
    np.testing.assert_allclose(o, z["o"].reshape(B * H, dv), rtol=1e-6, atol=0)


# Max-abs tolerance of the general (non-one-hot key) gated delta-rule path against transformers'
# torch_recurrent_gated_delta_rule: the oracle sums over the key index in order (each product
# rounded before it is added), torch's .sum(dim=-2) in its own reduction order, so the last bits
# differ (measured: at most 2.4e-7 on values of magnitude <= 2, i.e. 2 ulp).
GDN_GENERAL_ATOL = 1e-6


@pytest.mark.parametrize("case", ["gauss", "mix"])
def test_gdn_general_keys_match_transformers(case):
    """Unit-norm Gaussian keys (every head, beta in {1, 1/2}; and the 1,024 x 48-head step's mix):
    the oracle's state and read agree with transformers' recurrence within GDN_GENERAL_ATOL, and
    heads with a one-hot key and alpha == 1 agree bit for bit."""
    z = np.load(GOLDEN / "gdn_general.npz")
    B, H, dk, dv = z[f"{case}.S"].shape
    S = np.ascontiguousarray(z[f"{case}.S"].reshape(B * H, dk, dv).astype(np.float32))
    k = z[f"{case}.k"].reshape(B * H, dk)
    al = z[f"{case}.alpha"].reshape(-1)
    o = oracle.gdn_step(S, z[f"{case}.q"].reshape(B * H, dk), k, z[f"{case}.v"].reshape(B * H, dv), al,
                        z[f"{case}.beta"].reshape(-1))
    S_ref = z[f"{case}.S_out"].reshape(B * H, dk, dv)
    o_ref = z[f"{case}.o"].reshape(B * H, dv)
    assert np.abs(S - S_ref).max() <= GDN_GENERAL_ATOL
    assert np.abs(o - o_ref).max() <= GDN_GENERAL_ATOL
    light = ((k != 0).sum(1) == 1) & (al == 1.0)
    if light.any():
        assert np.array_equal(S[light], S_ref[light])


@pytest.mark.parametrize("name", ["div_fuzz_0", "gen_small_7"])
def test_oracle_step_matches_stock_hf_modules(graph, oracle_, programs, name):
    """A third witness for the compiled weights: the reference emits the stack as stock
    transformers Qwen3_5ForCausalLM weights (bf16, torch kernels) and decodes the trace from the
    injected snapshot (tests/golden/hf_residual.npz); the oracle's residual equals those modules'
    on every dim at every position."""
    h = np.load(GOLDEN / "hf_residual.npz")
    st = oracle_.new_state(1)
    oracle_.snapshot(st, 0, oracle.Machine.from_program(programs[name]["prog"]))
    want = h[f"{name}.resid"]
    for t, tok in enumerate(h[f"{name}.tokens"]):
        x = graph.embed([int(tok)])
        oracle_.step(st, x, nthreads=1)
        bad = np.nonzero(x[0, 1:] != want[t])[0]
        assert not len(bad), (t, bad[:5])
