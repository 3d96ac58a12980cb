"""The compiled phase program, run by a CPU interpreter, equals the oracle's Executor2 step on
every dim (checks the plan compiler: residual slots, form groups, lag staging, temporaries)."""

import numpy as np
import pytest

import oracle
from plan_interp import PlanInterp


@pytest.mark.parametrize("names,cluster,tc,group", [(["gen_small_7", "div_fuzz_0"], 1, False, 32),
                                                     (["digit_file", "refresh_70"], 8, False, 32),
                                                     (["gen_bignum_5", "mul_fuzz_1"], 1, True, 32),
                                                     (["zba_rodata", "div_fuzz_1"], 4, True, 32),
                                                     (["gen_bignum_5", "digit_file"], 1, False, 16),
                                                     (["mul_fuzz_1", "refresh_70"], 1, False, 8),
                                                     (["div_fuzz_0", "zba_rodata"], 1, False, 4)])
def test_plan_program_matches_oracle(oracle_, graph, programs, names, cluster, tc, group):
    from qwenputer_b200.plan import compile_plan

    P = compile_plan(graph, cluster=cluster, tc=tc, group=group)
    B = len(names)
    it = PlanInterp(P, B)
    ost = oracle_.new_state(B)
    for r, n in enumerate(names):
        oracle_.snapshot(ost, r, oracle.Machine.from_program(programs[n]["prog"]))
    for i in range(len(it.S)):
        it.S[i][...] = ost["S"][i]
    traces = [programs[n]["trace"] for n in names]
    for t in range(12):
        toks = [int(tr[min(t, len(tr) - 1)]) for tr in traces]
        emb = graph.embed(toks)
        x = emb.copy()
        it.step(x)
        oracle_.step(ost, emb, nthreads=1)
        bad = np.argwhere(x != emb)
        assert not len(bad), (t, [(int(b), int(d), x[b, d], emb[b, d]) for b, d in bad[:5]])
    for i in range(len(it.S)):
        assert np.array_equal(it.S[i], ost["S"][i]), i
