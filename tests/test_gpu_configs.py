"""Parity at the workload sizes the executor is measured on: every trace token and the final
machine state (registers, PC, RAM checksum) against the oracle machine.

  * config 0: one machine of the base generator, 20,000 tokens;
  * config 2: 256 machines (distinct seeds, 1-4 KB data images), 50,000 tokens each;
  * config 3's batch: 4,096 machines of the bignum mix on one GPU (one CTA per 32 machines),
    1,500 tokens each (the full 100,000-token runs are the bench's; their device checksums are
    what the multi-GPU gather combines).
"""

import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def qx():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from qwenputer_b200 import build

    build.build()
    from qwenputer_b200 import executor

    return executor


@pytest.mark.parametrize("kind,batch,n,seed", [("base", 1, 20000, 1000), ("many", 256, 50000, 2000),
                                               ("bignum", 4096, 1500, 3000)])
def test_workload_parity(qx, kind, batch, n, seed):
    from qwenputer_b200 import workload

    progs = workload.workload_programs(kind, batch, seed)
    ex = qx.Executor(None, batch=batch)
    ex.load_machines(0, progs)
    ex.reset()
    go = int(oracle.lib().qxo_tok_family(18, 0))  # GO: the seventh control after 12 families
    ex.set_tokens(0, [go] * batch)
    out = torch.empty(n, batch, dtype=torch.int32, device="cuda")
    chunk = 10000
    for t0 in range(0, n, chunk):
        ex.run(min(chunk, n - t0), out[t0:t0 + chunk])
    got = out.cpu().numpy().T
    sums = ex.checksums().cpu().numpy().view(np.uint64)
    assert ex.errors() == 0
    compared = 0
    for r, p in enumerate(progs):
        toks, st = oracle.Machine.from_program(p).trace_and_state(n)
        want = toks[1:]
        assert np.array_equal(got[r, :len(want)], want), (r, int(np.argmax(got[r, :len(want)] != want)))
        if len(toks) >= n + 1:  # not halted: the states must agree too
            assert int(sums[r]) == st.checksum(), r
            compared += 1
    assert compared > 0
