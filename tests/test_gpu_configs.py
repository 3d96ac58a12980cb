"""Parity at the workload sizes the executor is measured on: every trace token and the final
machine state (registers, PC, RAM checksum) against the oracle machine.

  * config 0: one machine of the base generator, 20,000 tokens;
  * config 2: 256 machines (distinct seeds, 1-4 KB data images), 50,000 tokens each;
  * config 3 at full length: 4,096 machines of the bignum mix on one GPU (one CTA per 32
    machines), 100,000 tokens each: every token, and the device state checksums, against the
    oracle machine run on every host thread.
"""

import os
from concurrent.futures import ThreadPoolExecutor

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


@pytest.mark.parametrize("kind,batch,n,seed,tc", [("base", 1, 20000, 1000, False), ("many", 256, 50000, 2000, False),
                                                  ("many", 256, 50000, 2000, True)])
def test_workload_parity(qx, kind, batch, n, seed, tc):
    from qwenputer_b200 import workload

    progs = workload.workload_programs(kind, batch, seed)
    ex = qx.Executor(None, batch=batch, tc=tc)
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


def test_bignum_4096_machines_100k_tokens(qx):
    """4,096 bignum-mix machines x 100,000 tokens each on one GPU (410 M tokens): every generated
    token equals the oracle machine's trace, every machine that has not halted ends in the
    oracle's state (device checksum of registers, PC and RAM), and the device's per-machine token
    hash and count agree with the tokens it wrote."""
    from qwenputer_b200 import workload

    B, n, chunk = 4096, 100_000, 5_000
    progs = workload.workload_programs("bignum", B, 3000)
    ex = qx.Executor(None, batch=B)
    ex.load_machines(0, progs)
    ex.reset()
    go = int(oracle.lib().qxo_tok_family(18, 0))
    ex.set_tokens(0, [go] * B)
    got = np.empty((B, n), np.int32)  # machine-major on the host (1.6 GB)
    dbuf = torch.empty(chunk, B, dtype=torch.int32, device="cuda")
    hbuf = torch.empty(chunk, B, dtype=torch.int32, pin_memory=True)
    for t0 in range(0, n, chunk):
        ex.run(chunk, dbuf)
        hbuf.copy_(dbuf)
        got[:, t0:t0 + chunk] = hbuf.numpy().T
    sums = ex.checksums().cpu().numpy().view(np.uint64)
    hashes = ex.hash.cpu().numpy()
    counts = ex.count.cpu().numpy()
    assert ex.errors() == 0
    assert np.all(counts == n)

    def check(r):
        toks, st = oracle.Machine.from_program(progs[r]).trace_and_state(n)
        want = toks[1:]
        if not np.array_equal(got[r, :len(want)], want):
            return ("tokens", r, int(np.argmax(got[r, :len(want)] != want)))
        if oracle.fnv1a(got[r].view(np.uint32)) != int(hashes[r]):
            return ("hash", r, 0)
        if len(toks) >= n + 1:
            return ("state", r, 0) if int(sums[r]) != st.checksum() else ("ok", r, 1)
        return ("ok", r, 0)

    with ThreadPoolExecutor(max_workers=os.cpu_count() or 1) as pool:
        res = list(pool.map(check, range(B)))
    bad = [x for x in res if x[0] != "ok"]
    assert not bad, bad[:5]
    assert sum(x[2] for x in res) > B // 2  # most machines run the whole 100,000 tokens
