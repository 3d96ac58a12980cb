"""The multi-GPU run's host logic on CPU: two gloo ranks take their machines (a split of a fixed
job, as `--strong` does, or a shard of their own with seeds that follow the previous rank's, as
the default weak run does), compute each machine's state checksum (here with the oracle machine
instead of the device), and the one all-gather + XOR gives the same run checksum as a single rank
over all machines of the job."""

import os
import socket

import numpy as np
import pytest

torch = pytest.importorskip("torch")

import oracle  # noqa: E402
from qwenputer_b200 import workload  # noqa: E402
from qwenputer_b200.shard import combine, gather_checksums, shard  # noqa: E402

MACHINES, TOKENS, SEED = 6, 300, 4242


def _checksums(b: int, seed0: int) -> np.ndarray:
    progs = workload.workload_programs("many", b, seed0)
    out = []
    for p in progs:
        _, st = oracle.Machine.from_program(p).trace_and_state(TOKENS)
        out.append(st.checksum())
    return np.asarray(out, np.uint64)


def _rank(rank: int, world: int, port: int, q, per: int, weak: bool):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        b, seed0 = shard(per, world, rank, weak, seed=SEED)
        sums = torch.from_numpy(_checksums(b, seed0).view(np.int64))
        allsums = gather_checksums(sums, dist)
        q.put((rank, combine(allsums), allsums.numpy().view(np.uint64).tolist()))
    finally:
        dist.destroy_process_group()


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("per,weak", [(MACHINES, False), (MACHINES // 2, True)])
def test_two_gloo_ranks_gather_the_single_rank_checksum(per, weak):
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q, per, weak)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    want_sums = _checksums(MACHINES, SEED)
    assert res[0][2] == want_sums.tolist() == res[1][2]  # every rank holds all, in machine order
    assert res[0][1] == res[1][1] == combine(want_sums)


def test_shard_rules():
    assert shard(4096, 8, 3) == (512, 1000 + 3 * 512)
    assert shard(4096, 1, 0) == (4096, 1000)
    assert shard(4096, 8, 5, weak=True) == (4096, 1000 + 5 * 4096)
    with pytest.raises(ValueError):
        shard(4096, 3, 0)
