"""qx_gdn_step_noalloc, the gated delta-rule step for callers that cannot allocate device memory.

Some callers of the step may not call cudaMalloc: hosts whose own allocator has been handed the
whole device heap, and latency-bound loops in which an allocation, which can synchronise the
device, is not allowed.  For them the library keeps the step's scratch in a fixed array of its
own (QX_GDN_NOALLOC_MAX_BH heads).  These tests call that entry point through the C ABI and check
that it gives the same states and outputs as qx_gdn_step with a caller-provided scratch buffer,
bit for bit, on two calls in a row (the second sees the array as the first left it).  The file is
named to be collected last, so that it also runs after every other test in one process; it passes
alone in a fresh process too.
"""

import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

HD = 128


@pytest.fixture(scope="module")
def lib():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from qwenputer_b200 import build

    build.build()
    from qwenputer_b200 import executor

    return executor.lib()


def _case(BH, seed, general):
    g = torch.Generator().manual_seed(seed)
    S = torch.randint(0, 2, (BH, HD, HD), generator=g).float()
    k = torch.zeros(BH, HD)
    k[torch.arange(BH), torch.randint(0, HD, (BH,), generator=g)] = 1.0
    gen = torch.rand(BH, generator=g) < general
    kg = torch.randn(int(gen.sum()), HD, generator=g)
    k[gen] = kg / kg.norm(dim=1, keepdim=True)
    q = torch.zeros(BH, HD)
    q[torch.arange(BH), torch.randint(0, HD, (BH,), generator=g)] = 1.0
    v = torch.randint(0, 2, (BH, HD), generator=g).float()
    u = torch.rand(BH, generator=g)
    alpha = torch.where(u < 0.9, 1.0, torch.where(u < 0.95, 0.5, 0.0))
    beta = torch.ones(BH)
    return [t.cuda() for t in (S, q, k, v, alpha, beta)]


def _ptr(t):
    return C.c_void_p(t.data_ptr())


def _stream():
    return C.c_void_p(torch.cuda.current_stream().cuda_stream)


def _with_buffer(lib, S, q, k, v, alpha, beta):
    BH = S.shape[0]
    o = torch.empty(BH, HD, device="cuda")
    work = torch.empty(int(lib.qx_gdn_work_bytes(BH)), dtype=torch.uint8, device="cuda")
    st = lib.qx_gdn_step(C.c_int64(BH), *[_ptr(t) for t in (S, q, k, v, alpha, beta, o, work)], _stream())
    assert st == 0, lib.qx_last_error()
    return o, work[4:8].view(torch.int32)


def _no_alloc(lib, S, q, k, v, alpha, beta):
    BH = S.shape[0]
    o = torch.empty(BH, HD, device="cuda")
    err = torch.full((1,), -1, dtype=torch.int32, device="cuda")
    st = lib.qx_gdn_step_noalloc(C.c_int64(BH), *[_ptr(t) for t in (S, q, k, v, alpha, beta, o, err)], _stream())
    assert st == 0, lib.qx_last_error()
    return o, err


@pytest.mark.parametrize("BH,seed,general", [(3000, 21, 0.05), (49152, 22, 0.05), (700, 23, 1.0)])
def test_no_alloc_matches_buffered_step_twice(lib, BH, seed, general):
    S, q, k, v, alpha, beta = _case(BH, seed, general)
    Sa, Sb = S.clone(), S.clone()
    for call in range(2):
        oa, ea = _with_buffer(lib, Sa, q, k, v, alpha, beta)
        ob, eb = _no_alloc(lib, Sb, q, k, v, alpha, beta)
        torch.cuda.synchronize()
        # exact arithmetic on {0, 1/2, 1}-valued states: the two paths agree bit for bit
        assert torch.equal(oa, ob), call
        assert torch.equal(Sa, Sb), call
        assert int(ea.item()) == 0 and int(eb.item()) == 0, call
        # the second call: other query and key rows, states as the first call left them
        q, k = q.roll(1, 0), k.roll(3, 0)


def test_no_alloc_rejects_too_many_heads(lib):
    big = 65536 + 1
    null = C.c_void_p(0)
    st = lib.qx_gdn_step_noalloc(C.c_int64(big), null, null, null, null, null, null, null, null, _stream())
    assert st != 0
    assert b"at most 65536" in lib.qx_last_error()
