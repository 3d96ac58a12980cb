"""The CUDA executor against the CPU oracle (bit-exact tokens and states; residuals equal on every
dim, as the reference's own check compares them: tritonexec.py:292-305)."""

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


def _oracle_state(o, progs):
    st = o.new_state(len(progs))
    for r, p in enumerate(progs):
        o.snapshot(st, r, oracle.Machine.from_program(p))
    return st


def test_load_machines_matches_snapshot(qx, oracle_, programs):
    names = ["gen_base_0", "digit_file", "zba_rodata", "gen_bignum_5", "fault_ecall"]
    progs = [programs[n]["prog"] for n in names]
    ex = qx.Executor(None, batch=len(progs))
    ex.load_machines(0, progs)
    want = _oracle_state(oracle_, progs)
    heads = [s for s in ex.steps if s["kind"] == "head"]
    for i, st in enumerate(heads):
        got = st["S"].cpu().numpy()
        assert np.array_equal(got, want["S"][i]), f"head sublayer {i}"


def test_load_over_used_state(qx, oracle_, programs):
    """A load writes every head-state row of its machines: rows that held other values (garbage,
    or a machine that ran before) end equal to the snapshot, rows of other machines keep theirs,
    and the reloaded machines then run as fresh ones."""
    names = ["gen_bignum_5", "zba_rodata", "digit_file", "gen_base_0", "div_fuzz_0", "mul_fuzz_1"]
    progs = [programs[n]["prog"] for n in names]
    ex = qx.Executor(None, batch=6)
    heads = [s for s in ex.steps if s["kind"] == "head"]
    for st in heads:
        st["S"].fill_(-3.25)
    ex.load_machines(1, progs[:4])
    torch.cuda.synchronize()
    want = _oracle_state(oracle_, progs[:4])
    for i, st in enumerate(heads):
        got = st["S"].cpu().numpy()
        assert np.array_equal(got[1:5], want["S"][i]), f"head sublayer {i}"
        assert (got[0] == -3.25).all() and (got[5] == -3.25).all(), f"head sublayer {i}: rows outside the load"
    # every machine valid, 40 free-running tokens, then rows 1-4 reloaded with other programs
    go = int(oracle.lib().qxo_tok_family(18, 0))
    ex.load_machines(0, progs)
    ex.reset()
    ex.set_tokens(0, [go] * 6)
    ex.run(40)
    again = progs[1:5][::-1]
    ex.load_machines(1, again)
    torch.cuda.synchronize()
    want = _oracle_state(oracle_, again)
    for i, st in enumerate(heads):
        assert np.array_equal(st["S"].cpu().numpy()[1:5], want["S"][i]), f"head sublayer {i} after a run"
    ex.reset()
    ex.set_tokens(0, [go] * 6)
    n = 300
    out = torch.zeros(n, 6, dtype=torch.int32, device="cuda")
    ex.run(n, out)
    got = out.cpu().numpy().T
    for r, p in enumerate(again, start=1):
        toks = oracle.Machine.from_program(p).trace_and_state(n)[0][1:]
        assert np.array_equal(got[r, :len(toks)], toks), r
    assert ex.errors() == 0


@pytest.mark.parametrize("batch,cluster,tc,group", [(1, None, False, None), (5, 1, False, None),
                                                    (37, None, False, None), (37, 2, False, None),
                                                    (37, None, False, 16), (37, None, False, 8),
                                                    (1, None, True, None), (37, 1, True, None), (37, 4, True, None)])
def test_step_matches_oracle(qx, oracle_, graph, programs, batch, cluster, tc, group):
    """Teacher-forced steps: every dim of every row equals the oracle's Executor2 step (cluster
    and group None: the executor's own choice, 4 machines a CTA at these batches; a cluster:
    groups of 32 on that many CTAs; tc: linear forms on the tensor cores)."""
    pool = ["gen_small_7", "div_fuzz_0", "mul_fuzz_1", "digit_file", "gen_base_1", "refresh_70",
            "zba_rodata", "gen_many_11", "csr_putchar"]
    names = [pool[i % len(pool)] for i in range(batch)]
    progs = [programs[n]["prog"] for n in names]
    traces = [programs[n]["trace"] for n in names]
    ex = qx.Executor(None, batch=batch, cluster=cluster, tc=tc, group=group)
    ex.load_machines(0, progs)
    ost = _oracle_state(oracle_, progs)
    T = 60 if batch > 8 else 120
    for t in range(T):
        toks = [int(tr[min(t, len(tr) - 1)]) for tr in traces]
        emb = graph.embed(toks)
        x = torch.from_numpy(emb).cuda()
        ex.step(x)
        oracle_.step(ost, emb)
        got = x.cpu().numpy()
        bad = np.argwhere(got != emb)
        assert not len(bad), (t, bad[:5], got[tuple(bad[0])], emb[tuple(bad[0])])
    for i, st in enumerate([s for s in ex.steps if s["kind"] == "head"]):
        assert np.array_equal(st["S"].cpu().numpy(), ost["S"][i])
    assert ex.errors() == 0


@pytest.mark.parametrize("batch,n,cluster,tc,group", [(1, 3000, None, False, None), (40, 1500, None, False, None),
                                                      (40, 1500, None, False, 8), (40, 1500, None, False, 16),
                                                      (40, 1500, 1, False, None), (40, 1500, 1, True, None),
                                                      (1, 3000, None, True, None)])
def test_free_run_matches_machine(qx, programs, batch, n, cluster, tc, group):
    """Free-running generation: every token equals the traced machine's, and the machine state
    read back from the heads equals the traced state after the last complete record."""
    from qwenputer_b200 import workload

    progs = [programs[k]["prog"] for k in sorted(programs)]
    progs += workload.workload_programs("many", max(0, batch - len(progs)), 500)
    progs = progs[:batch]
    ex = qx.Executor(None, batch=batch, cluster=cluster, tc=tc, group=group)
    ex.load_machines(0, progs)
    ex.reset()
    go = int(oracle.lib().qxo_tok_family(18, 0))  # GO: the seventh control after 12 families
    ex.set_tokens(0, [go] * batch)
    out = torch.zeros(n, batch, dtype=torch.int32, device="cuda")
    ex.run(n, out)
    got = out.cpu().numpy().T
    sums = ex.checksums().cpu().numpy().view(np.uint64)
    for r, p in enumerate(progs):
        toks, st = oracle.Machine.from_program(p).trace_and_state(n)
        want = toks[1:]
        assert np.array_equal(got[r, :len(want)], want), (r, np.argmax(got[r, :len(want)] != want))
        if len(toks) < n + 1:
            continue  # halted: the reference machine stops there, the circuit does not
        rb = ex.readback(r)
        assert list(rb.x)[1:] == list(st.x)[1:], r
        assert (rb.anchor, rb.n) == (st.anchor, st.n), r
        assert np.array_equal(np.ctypeslib.as_array(rb.ram), np.ctypeslib.as_array(st.ram)), r
        assert int(sums[r]) == st.checksum(), r
    assert ex.errors() == 0


def test_machine_groups_agree(qx):
    """Groups of 32, 16, 8 and 4 machines a CTA (the smaller ones with 2, 4 and 8 stream records
    side by side in a warp): the same tokens, states, checksums and residuals (100 machines of the
    bignum workload, a partial last group, 400 tokens)."""
    from qwenputer_b200 import workload

    B = 100
    progs = workload.workload_programs("bignum", B, 78)
    go = int(oracle.lib().qxo_tok_family(18, 0))
    outs = []
    for group in (32, 16, 8, 4):
        ex = qx.Executor(None, batch=B, group=group, cluster=1 if group == 32 else None)
        assert ex.group == group and ex.info(2) == -(-B // group)
        ex.load_machines(0, progs)
        ex.reset()
        ex.set_tokens(0, [go] * B)
        out = torch.zeros(400, B, dtype=torch.int32, device="cuda")
        ex.run(400, out)
        heads = [s["S"] for s in ex.steps if s["kind"] == "head"]
        outs.append((out.cpu().numpy(), ex.checksums().cpu().numpy(),
                     [float(h.double().sum()) for h in heads], ex.x.cpu().numpy()))
        assert ex.errors() == 0
        del ex
    for o in outs[1:]:
        assert np.array_equal(o[0], outs[0][0])
        assert np.array_equal(o[1], outs[0][1])
        assert o[2] == outs[0][2]
        assert np.array_equal(o[3], outs[0][3])


def test_cluster_sizes_agree(qx):
    """One group of 32 machines on 1, 2, 4 or 8 CTAs of a cluster, linear forms on the CUDA cores
    or the tensor cores: the same tokens, states and checksums (96 machines of the bignum
    workload, 400 tokens)."""
    from qwenputer_b200 import workload

    progs = workload.workload_programs("bignum", 96, 77)
    go = int(oracle.lib().qxo_tok_family(18, 0))
    outs = []
    for cluster, tc in ((1, False), (2, False), (4, False), (8, False), (1, True), (2, True), (8, True)):
        ex = qx.Executor(None, batch=96, cluster=cluster, tc=tc)
        assert ex.group == 32
        assert ex.info(0) == cluster and ex.info(2) == 3 * cluster and ex.info(1) >= 1
        ex.load_machines(0, progs)
        ex.reset()
        ex.set_tokens(0, [go] * 96)
        out = torch.zeros(400, 96, dtype=torch.int32, device="cuda")
        ex.run(400, out)
        heads = [s["S"] for s in ex.steps if s["kind"] == "head"]
        outs.append((out.cpu().numpy(), ex.checksums().cpu().numpy(),
                     [float(h.double().sum()) for h in heads], ex.x.cpu().numpy()))
        assert ex.errors() == 0
        del ex
    for o in outs[1:]:
        assert np.array_equal(o[0], outs[0][0])
        assert np.array_equal(o[1], outs[0][1])
        assert o[2] == outs[0][2]
        assert np.array_equal(o[3], outs[0][3])


@pytest.mark.parametrize("tc", [False, True])
def test_step_matches_stock_hf_modules(qx, graph, programs, tc):
    """Teacher-forced steps against the stock transformers Qwen3.5 modules running the emitted
    compiled stack (bf16 torch kernels, tests/golden/hf_residual.npz): every dim at every
    position, two programs as a batch of two."""
    from conftest import GOLDEN

    h = np.load(GOLDEN / "hf_residual.npz")
    names = [str(n) for n in h["names"]]
    ex = qx.Executor(None, batch=len(names), tc=tc)
    ex.load_machines(0, [programs[n]["prog"] for n in names])
    toks = np.stack([h[f"{n}.tokens"] for n in names], 1)
    for t in range(toks.shape[0]):
        x = torch.from_numpy(graph.embed([int(v) for v in toks[t]])).cuda()
        ex.step(x)
        got = x.cpu().numpy()
        for r, n in enumerate(names):
            bad = np.nonzero(got[r, 1:] != h[f"{n}.resid"][t])[0]
            assert not len(bad), (n, t, bad[:5])
    assert ex.errors() == 0


def test_free_run_in_chunks_equals_one_run(qx, programs):
    """Two launches of n/2 tokens generate what one launch of n does (x, lag history and head
    states carry over between launches)."""
    p = [programs["gen_base_2"]["prog"], programs["div_fuzz_1"]["prog"]]
    outs = []
    for chunks in ([800], [300, 500]):
        ex = qx.Executor(None, batch=2)
        ex.load_machines(0, p)
        ex.set_tokens(0, [int(programs["gen_base_2"]["trace"][0])] * 2)
        parts = []
        for c in chunks:
            o = torch.zeros(c, 2, dtype=torch.int32, device="cuda")
            ex.run(c, o)
            parts.append(o.cpu().numpy())
        outs.append(np.concatenate(parts))
    assert np.array_equal(outs[0], outs[1])


def _gdn_case(BH, seed, general=0.05):
    g = torch.Generator().manual_seed(seed)
    S = torch.randint(0, 2, (BH, 128, 128), generator=g).float()
    k = torch.zeros(BH, 128)
    k[torch.arange(BH), torch.randint(0, 128, (BH,), generator=g)] = 1.0
    gen = torch.rand(BH, generator=g) < general
    kg = torch.randn(int(gen.sum()), 128, generator=g)
    k[gen] = kg / kg.norm(dim=1, keepdim=True)
    q = torch.zeros(BH, 128)
    q[torch.arange(BH), torch.randint(0, 128, (BH,), generator=g)] = 1.0
    v = torch.randint(0, 2, (BH, 128), generator=g).float()
    u = torch.rand(BH, generator=g)
    alpha = torch.where(u < 0.9, 1.0, torch.where(u < 0.95, 0.5, 0.0))
    beta = torch.ones(BH)
    return S, q, k, v, alpha, beta


@pytest.mark.parametrize("BH,seed,general", [(512, 1, 0.05), (3000, 2, 0.05), (256, 3, 1.0), (777, 4, 0.0)])
def test_gdn_step_matches_oracle(qx, BH, seed, general):
    S, q, k, v, alpha, beta = _gdn_case(BH, seed, general)
    So = S.numpy().copy()
    o_want = oracle.gdn_step(So, q.numpy(), k.numpy(), v.numpy(), alpha.numpy(), beta.numpy())
    Sd = S.cuda()
    o = qx.gdn_step(Sd, q.cuda(), k.cuda(), v.cuda(), alpha.cuda(), beta.cuda())
    torch.cuda.synchronize()
    assert np.array_equal(Sd.cpu().numpy(), So)
    assert np.array_equal(o.cpu().numpy(), o_want)


def test_gdn_two_steps_and_beta(qx):
    """Two consecutive steps with beta in {0, 1/2, 1} and a second, denser write pattern."""
    S, q, k, v, alpha, beta = _gdn_case(1024, 9)
    beta = torch.tensor([0.0, 0.5, 1.0])[torch.randint(0, 3, (1024,), generator=torch.Generator().manual_seed(5))]
    So = S.numpy().copy()
    Sd = S.cuda()
    for step in range(2):
        ow = oracle.gdn_step(So, q.numpy(), k.numpy(), v.numpy(), alpha.numpy(), beta.numpy())
        od = qx.gdn_step(Sd, q.cuda(), k.cuda(), v.cuda(), alpha.cuda(), beta.cuda())
        torch.cuda.synchronize()
        assert np.array_equal(od.cpu().numpy(), ow), step
        assert np.array_equal(Sd.cpu().numpy(), So), step
        q = q.roll(1, 0)


GDN_GENERAL_ATOL = 1e-6  # against transformers' recurrence (its own summation order); see test_oracle


@pytest.mark.parametrize("case", ["gauss", "mix"])
def test_gdn_general_keys_match_transformers(qx, case):
    """The device step on unit-norm Gaussian keys (and the 1,024 x 48-head mix) equals the
    oracle bit for bit and transformers' torch_recurrent_gated_delta_rule within
    GDN_GENERAL_ATOL (tests/golden/gdn_general.npz)."""
    from conftest import GOLDEN

    z = np.load(GOLDEN / "gdn_general.npz")
    B, H, dk, dv = z[f"{case}.S"].shape
    BH = B * H
    S0 = np.ascontiguousarray(z[f"{case}.S"].reshape(BH, dk, dv).astype(np.float32))
    ins = [np.ascontiguousarray(z[f"{case}.{n}"].reshape(BH, -1)) for n in ("q", "k", "v")]
    al, be = z[f"{case}.alpha"].reshape(-1), z[f"{case}.beta"].reshape(-1)
    So = S0.copy()
    o_or = oracle.gdn_step(So, *ins, al, be)
    Sd = torch.from_numpy(S0).cuda()
    od = qx.gdn_step(Sd, *[torch.from_numpy(a).cuda() for a in ins], torch.from_numpy(al).cuda(),
                     torch.from_numpy(be).cuda())
    torch.cuda.synchronize()
    Sg, og = Sd.cpu().numpy(), od.cpu().numpy()
    assert np.array_equal(Sg, So) and np.array_equal(og, o_or)
    assert np.abs(Sg - z[f"{case}.S_out"].reshape(BH, dk, dv)).max() <= GDN_GENERAL_ATOL
    assert np.abs(og - z[f"{case}.o"].reshape(BH, dv)).max() <= GDN_GENERAL_ATOL


def test_gdn_full_size_step_matches_oracle(qx):
    """The measured step itself: 1,024 sequences x 48 heads (49,152 heads, 3.2 GB of state; 95%
    one-hot keys, 5% Gaussian, alpha 1 / 0.5 / 0 at 90 / 5 / 5%), the same draws as the bench;
    every state element and every read equal to the oracle's, compared in chunks of heads."""
    from qwenputer_b200 import workload

    inp = workload.gdn_inputs(1024, 48, seed=7)
    BH = inp["S"].shape[0]
    Sd = inp["S"].cuda().float()
    dev = {n: inp[n].cuda() for n in ("q", "k", "v", "alpha", "beta")}
    work = torch.zeros(int(qx.lib().qx_gdn_work_bytes(BH)), dtype=torch.uint8, device="cuda")
    od = qx.gdn_step(Sd, dev["q"], dev["k"], dev["v"], dev["alpha"], dev["beta"], None, work)
    torch.cuda.synchronize()
    assert qx.gdn_error(work) == 0
    n_full = int(((inp["alpha"] != 1.0) | inp["general"]).sum())
    assert n_full > 0.09 * BH  # the matrix path is exercised, not only the row path
    og = od.cpu().numpy()
    chunk = 4096
    for h0 in range(0, BH, chunk):
        h1 = min(BH, h0 + chunk)
        So = inp["S"][h0:h1].numpy().astype(np.float32)
        ow = oracle.gdn_step(So, *[np.ascontiguousarray(inp[n][h0:h1].numpy()) for n in ("q", "k", "v", "alpha", "beta")])
        assert np.array_equal(Sd[h0:h1].cpu().numpy(), So), h0
        assert np.array_equal(og[h0:h1], ow), h0


def test_gdn_step_on_two_devices_from_one_thread(qx):
    """The step's per-device set-up: the same host thread steps states on cuda:0, then cuda:1."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two CUDA devices")
    for d in (0, 1):
        S, q, k, v, alpha, beta = _gdn_case(512, 20 + d)
        So = S.numpy().copy()
        ow = oracle.gdn_step(So, q.numpy(), k.numpy(), v.numpy(), alpha.numpy(), beta.numpy())
        dev = torch.device("cuda", d)
        Sd = S.to(dev)
        od = qx.gdn_step(Sd, *[t.to(dev) for t in (q, k, v, alpha, beta)])
        torch.cuda.synchronize(dev)
        assert np.array_equal(Sd.cpu().numpy(), So) and np.array_equal(od.cpu().numpy(), ow), d


@pytest.mark.parametrize("cluster,tc", [(1, False), (4, False), (1, True)])
def test_step_in_cuda_graph(qx, graph, programs, cluster, tc):
    """Executor.step captured in a CUDA graph (as ExecRow captures Executor2.step) replays the
    same residuals and head states as eager steps."""
    names = ["gen_small_7", "div_fuzz_0", "mul_fuzz_1"]
    progs = [programs[n]["prog"] for n in names]
    traces = [programs[n]["trace"] for n in names]
    eager = qx.Executor(None, batch=3, cluster=cluster, tc=tc)
    capt = qx.Executor(None, batch=3, cluster=cluster, tc=tc)
    for ex in (eager, capt):
        ex.load_machines(0, progs)
    xbuf = torch.zeros(3, graph.D, device="cuda")
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        capt.step(xbuf.clone())  # warm-up outside the graph on the capture stream
    torch.cuda.current_stream().wait_stream(s)
    # the warm-up step moved capt one token ahead: restart both from the same state
    for ex in (eager, capt):
        ex.load_machines(0, progs)
        ex.reset()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        capt.step(xbuf)
    for t in range(20):
        toks = [int(tr[min(t, len(tr) - 1)]) for tr in traces]
        emb = torch.from_numpy(graph.embed(toks)).cuda()
        xe = emb.clone()
        eager.step(xe)
        xbuf.copy_(emb)
        g.replay()
        torch.cuda.synchronize()
        assert torch.equal(xe, xbuf), t
    for a, b in zip([s_["S"] for s_ in eager.steps if s_["kind"] == "head"],
                    [s_["S"] for s_ in capt.steps if s_["kind"] == "head"]):
        assert torch.equal(a, b)
    del g


def test_shared_table_images_match_private_copies(qx):
    """96 machines running 3 firmware images (each with its own RAM data): with the ROM / DROM
    tables shared in 3 image slots, free running generates the tokens, final states and
    checksums of an executor whose machines hold private copies; the shared sublayers hold 3
    copies; a 4th distinct image is refused."""
    import random

    from qwenputer_b200 import workload

    base = workload.workload_programs("base", 3, 4242)
    progs = []
    for i in range(96):
        rng = random.Random(i)
        p = base[i % 3]
        progs.append(workload.Program(p.text, bytes(rng.getrandbits(8) for _ in range(2048)), p.data_base,
                                      p.rodata, p.entry))
    go = int(oracle.lib().qxo_tok_family(18, 0))
    outs = []
    for shared in (0, 3):
        ex = qx.Executor(None, batch=96, table_images=shared or None)
        ex.load_machines(0, progs)
        ex.reset()
        ex.set_tokens(0, [go] * 96)
        out = torch.zeros(1500, 96, dtype=torch.int32, device="cuda")
        ex.run(1500, out)
        if shared:
            heads = [s_ for s_ in ex.steps if s_["kind"] == "head"]
            assert sum(h["shared"] for h in heads) == 3
            assert all(h["S"].shape[0] == 3 for h in heads if h["shared"])
            assert sorted(set(ex.table_image.cpu().tolist())) == [0, 1, 2]
            with pytest.raises(qx.QxError, match="table slots"):
                ex.load_machines(0, workload.workload_programs("base", 1, 999))
        outs.append((out.cpu().numpy(), ex.checksums().cpu().numpy(),
                     [list(ex.readback(r).x) for r in (0, 1, 2, 95)]))
        assert ex.errors() == 0
        del ex
    assert np.array_equal(outs[0][0], outs[1][0])
    assert np.array_equal(outs[0][1], outs[1][1])
    assert outs[0][2] == outs[1][2]


def test_fresh_executor_counters_are_zero(qx):
    """A new executor's device counters start at zero (the head-state byte counter included)."""
    ex = qx.Executor(None, batch=3)
    torch.cuda.synchronize()
    assert int(ex.state_bytes.cpu().numpy().view(np.uint64)[0]) == 0
    assert int(ex.count.cpu().sum()) == 0 and int(ex.err.cpu().numpy().sum()) == 0
