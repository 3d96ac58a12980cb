"""Generates the golden fixtures of tests/golden/ by running the reference itself.

Needs the reference tree importable (``ERV`` = ``experimental/riscv``), given as the argument
or as ``QX_REFERENCE_ROOT``::

    python tests/golden/make_golden.py /path/to/reference/experimental/riscv [--only gdn]

``--only gdn`` rewrites only the two gated delta-rule fixtures (they need transformers, not the
reference tree).

Writes:
  programs.npz   program images (our seeded generator, plus programs assembled by the
                 reference's own assembler from its test sources' shapes: faults, DIV / MUL edge
                 fuzz, Zba + DROM loads, CSR stubs, the digit file), each with the reference
                 trace (``ref.Machine.run``) and final machine state
  romword.npz    ``ref.rom_word`` of every text word above plus random words
  divrec.npz     ``ref.div_record`` on random and edge operands (ERV/tests/test_rv_ref.py:97-110)
  residual.npz   ``ir.evaluate`` (fp64, exact) on teacher-forced prefixes: per position an FNV-1a
                 hash of the float32 residual, the full residual of the first positions, and
                 ``core.predictions``
  snapshot.npz   per program, an FNV-1a hash of every head sublayer's state after
                 ``core.snapshot`` + ``Executor2.load_init`` (tritonexec.py:246-258)
  gdn.npz        transformers' ``torch_recurrent_gated_delta_rule`` on one-hot keys / queries
                 (the query pre-multiplied by sqrt(dk) to undo its scale)
  gdn_general.npz  the same function on unit-norm Gaussian keys (every head), and on a mix drawn
                 like the 1,024 x 48-head step (95% one-hot keys, alpha 90 / 5 / 5% at 1 / 0.5 /
                 0); one-hot queries
  merged.npz     the machine with the text bridge (``core.build(text=ByteVocab())``, the graph
                 file ``rv32im_merged_graph.npz``): firmware assembled by the reference's assembler,
                 parked (``bridge.park``), then driven by ``bridge.Session`` (text, a tool call,
                 the run with its echoes); per session the parked state, the token stream, who
                 owns each position, and ``ir.evaluate`` residual hashes and ``core.predictions``
                 (``--only merged`` rewrites only this file and calc.npz)
  calc.npz       the calculator firmware (qwenputer_b200/calc.py) in bridge sessions on the merged
                 machine: tool calls A*B, the reference evaluator's residual hashes and the owned
                 tokens (checked against A*B)
  hf_residual.npz  the compiled stack emitted as stock transformers Qwen3_5ForCausalLM weights
                 (the reference's ``hf.build_model``, bf16, torch kernels), the snapshot injected
                 into its cache, decoded token by token: the residual of every IR dim after the
                 last compiled layer at every position (ERV/chipformer/rv/hf.py:74-112), for
                 programs of programs.npz (``--only hf`` rewrites only this file)
"""

import argparse
import os

import random
import sys
import time
from pathlib import Path
from types import SimpleNamespace

sys.dont_write_bytecode = True
HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]


def fnv1a_bytes(b: bytes) -> int:
    h = 0xcbf29ce484222325
    for x in b:
        h ^= x
        h = (h * 0x100000001b3) & 0xFFFFFFFFFFFFFFFF
    return h


def main(ref_root: str) -> None:
    sys.path.insert(0, ref_root)
    sys.path.insert(0, str(REPO))
    import numpy as np

    from chipformer.q35 import ir
    from chipformer.rv import core, ref
    from chipformer.rv import spec as S
    from chipformer.rv.asm import assemble

    from qwenputer_b200 import workload

    t0 = time.time()
    c = core.build()
    print(f"graph built {time.time() - t0:.1f} s", flush=True)

    # ---------------- programs -----------------------------------------------------------
    progs = {}  # name -> Program-like
    for s in range(3):
        progs[f"gen_base_{s}"] = workload.gen_program(s)
    progs["gen_small_7"] = workload.gen_program(7, n_instr=48, iters=3)
    progs["gen_many_11"] = workload.workload_programs("many", 1, 11)[0]
    progs["gen_bignum_5"] = workload.workload_programs("bignum", 1, 5)[0]
    EXIT = "\nli a7, 93\necall"
    srcs = {
        "fault_illegal": "_start: li a0, 7\n.word 0x0000000b",
        "fault_csr_write": "_start: li a0, 1\ncsrw mscratch, a0",
        "fault_ebreak": "_start: nop\nebreak",
        "fault_mis_load": "_start: li a0, 0x102\nlw a1, 0(a0)",
        "fault_mis_store": "_start: li a0, 0x101\nsh a0, 0(a0)",
        "fault_load_range": "_start: li a0, 0x8000\nlw a1, 0(a0)",
        "fault_store_range": "_start: li a0, -4\nsb a0, 0(a0)",
        "fault_bad_jump": "_start: li a0, 0x4000\njr a0",
        "fault_ecall": "_start: li a7, 5\necall",
        "refresh_70": "_start: " + "\n".join(f"addi a0, a0, {i % 7}" for i in range(70)) + EXIT,
        "csr_putchar": """_start: csrr a0, mhartid
            csrr a1, misa
            csrr a2, cycle
            li a7, 1
            li a0, 72
            ecall
            li a0, 105
            ecall""" + EXIT,
        "zba_rodata": """_start: li a0, 0x1234567
            li a1, -77
            sh1add a2, a0, a1
            sh2add a3, a1, a0
            sh3add a4, a0, a0
            la s0, tab
            lw t0, 0(s0)
            lw t1, 4(s0)
            lb t2, 5(s0)
            lbu t3, 7(s0)
            lh t4, 6(s0)
            lhu t5, 2(s0)""" + EXIT + """
            .rodata
            tab: .word 0x89abcdef, 0x80ff7f01""",
        "digit_file": """_start: la a0, txt
            bscan a1, a0
            add a2, a0, a1
            slli t2, a1, 7
            ori t0, t2, 1
            bld zero, a2, t0
            li a2, 1048986
            bmac a3, zero, a2
            bmac a3, zero, a2
            li t0, 7341739
            bmac a4, zero, t0
            li t0, 3163802
            bmsb a6, zero, t0
            bprd 2, 7
            bprd 2, 5
            li t1, 24579
            bget a5, zero, t1""" + EXIT + """
            .data
            txt: .byte 0x31, 0x32, 0x33, 0x34, 0x39, 0x2b, 0x37, 0x41""",
    }
    rng = random.Random(200)
    edge = [0, 1, -1, 2, -2, 7, -7, 15, 16, 255, 256, 1000, 2**31 - 1, -2**31, -2**31 + 1,
            0xFFFF, -0x10000, 10, 3]
    regs = ["a0", "a1", "a2", "a3", "t0", "t1", "s1"]

    def dval():
        return rng.choice([rng.choice(edge), rng.randint(-2**31, 2**31 - 1),
                           rng.randint(-2**(rng.randint(1, 31)), 2**rng.randint(1, 31))])

    for seed in range(2):
        lines = [f"li {r}, {dval()}" for r in regs]
        for i in range(36):
            if i % 6 == 5:
                lines += [f"li {r}, {dval()}" for r in rng.sample(regs, 3)]
            op = rng.choice(["div", "divu", "rem", "remu"])
            d = "zero" if rng.random() < 0.1 else rng.choice(regs)
            lines.append(f"{op} {d}, {rng.choice(regs)}, {rng.choice(regs)}")
        srcs[f"div_fuzz_{seed}"] = "_start: " + "\n".join(lines) + EXIT
        lines = [f"li {r}, {rng.choice([rng.randint(-2**31, 2**31 - 1), rng.randint(-9, 9)])}"
                 for r in regs[:6]]
        for _ in range(60):
            op = rng.choice(["mul", "mulh", "mulhsu", "mulhu", "add", "xor"])
            lines.append(f"{op} {rng.choice(regs[:6])}, {rng.choice(regs[:6])}, "
                         f"{rng.choice(regs[:6])}")
        srcs[f"mul_fuzz_{seed}"] = "_start: " + "\n".join(lines) + EXIT
    for name, src in srcs.items():
        progs[name] = assemble(src)
    for name, p in list(progs.items()):  # plain ints for the reference machine
        progs[name] = SimpleNamespace(text=[int(w) for w in p.text], data=bytes(p.data),
                                      data_base=int(p.data_base), entry=int(p.entry),
                                      rodata=bytes(getattr(p, "rodata", b"")))

    out = {}
    names = sorted(progs)
    out["names"] = np.asarray(names)
    max_tok = 60000
    for name in names:
        p = progs[name]
        m = ref.Machine.from_program(p)
        toks = m.run(max_tok)
        out[f"{name}.text"] = np.asarray(list(p.text), np.uint32)
        out[f"{name}.data"] = np.frombuffer(bytes(p.data), np.uint8)
        out[f"{name}.data_base"] = np.int64(p.data_base)
        out[f"{name}.rodata"] = np.frombuffer(bytes(getattr(p, "rodata", b"")), np.uint8)
        out[f"{name}.entry"] = np.int64(p.entry)
        out[f"{name}.trace"] = np.asarray(toks, np.int32)
        out[f"{name}.x"] = np.asarray(m.x, np.uint32)
        out[f"{name}.anchor_n"] = np.asarray([m.anchor, m.n], np.uint32)
        out[f"{name}.ram"] = np.asarray(m.ram, np.uint32)
        out[f"{name}.halted"] = np.int64(m.halted)
        print(f"  {name}: {len(toks)} tokens, halted={m.halted}", flush=True)
    np.savez_compressed(HERE / "programs.npz", **out)

    # ---------------- rom words ----------------------------------------------------------
    words, pcs = [], []
    for name in names:
        for i, w in enumerate(progs[name].text):
            words.append(int(w))
            pcs.append(S.ROM_BASE + 4 * i)
    r2 = random.Random(5)
    for _ in range(20000):
        words.append(r2.getrandbits(32))
        pcs.append(S.ROM_BASE + 4 * r2.randrange(S.ROM_WORDS + 64))
    rw = [ref.rom_word(w, pc) for w, pc in zip(words, pcs)]
    np.savez_compressed(HERE / "romword.npz", w=np.asarray(words, np.uint32),
                        pc=np.asarray(pcs, np.uint32), rom=np.asarray(rw, np.uint32))

    # ---------------- DIV records --------------------------------------------------------
    r3 = random.Random(1)
    M = 0xFFFFFFFF
    edge2 = [0, 1, 2, 7, 15, 16, 255, 256, 0x7FFFFFFF, 0x80000000, 0x80000001, M, M - 1, 10, 1000]
    vals = edge2 + [r3.getrandbits(r3.choice([4, 8, 16, 24, 32])) for _ in range(500)]
    ops, A, B, recs, lens = [], [], [], [], []
    for oi, op in enumerate(("DIV", "DIVU", "REM", "REMU")):
        for _ in range(1000):
            a, b = r3.choice(vals), r3.choice(vals)
            rec = ref.div_record(op, a, b)
            ops.append(oi)
            A.append(a)
            B.append(b)
            lens.append(len(rec))
            recs.append(rec + [0] * (16 - len(rec)))
    np.savez_compressed(HERE / "divrec.npz", op=np.asarray(ops, np.int32),
                        a=np.asarray(A, np.uint32), b=np.asarray(B, np.uint32),
                        rec=np.asarray(recs, np.int32), len=np.asarray(lens, np.int32))

    # ---------------- ir.evaluate residuals + snapshots ----------------------------------
    from qwenputer_b200.graphfile import export_graph
    g = export_graph(c)
    head_levels = g.head_sublayers()
    res, snap = {}, {}
    res_cases = {"gen_base_0": 600, "gen_small_7": 400, "div_fuzz_0": 400, "mul_fuzz_0": 300,
                 "zba_rodata": 200, "digit_file": 300, "fault_bad_jump": 100,
                 "refresh_70": 200, "gen_bignum_5": 400, "csr_putchar": 100}
    for name in names:
        p = progs[name]
        core.snapshot(c, ref.Machine.from_program(p))
        # Executor2.load_init's buffers (tritonexec.py:246-258)
        hs = []
        for lv in head_levels:
            heads = [n for n in c.nodes if n.level == lv and isinstance(n, ir.Head)]
            V = sum(len(n.vheads()) for n in heads)
            buf = np.zeros((V, 128, 128), np.float32)
            j = 0
            for n in heads:
                init = n.init or []
                for x in range(len(n.vheads())):
                    for r, vec in (init[x] if x < len(init) else {}).items():
                        buf[j, r] = vec
                    j += 1
            hs.append(fnv1a_bytes(buf.tobytes()))
        snap[name] = np.asarray(hs, np.uint64)
        if name in res_cases:
            toks = ref.Machine.from_program(p).run(res_cases[name] + 1)[:res_cases[name]]
            t1 = time.time()
            mat = ir.evaluate(c, toks, check=False)
            pred = core.predictions(c, mat)
            m32 = mat.astype(np.float32)
            assert np.all(m32.astype(np.float64) == mat), "residual not exact in float32"
            res[f"{name}.tokens"] = np.asarray(toks, np.int32)
            res[f"{name}.hash"] = np.asarray([fnv1a_bytes(r.tobytes()) for r in m32], np.uint64)
            res[f"{name}.head"] = m32[:8]
            res[f"{name}.pred"] = np.asarray(pred, np.int64)
            print(f"  ir.evaluate {name}: {len(toks)} tokens {time.time() - t1:.1f} s", flush=True)
    np.savez_compressed(HERE / "residual.npz", names=np.asarray(sorted(res_cases)), **res)
    np.savez_compressed(HERE / "snapshot.npz", names=np.asarray(names),
                        **{k: v for k, v in snap.items()})

    gdn_goldens()
    print(f"done in {time.time() - t0:.1f} s")


def _gdn_ref(S, q, k, v, al, be):
    """transformers' recurrence for one step; the query pre-multiplied by sqrt(dk) undoes its
    scale (exactly for one-hot queries up to the last bit)."""
    import torch
    from transformers.models.qwen3_5.modeling_qwen3_5 import torch_recurrent_gated_delta_rule

    dk = S.shape[-1]
    return torch_recurrent_gated_delta_rule(
        (q * dk ** 0.5)[:, None], k[:, None], v[:, None], torch.log(al)[:, None], be[:, None],
        S.clone(), True)


def gdn_goldens() -> None:
    import numpy as np
    import torch

    # one-hot keys and queries
    gen = torch.Generator().manual_seed(1234)
    Bn, H, dk = 3, 4, 128
    Sg = torch.randint(0, 2, (Bn, H, dk, dk), generator=gen).float()
    kk = torch.zeros(Bn, H, dk)
    qq = torch.zeros(Bn, H, dk)
    kr = torch.randint(0, dk, (Bn, H), generator=gen)
    qr = torch.randint(0, dk, (Bn, H), generator=gen)
    for b in range(Bn):
        for h in range(H):
            kk[b, h, kr[b, h]] = 1.0
            qq[b, h, qr[b, h]] = 1.0
    vv = torch.randint(0, 2, (Bn, H, dk), generator=gen).float()
    al = torch.tensor([1.0, 0.5, 0.0, 1.0])[torch.randint(0, 4, (Bn, H), generator=gen)]
    be = torch.ones(Bn, H)
    o, Sf = _gdn_ref(Sg, qq, kk, vv, al, be)
    np.savez_compressed(HERE / "gdn.npz", S=Sg.numpy(), q=qq.numpy(), k=kk.numpy(),
                        v=vv.numpy(), alpha=al.numpy(), beta=be.numpy(),
                        o=o[:, 0].numpy(), S_out=Sf.numpy())

    # general keys: unit-norm Gaussian on every head ("gauss"), and the 1,024 x 48-head step's
    # mix on 4 x 48 heads ("mix"); beta in {1, 1/2} on the Gaussian case; initial states {0, 1}
    # are stored as uint8
    out = {}
    gen = torch.Generator().manual_seed(4321)
    for case, (Bn, H) in (("gauss", (2, 4)), ("mix", (4, 48))):
        S0 = torch.randint(0, 2, (Bn, H, dk, dk), generator=gen).float()
        q = torch.zeros(Bn, H, dk)
        q[torch.arange(Bn)[:, None], torch.arange(H)[None], torch.randint(0, dk, (Bn, H), generator=gen)] = 1.0
        v = torch.randint(0, 2, (Bn, H, dk), generator=gen).float()
        if case == "gauss":
            k = torch.randn(Bn, H, dk, generator=gen)
            k = k / k.norm(dim=-1, keepdim=True)
            al = torch.tensor([1.0, 0.5, 0.0, 1.0])[torch.randint(0, 4, (Bn, H), generator=gen)]
            be = torch.tensor([1.0, 0.5])[torch.randint(0, 2, (Bn, H), generator=gen)]
        else:
            k = torch.zeros(Bn, H, dk)
            k[torch.arange(Bn)[:, None], torch.arange(H)[None], torch.randint(0, dk, (Bn, H), generator=gen)] = 1.0
            g = torch.rand(Bn, H, generator=gen) < 0.05
            kg = torch.randn(int(g.sum()), dk, generator=gen)
            k[g] = kg / kg.norm(dim=1, keepdim=True)
            u = torch.rand(Bn, H, generator=gen)
            al = torch.where(u < 0.9, 1.0, torch.where(u < 0.95, 0.5, 0.0))
            be = torch.ones(Bn, H)
        o, Sf = _gdn_ref(S0, q, k, v, al, be)
        out.update({f"{case}.S": S0.numpy().astype(np.uint8), f"{case}.q": q.numpy(), f"{case}.k": k.numpy(),
                    f"{case}.v": v.numpy(), f"{case}.alpha": al.numpy(), f"{case}.beta": be.numpy(),
                    f"{case}.o": o[:, 0].numpy(), f"{case}.S_out": Sf.numpy()})
    np.savez_compressed(HERE / "gdn_general.npz", **out)


HF_CASES = {"div_fuzz_0": 40, "gen_small_7": 40}


def hf_goldens(ref_root: str) -> None:
    """Residuals of the stock HF modules (bf16) running the emitted compiled stack, decoded
    token by token from the snapshot of each HF_CASES program (its first n trace tokens)."""
    sys.path.insert(0, ref_root)
    sys.path.insert(0, str(REPO))
    import numpy as np
    import torch
    from chipformer.rv import core, hf, ref

    t0 = time.time()
    c = core.build()
    z = np.load(HERE / "programs.npz")
    out = {"names": np.asarray(sorted(HF_CASES))}
    for name, n in sorted(HF_CASES.items()):
        p = SimpleNamespace(text=[int(w) for w in z[f"{name}.text"]], data=z[f"{name}.data"].tobytes(),
                            data_base=int(z[f"{name}.data_base"]), entry=int(z[f"{name}.entry"]),
                            rodata=z[f"{name}.rodata"].tobytes())
        core.snapshot(c, ref.Machine.from_program(p))
        toks = [int(t) for t in ref.Machine.from_program(p).run(n + 1)[:n]]
        model, lay, ids = hf.build_model(c, toks)
        print(f"  hf model for {name}: hidden {lay.hidden}, {time.time() - t0:.0f} s", flush=True)
        dims = list(range(1, len(c.dims)))
        cols = [lay.dim(d) for d in dims]
        r = c.target.value_heads // c.target.key_heads
        with torch.no_grad():
            o = model(input_ids=torch.tensor([[ids[None]]]), use_cache=True)  # the zero prefix
            cache = o.past_key_values
            # the snapshot into the linear-attention states (hf.inject's layout; this
            # transformers keeps a layer's recurrent state as one [B, H, dk, dv] tensor)
            for ni, (L, j) in hf.head_slots(c).items():
                st = cache.layers[L].recurrent_states
                init = c.nodes[ni].init or []
                for x in range(len(c.nodes[ni].vheads())):
                    S = st[0, j * r + x]
                    S.zero_()
                    for row, vec in (init[x] if x < len(init) else {}).items():
                        S[row] = torch.tensor(vec, dtype=S.dtype)
            hs = []
            for t in range(n):
                o = model(input_ids=torch.tensor([[ids[toks[t]]]]), past_key_values=cache, use_cache=True,
                          output_hidden_states=True)
                hs.append(o.hidden_states[c.n_layers()][0])
        h = torch.cat(hs).float().numpy()[:, cols]
        out[f"{name}.tokens"] = np.asarray(toks, np.int32)
        out[f"{name}.resid"] = np.ascontiguousarray(h, np.float32)  # [n, D - 1]: dims 1 .. D - 1
        print(f"  hf decode {name}: {n} positions, {time.time() - t0:.0f} s", flush=True)
    np.savez_compressed(HERE / "hf_residual.npz", **out)


# firmware for the bridge sessions: park at once; each run (GO) prints the first byte of every
# captured text row (TEXT_ADDR + 16 i, i = 1, 2, ..), then a special token (putchar(256 + k)),
# then parks again (exit ecall) and loops
ECHO_FIRMWARE = """_start:
      li a7, 93
      ecall
loop: li t0, 0x8010
next: lbu a0, 0(t0)
      beq a0, zero, done
      li a7, 1
      ecall
      addi t0, t0, 16
      j next
done: li a0, 257
      li a7, 1
      ecall
      li a7, 93
      ecall
      j loop"""


def merged_goldens(ref_root: str) -> None:
    sys.path.insert(0, ref_root)
    sys.path.insert(0, str(REPO))
    import numpy as np
    from chipformer.q35 import ir
    from chipformer.rv import bridge, core, ref
    from chipformer.rv.asm import assemble

    from qwenputer_b200.plans.export_rv32im import ByteVocab

    T = ByteVocab()
    c = core.build(text=T)
    p = assemble(ECHO_FIRMWARE)
    prog = SimpleNamespace(text=[int(w) for w in p.text], data=bytes(p.data), data_base=int(p.data_base),
                           entry=int(p.entry), rodata=bytes(getattr(p, "rodata", b"")))
    enc = lambda b: [int(x) for x in b]  # bytes -> the byte tokens of ByteVocab
    from qwenputer_b200.plans.export_rv32im import CALL_TOKENS, SPECIAL_TOKENS

    w0 = 256 + len(SPECIAL_TOKENS) + len(CALL_TOKENS)  # the first seeded multi-byte token
    sessions = {
        "echo_short": [enc(b"hi "), [T.TCO] + enc(b"7*6") + [T.TCC]],
        "echo_words": [enc(b"calc: ") + [w0 + 5, w0 + 17], [T.TCO] + enc(b"\n12345678*987654321\n") + [T.TCC]],
    }
    out = {"names": np.asarray(sorted(sessions)), "text": np.asarray(prog.text, np.uint32),
           "data": np.frombuffer(prog.data, np.uint8), "data_base": np.int64(prog.data_base),
           "entry": np.int64(prog.entry)}
    for name, parts in sorted(sessions.items()):
        m = ref.Machine.from_program(prog)
        bridge.park(m)
        core.snapshot(c, m)
        out[f"{name}.x"] = np.asarray(m.x, np.uint32)
        out[f"{name}.anchor_n"] = np.asarray([m.anchor, m.n], np.uint32)
        out[f"{name}.ram"] = np.asarray(m.ram, np.uint32)
        s_ = bridge.Session(T, m)
        for q in parts:
            s_.qwen(q)
        toks = s_.toks
        t0 = time.time()
        mat = ir.evaluate(c, toks, check=False)
        pred = core.predictions(c, mat)
        m32 = mat.astype(np.float32)
        assert np.all(m32.astype(np.float64) == mat), "residual not exact in float32"
        own = s_.own
        assert all(pred[i] == toks[i + 1] for i in range(len(toks) - 1) if own[i])
        out[f"{name}.tokens"] = np.asarray(toks, np.int64)
        out[f"{name}.own"] = np.asarray(own, bool)
        out[f"{name}.hash"] = np.asarray([fnv1a_bytes(r.tobytes()) for r in m32], np.uint64)
        out[f"{name}.head"] = m32[:4]
        out[f"{name}.pred"] = np.asarray(pred, np.int64)
        print(f"  merged session {name}: {len(toks)} tokens, {sum(own)} owned, {time.time() - t0:.1f} s", flush=True)
    np.savez_compressed(HERE / "merged.npz", **out)
    calc_goldens(c, T)


# two 18-digit operands each, so that every session reaches its </tool_call> at the same position
CALC_CASES = [(123456789012345678, 987654321098765432), (999999999999999999, 888888888888888888)]


def calc_tool_call(T, a: int, b: int) -> list[int]:
    """Qwen's tool-call syntax naming calc with the expression A*B, in ByteVocab tokens."""
    ids = T.ids
    return ([T.TCO, 10, ids["<function="], ids["calc>"], 10, ids["<parameter="], ids["expression>"], 10]
            + list(str(a).encode()) + [ord("*")] + list(str(b).encode())
            + [10, ids["</parameter>"], 10, ids["</function>"], 10, T.TCC])


def calc_goldens(c, T) -> None:
    """calc.npz: the calculator firmware (qwenputer_b200/calc.py) on the merged machine, parked,
    then a bridge session per CALC_CASES (a little text, the tool call, the run); the token
    stream, who owns each position, ir.evaluate residual hashes, and the firmware's printed
    bytes checked against A*B."""
    import numpy as np
    from chipformer.q35 import ir
    from chipformer.rv import bridge, core, ref

    from qwenputer_b200.calc import calc_program, expected_response

    p = calc_program()
    prog = SimpleNamespace(text=[int(w) for w in p.text], data=b"", data_base=int(p.data_base),
                           entry=int(p.entry), rodata=b"")
    out = {"names": np.asarray([f"calc{i}" for i in range(len(CALC_CASES))]),
           "text": np.asarray(prog.text, np.uint32)}
    for i, (a, b) in enumerate(CALC_CASES):
        name = f"calc{i}"
        m = ref.Machine.from_program(prog)
        bridge.park(m)
        core.snapshot(c, m)
        out[f"{name}.x"] = np.asarray(m.x, np.uint32)
        out[f"{name}.anchor_n"] = np.asarray([m.anchor, m.n], np.uint32)
        out[f"{name}.ram"] = np.asarray(m.ram, np.uint32)
        s_ = bridge.Session(T, m)
        s_.qwen(list(b"result: "))
        s_.qwen(calc_tool_call(T, a, b))
        assert b"".join(T.bytes[q] for q in s_.runs[-1][:-1]) == expected_response(a, b)
        toks, own = s_.toks, s_.own
        t0 = time.time()
        mat = ir.evaluate(c, toks, check=False)
        pred = core.predictions(c, mat)
        assert all(pred[j] == toks[j + 1] for j in range(len(toks) - 1) if own[j])
        m32 = mat.astype(np.float32)
        assert np.all(m32.astype(np.float64) == mat)
        out[f"{name}.a_b"] = np.asarray([a, b], np.uint64)
        out[f"{name}.tokens"] = np.asarray(toks, np.int64)
        out[f"{name}.own"] = np.asarray(own, bool)
        out[f"{name}.hash"] = np.asarray([fnv1a_bytes(r.tobytes()) for r in m32], np.uint64)
        print(f"  calc session {name}: {len(toks)} tokens, {sum(own)} owned, {time.time() - t0:.1f} s", flush=True)
    np.savez_compressed(HERE / "calc.npz", **out)


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("ref_root", nargs="?", default=os.environ.get("QX_REFERENCE_ROOT"),
                    help="the reference's experimental/riscv directory (or QX_REFERENCE_ROOT)")
    ap.add_argument("--only", choices=["gdn", "hf", "merged"], default=None)
    a = ap.parse_args()
    if a.only == "gdn":
        gdn_goldens()
    elif a.only in ("hf", "merged"):
        if not a.ref_root:
            ap.error("give the reference's experimental/riscv directory or set QX_REFERENCE_ROOT")
        (hf_goldens if a.only == "hf" else merged_goldens)(a.ref_root)
    else:
        if not a.ref_root:
            ap.error("give the reference's experimental/riscv directory or set QX_REFERENCE_ROOT")
        main(a.ref_root)
