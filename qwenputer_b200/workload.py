"""Seeded synthetic RV32IM programs for the executor's workloads.

Modelled on the reference's fuzz generator (``ERV/chipformer/rv/fuzz.py:31-75``): a counted outer
loop over a block of random instructions on random registers, with loads and stores through
masked, word-aligned addresses into a data image, forward branches, forward jumps and calls to a
leaf function.  Unlike the reference it emits machine code directly (the standard RV32 encodings),
so no assembler is needed where the workload is built.

Reserved registers (never random operands): x0; ra (x1, the call link); s0 (x8, the loop
counter); a7 (x17, the ecall number at exit); s11 (x27, the data base); t5 (x30, the address
temporary).  Every other register is an operand.

Workloads:
  * ``base``   512 instructions from ADD / SUB / MUL / DIV / REM / SH1ADD / LW / SW / BEQ / BNE /
               JAL, a 4 KB data image of uniform random bytes at RAM 0x100, 50 loop iterations.
  * ``bignum`` 40% MUL / MULH / DIVU chains on random 32-bit operands, 20% LW / SW over a 16 KB
               range, the rest as ``base``.
"""

from __future__ import annotations

import dataclasses
import random

import numpy as np

ROM_BASE = 0x40000
DATA_BASE = 0x100
RAM_BYTES = 1 << 15

X0, RA, S0, A0, A7, S11, T5 = 0, 1, 8, 10, 17, 27, 30
RESERVED = {X0, RA, S0, A7, S11, T5}
OPERANDS = [r for r in range(32) if r not in RESERVED]


def _r(f7, rs2, rs1, f3, rd, opc):
    return (f7 << 25 | rs2 << 20 | rs1 << 15 | f3 << 12 | rd << 7 | opc) & 0xFFFFFFFF


def _i(imm, rs1, f3, rd, opc):
    assert -2048 <= imm < 2048
    return ((imm & 0xFFF) << 20 | rs1 << 15 | f3 << 12 | rd << 7 | opc) & 0xFFFFFFFF


def _s(imm, rs2, rs1, f3, opc=0x23):
    assert -2048 <= imm < 2048
    i = imm & 0xFFF
    return (i >> 5 << 25 | rs2 << 20 | rs1 << 15 | f3 << 12 | (i & 31) << 7 | opc) & 0xFFFFFFFF


def _b(off, rs2, rs1, f3):
    assert off % 2 == 0 and -4096 <= off < 4096
    o = off & 0x1FFF
    return ((o >> 12 & 1) << 31 | (o >> 5 & 63) << 25 | rs2 << 20 | rs1 << 15 | f3 << 12
            | (o >> 1 & 15) << 8 | (o >> 11 & 1) << 7 | 0x63) & 0xFFFFFFFF


def _j(off, rd):
    assert off % 2 == 0 and -(1 << 20) <= off < (1 << 20)
    o = off & 0x1FFFFF
    return ((o >> 20 & 1) << 31 | (o >> 1 & 0x3FF) << 21 | (o >> 11 & 1) << 20
            | (o >> 12 & 0xFF) << 12 | rd << 7 | 0x6F) & 0xFFFFFFFF


def _u(imm20, rd, opc=0x37):
    return ((imm20 & 0xFFFFF) << 12 | rd << 7 | opc) & 0xFFFFFFFF


R_OPS = {  # name -> (funct7, funct3)
    "add": (0x00, 0), "sub": (0x20, 0), "mul": (0x01, 0), "mulh": (0x01, 1),
    "mulhsu": (0x01, 2), "mulhu": (0x01, 3), "div": (0x01, 4), "divu": (0x01, 5),
    "rem": (0x01, 6), "remu": (0x01, 7), "sh1add": (0x10, 2), "sh2add": (0x10, 4),
    "sh3add": (0x10, 6), "xor": (0x00, 4), "and": (0x00, 7), "or": (0x00, 6),
}


def r_type(op, rd, rs1, rs2):
    f7, f3 = R_OPS[op]
    return _r(f7, rs2, rs1, f3, rd, 0x33)


def addi(rd, rs1, imm):
    return _i(imm, rs1, 0, rd, 0x13)


def slli(rd, rs1, sh):
    return _i(sh, rs1, 1, rd, 0x13)


def srli(rd, rs1, sh):
    return _i(sh, rs1, 5, rd, 0x13)


def lw(rd, rs1, imm=0):
    return _i(imm, rs1, 2, rd, 0x03)


def sw(rs2, rs1, imm=0):
    return _s(imm, rs2, rs1, 2)


def beq(rs1, rs2, off):
    return _b(off, rs2, rs1, 0)


def bne(rs1, rs2, off):
    return _b(off, rs2, rs1, 1)


def jal(rd, off):
    return _j(off, rd)


def jalr(rd, rs1, imm=0):
    return _i(imm, rs1, 0, rd, 0x67)


def ecall():
    return 0x00000073


def li(rd, v) -> list[int]:
    """LUI + ADDI (or ADDI alone) loading a 32-bit constant."""
    v &= 0xFFFFFFFF
    sv = v - (1 << 32) if v >> 31 else v
    if -2048 <= sv < 2048:
        return [addi(rd, X0, sv)]
    lo = v & 0xFFF
    lo = lo - 4096 if lo >= 2048 else lo
    hi = ((v - lo) >> 12) & 0xFFFFF
    out = [_u(hi, rd)]
    if lo:
        out.append(addi(rd, rd, lo))
    return out


@dataclasses.dataclass
class Program:
    """An RV32 program image: text words from ROM_BASE, data bytes from data_base."""

    text: np.ndarray  # uint32
    data: bytes
    data_base: int = DATA_BASE
    rodata: bytes = b""
    entry: int = ROM_BASE


def _addr(rng: random.Random, rs: int, span_bits: int) -> list[int]:
    """t5 = s11 + (rs mod 2^span_bits, word aligned)."""
    return [slli(T5, rs, 32 - span_bits), srli(T5, T5, 32 - span_bits + 2), slli(T5, T5, 2),
            r_type("add", T5, T5, S11)]


def gen_program(seed: int, n_instr: int = 512, iters: int = 50, data_bytes: int = 4096,
                mix: str = "base", span_bits: int | None = None) -> Program:
    """A seeded, fault-free program (see the module doc)."""
    rng = random.Random(seed)
    span_bits = span_bits or (14 if mix == "bignum" else int(data_bytes - 1).bit_length())
    span_bits = max(span_bits, 3)
    data = bytes(rng.getrandbits(8) for _ in range(max(data_bytes, 1 << span_bits)))
    text: list[int] = []
    pend: list[tuple[int, str]] = []  # (index, label) of calls to patch

    def emit(ws):
        text.extend(ws if isinstance(ws, list) else [ws])

    def val():
        return rng.choice([rng.getrandbits(32), rng.randint(-40, 40), rng.randint(0, 0x3FF)])

    emit(li(S11, DATA_BASE))
    emit(li(S0, iters))
    for r in OPERANDS:
        emit(li(r, val()))
    loop = len(text)
    body = 0
    while body < n_instr:
        k = rng.random()
        d, a, b = rng.choice(OPERANDS), rng.choice(OPERANDS), rng.choice(OPERANDS)
        if mix == "bignum" and k < 0.40:
            # a short chain of wide multiplies / unsigned divides on random 32-bit operands
            emit(li(a, rng.getrandbits(32)))
            emit(r_type(rng.choice(["mul", "mulh", "mulhu"]), d, a, b))
            emit(r_type(rng.choice(["mul", "mulh", "divu"]), b, d, a))
            body += 3
            continue
        if mix == "bignum":
            k = (k - 0.40) / 0.60
            if k < 0.20 / 0.60:
                if rng.random() < 0.5:
                    emit(_addr(rng, a, span_bits) + [lw(d, T5)])
                else:
                    emit(_addr(rng, a, span_bits) + [sw(b, T5)])
                body += 1
                continue
            k = rng.random()
        if k < 0.45:
            emit(r_type(rng.choice(["add", "sub", "mul", "div", "rem", "sh1add"]), d, a, b))
            body += 1
        elif k < 0.60:
            emit(_addr(rng, a, span_bits) + [lw(d, T5)])
            body += 1
        elif k < 0.72:
            emit(_addr(rng, a, span_bits) + [sw(b, T5)])
            body += 1
        elif k < 0.88:
            n_skip = rng.randint(1, 3)
            br = beq if rng.random() < 0.5 else bne
            emit(br(a, b, 4 * (n_skip + 1)))
            for _ in range(n_skip):
                emit(r_type(rng.choice(["add", "sub", "sh1add"]), rng.choice(OPERANDS),
                            rng.choice(OPERANDS), rng.choice(OPERANDS)))
            body += 1 + n_skip
        elif k < 0.94:
            pend.append((len(text), "leaf"))
            emit(jal(RA, 0))  # patched below
            body += 1
        else:
            n_skip = rng.randint(1, 2)
            emit(jal(X0, 4 * (n_skip + 1)))
            for _ in range(n_skip):
                emit(r_type("add", rng.choice(OPERANDS), rng.choice(OPERANDS),
                            rng.choice(OPERANDS)))
            body += 1 + n_skip
    emit(addi(S0, S0, -1))
    if -4096 <= 4 * (loop - len(text)):
        emit(bne(S0, X0, 4 * (loop - len(text))))
    else:  # a body longer than a branch reaches: skip a backward JAL on exit
        emit(beq(S0, X0, 8))
        emit(jal(X0, 4 * (loop - len(text))))
    emit(li(A0, 0))
    emit(li(A7, 93))
    emit(ecall())
    leaf = len(text)
    ld, la, lb = rng.choice(OPERANDS), rng.choice(OPERANDS), rng.choice(OPERANDS)
    emit(r_type("sh1add", ld, la, lb))
    emit(r_type("xor", la, la, ld))
    emit(jalr(X0, RA, 0))
    for i, _ in pend:
        text[i] = jal(RA, 4 * (leaf - i))
    assert len(text) < 60000
    return Program(np.asarray(text, np.uint32), data)


def workload_programs(kind: str, n: int, base_seed: int) -> list[Program]:
    """Seeded programs ``base_seed + i`` of a named workload.

    * ``base``   the single-machine program family (4 KB data image);
    * ``many``   as ``base`` with 1-4 KB data images;
    * ``bignum`` the bignum-heavy mix with a 16 KB load/store range and enough loop iterations
                 for at least 100,000 trace tokens.
    """
    out = []
    for i in range(n):
        s = base_seed + i
        if kind == "base":
            out.append(gen_program(s))
        elif kind == "many":
            out.append(gen_program(s, data_bytes=1024 * (1 + s % 4)))
        elif kind == "bignum":
            out.append(gen_program(s, mix="bignum", iters=200))
        else:
            raise ValueError(kind)
    return out


def gdn_inputs(sequences: int = 1024, heads: int = 48, seed: int = 7, dk: int = 128) -> dict:
    """Inputs of one gated delta-rule decode step over sequences x heads independent heads, on
    the CPU (torch tensors): S {0, 1} bits (uint8, [BH, dk, dk]); keys one-hot at a uniform row,
    except a 5% share of unit-norm Gaussian keys ("general"); queries one-hot; v {0, 1}^dk; beta
    1; alpha 1 / 0.5 / 0 with probability 0.90 / 0.05 / 0.05."""
    import torch

    BH = sequences * heads
    g = torch.Generator(device="cpu").manual_seed(seed)
    S = torch.randint(0, 2, (BH, dk, dk), generator=g, dtype=torch.uint8)
    kr = torch.randint(0, dk, (BH,), generator=g)
    k = torch.zeros(BH, dk)
    k[torch.arange(BH), kr] = 1.0
    general = torch.rand(BH, generator=g) < 0.05
    kg = torch.randn(int(general.sum()), dk, generator=g)
    k[general] = kg / kg.norm(dim=1, keepdim=True)
    q = torch.zeros(BH, dk)
    q[torch.arange(BH), torch.randint(0, dk, (BH,), generator=g)] = 1.0
    v = torch.randint(0, 2, (BH, dk), generator=g).float()
    u = torch.rand(BH, generator=g)
    alpha = torch.where(u < 0.9, 1.0, torch.where(u < 0.95, 0.5, 0.0))
    beta = torch.ones(BH)
    return {"S": S, "q": q, "k": k, "v": v, "alpha": alpha, "beta": beta, "general": general}


def gdn_algorithmic_bytes(inp: dict) -> int:
    """HBM bytes one step must move for these draws: the inputs as stored (q, k, v, o rows,
    alpha, beta), then per head the whole 64 KB state read and written when alpha != 1 or the key
    is general (only written when alpha == 0), else the key row read and written and the query
    row read."""
    S, alpha, general = inp["S"], inp["alpha"], inp["general"]
    BH, dk = S.shape[0], S.shape[1]
    full = (alpha != 1.0) | general
    rd_full = int((full & (alpha != 0.0)).sum()) * dk * dk * 4
    wr_full = int(full.sum()) * dk * dk * 4
    light = int((~full).sum())
    return BH * (3 * dk * 4 + 8 + dk * 4) + rd_full + wr_full + light * 3 * dk * 4
