"""The tool-call calculator firmware of the merged machine's workload, in RV32IM machine code.

It follows the text bridge's calculator protocol (the reference's firmware source
``ERV/chipformer/rv/env/calc/calc.c:536-591``): the firmware parks (the ``exit`` ecall: HALT);
each run (GO, after ``</tool_call>``) reads the tool call's text from the text buffer (the call's
i-th token at TEXT_ADDR + 16 i, i = 1 .. 80, NUL-padded rows), takes what follows the second
``>`` up to the next ``<`` (newlines dropped) as the expression, prints

    \\n<tool_response>\\nVALUE\\n</tool_response>\\n<think>\\n\\n</think>\\n

(putchar 256 + k prints the k-th special: ``<tool_response>``, ``</tool_response>``, ``<think>``,
``</think>``) and parks again.  The reference's calculator evaluates general expressions on the
bignum digit file; this one evaluates ``A*B`` for two non-negative decimal integers of at most 20
digits each with the base RV32IM instructions (MUL, DIVU, REMU): the digits become base-10,000
limbs, the limb products (each partial sum below 5 * 9,999^2 < 2^32) are carried by DIVU / REMU,
and the value is printed limb by limb.  The reference's compiled calculator binary is not used.
"""

from __future__ import annotations

from .workload import (ROM_BASE, Program, _b, _i, _s, addi, ecall, jal, jalr, li, lw, r_type, slli,
                       sw)

ZERO, RA, T0, T1, T2, S0, S1, A0, A1, A2, A3, A4, A5, A6, A7 = 0, 1, 5, 6, 7, 8, 9, 10, 11, 12, 13, 14, 15, 16, 17
S2, S3, S4, S5, S6, S7, S8, S9, S10, S11, T3, T4, T5, T6 = 18, 19, 20, 21, 22, 23, 24, 25, 26, 27, 28, 29, 30, 31

TEXT_ADDR = 0x8000
ROWS = 80          # text rows the firmware scans (calc.c: ROWS)
MAX_DIGITS = 20    # digits kept per operand (5 limbs of 4)
A_DIG, B_DIG, A_LIMB, B_LIMB, PROD = 0x1000, 0x1100, 0x1200, 0x1240, 0x1280
TOOL_RESPONSE, TOOL_RESPONSE_END, THINK, THINK_END = 256, 257, 258, 259


def lbu(rd, rs1, imm=0):
    return _i(imm, rs1, 4, rd, 0x03)


def sb(rs2, rs1, imm=0):
    return _s(imm, rs2, rs1, 0)


class _Asm:
    """Words, some resolved against labels once every label is placed."""

    def __init__(self):
        self.words: list = []
        self.labels: dict[str, int] = {}

    def label(self, name: str) -> None:
        assert name not in self.labels, name
        self.labels[name] = len(self.words)

    def w(self, *words) -> None:
        for x in words:
            self.words.extend(x if isinstance(x, list) else [x])

    def br(self, f3: int, rs1: int, rs2: int, target: str) -> None:
        self.words.append(lambda i, L: _b((L[target] - i) * 4, rs2, rs1, f3))

    def jal(self, rd: int, target: str) -> None:
        self.words.append(lambda i, L: jal(rd, (L[target] - i) * 4))

    def words_out(self) -> list[int]:
        return [x(i, self.labels) if callable(x) else x for i, x in enumerate(self.words)]


BEQ, BNE, BLT, BGE, BLTU, BGEU = 0, 1, 4, 5, 6, 7


def _putc(a: _Asm, c: int) -> None:
    a.w(li(A0, c), li(A7, 1), ecall())


def calc_program() -> Program:
    """The firmware image (text from ROM_BASE, no data)."""
    a = _Asm()
    a.label("park")
    a.w(li(A7, 93), ecall())  # park: HALT; the next GO resumes here
    # ---- gather: the call's text after the second '>' up to '<' (digits, '*') ----
    a.w(li(T0, TEXT_ADDR + 16), li(T6, TEXT_ADDR + 16 * (ROWS + 1)), li(T1, 0), li(S2, 0), li(S3, 0),
        li(S4, 0), li(S5, A_DIG), li(S6, B_DIG))
    a.label("row")
    a.br(BGEU, T0, T6, "gathered")
    a.w(li(T2, 0))
    a.label("char")
    a.w(r_type("add", T3, T0, T2), lbu(A0, T3, 0))
    a.br(BEQ, A0, ZERO, "next_row")  # a row ends at its NUL
    a.w(li(T4, 2))
    a.br(BLTU, T1, T4, "header")
    a.w(li(T4, ord("<")))
    a.br(BEQ, A0, T4, "gathered")
    a.w(li(T4, ord("*")))
    a.br(BEQ, A0, T4, "star")
    a.w(addi(A0, A0, -ord("0")), li(T4, 10))
    a.br(BGEU, A0, T4, "next_char")  # not a digit (a newline)
    a.br(BNE, S4, ZERO, "digit_b")
    a.w(li(T4, MAX_DIGITS))
    a.br(BGEU, S2, T4, "next_char")
    a.w(r_type("add", T5, S5, S2), sb(A0, T5, 0), addi(S2, S2, 1))
    a.jal(ZERO, "next_char")
    a.label("digit_b")
    a.w(li(T4, MAX_DIGITS))
    a.br(BGEU, S3, T4, "next_char")
    a.w(r_type("add", T5, S6, S3), sb(A0, T5, 0), addi(S3, S3, 1))
    a.jal(ZERO, "next_char")
    a.label("star")
    a.w(li(S4, 1))
    a.jal(ZERO, "next_char")
    a.label("header")
    a.w(li(T4, ord(">")))
    a.br(BNE, A0, T4, "next_char")
    a.w(addi(T1, T1, 1))
    a.label("next_char")
    a.w(addi(T2, T2, 1), li(T4, 16))
    a.br(BLTU, T2, T4, "char")
    a.label("next_row")
    a.w(addi(T0, T0, 16))
    a.jal(ZERO, "row")
    a.label("gathered")
    _putc(a, ord("\n"))
    _putc(a, TOOL_RESPONSE)
    _putc(a, ord("\n"))
    # ---- operands to base-10,000 limbs (little-endian, 5 each) ----
    a.w(r_type("add", A1, S5, ZERO), r_type("add", A2, S2, ZERO), li(A3, A_LIMB))
    a.jal(RA, "to_limbs")
    a.w(r_type("add", A1, S6, ZERO), r_type("add", A2, S3, ZERO), li(A3, B_LIMB))
    a.jal(RA, "to_limbs")
    # ---- product: P[i + j] += A[i] B[j], then the carries ----
    a.w(li(T0, PROD), li(T1, 0), li(T2, 10))
    a.label("clear_p")
    a.w(sw(ZERO, T0, 0), addi(T0, T0, 4), addi(T1, T1, 1))
    a.br(BLTU, T1, T2, "clear_p")
    a.w(li(S7, 0))
    a.label("mul_i")
    a.w(li(S8, 0))
    a.label("mul_j")
    a.w(slli(T0, S7, 2), li(T1, A_LIMB), r_type("add", T0, T0, T1), lw(T2, T0, 0),
        slli(T0, S8, 2), li(T1, B_LIMB), r_type("add", T0, T0, T1), lw(T3, T0, 0),
        r_type("mul", T4, T2, T3),
        r_type("add", T0, S7, S8), slli(T0, T0, 2), li(T1, PROD), r_type("add", T0, T0, T1),
        lw(T5, T0, 0), r_type("add", T5, T5, T4), sw(T5, T0, 0),
        addi(S8, S8, 1), li(T1, 5))
    a.br(BLTU, S8, T1, "mul_j")
    a.w(addi(S7, S7, 1), li(T1, 5))
    a.br(BLTU, S7, T1, "mul_i")
    a.w(li(S7, 0), li(S9, 10000))
    a.label("carry")
    a.w(slli(T0, S7, 2), li(T1, PROD), r_type("add", T0, T0, T1), lw(T2, T0, 0),
        r_type("divu", T3, T2, S9), r_type("remu", T2, T2, S9), sw(T2, T0, 0),
        lw(T4, T0, 4), r_type("add", T4, T4, T3), sw(T4, T0, 4),
        addi(S7, S7, 1), li(T1, 9))
    a.br(BLTU, S7, T1, "carry")
    # ---- print: the top nonzero limb without leading zeros, the rest as four digits ----
    a.w(li(S7, 9))
    a.label("top")
    a.w(slli(T0, S7, 2), li(T1, PROD), r_type("add", T0, T0, T1), lw(A1, T0, 0))
    a.br(BNE, A1, ZERO, "print_top")
    a.br(BEQ, S7, ZERO, "print_top")
    a.w(addi(S7, S7, -1))
    a.jal(ZERO, "top")
    a.label("print_top")
    a.w(li(S10, 0))  # leading zeros are skipped until a digit is printed
    for d in (1000, 100, 10):
        a.w(li(T5, d), r_type("divu", A0, A1, T5), r_type("remu", A1, A1, T5))
        a.br(BNE, A0, ZERO, f"top_digit{d}")
        a.br(BEQ, S10, ZERO, f"top_skip{d}")
        a.label(f"top_digit{d}")
        a.w(addi(A0, A0, ord("0")), li(A7, 1), ecall(), li(S10, 1))
        a.label(f"top_skip{d}")
    a.w(addi(A0, A1, ord("0")), li(A7, 1), ecall())
    a.label("rest")
    a.br(BEQ, S7, ZERO, "printed")
    a.w(addi(S7, S7, -1), slli(T0, S7, 2), li(T1, PROD), r_type("add", T0, T0, T1), lw(A1, T0, 0))
    for d in (1000, 100, 10):
        a.w(li(T5, d), r_type("divu", A0, A1, T5), r_type("remu", A1, A1, T5),
            addi(A0, A0, ord("0")), li(A7, 1), ecall())
    a.w(addi(A0, A1, ord("0")), li(A7, 1), ecall())
    a.jal(ZERO, "rest")
    a.label("printed")
    for c in (ord("\n"), TOOL_RESPONSE_END, ord("\n"), THINK, ord("\n"), ord("\n"), THINK_END, ord("\n")):
        _putc(a, c)
    a.jal(ZERO, "park")
    # ---- to_limbs(a1 = digits, most significant first; a2 = count; a3 = 5 limbs) ----
    a.label("to_limbs")
    a.w(sw(ZERO, A3, 0), sw(ZERO, A3, 4), sw(ZERO, A3, 8), sw(ZERO, A3, 12), sw(ZERO, A3, 16),
        li(T0, 0), r_type("add", T1, A2, ZERO))
    a.label("limb")
    a.br(BEQ, T1, ZERO, "limbs_done")
    a.w(addi(T2, T1, -4))
    a.br(BGE, T2, ZERO, "limb_from")
    a.w(li(T2, 0))
    a.label("limb_from")
    a.w(li(T3, 0), r_type("add", T4, T2, ZERO))
    a.label("limb_digit")
    a.br(BGEU, T4, T1, "limb_store")
    a.w(li(T5, 10), r_type("mul", T3, T3, T5), r_type("add", T5, A1, T4), lbu(T5, T5, 0),
        r_type("add", T3, T3, T5), addi(T4, T4, 1))
    a.jal(ZERO, "limb_digit")
    a.label("limb_store")
    a.w(slli(T5, T0, 2), r_type("add", T5, T5, A3), sw(T3, T5, 0), addi(T0, T0, 1), r_type("add", T1, T2, ZERO))
    a.jal(ZERO, "limb")
    a.label("limbs_done")
    a.w(jalr(ZERO, RA, 0))
    import numpy as np

    return Program(np.asarray(a.words_out(), np.uint32), b"", entry=ROM_BASE)


def expected_response(a: int, b: int) -> bytes:
    """The bytes the firmware prints for the call A*B (before the HALT echo)."""
    return b"\n<tool_response>\n" + str(a * b).encode() + b"\n</tool_response>\n<think>\n\n</think>\n"
