"""CPU ORACLE (test infrastructure only; never the product path).

ctypes front end of ``liboracle.so`` (``qx_oracle.c``): the reference's executor step, free-run
decode, traced RV32 machine, snapshot / readback and gated delta-rule recurrence, restated in
plain C.  Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU legs import this
module, as the checker or as the timed CPU baseline.  Reference citations are in ``qx_oracle.c``.
"""

from __future__ import annotations

import ctypes as C
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "liboracle.so"
HD = 128
RAM_WORDS = 1 << 13
ROM_WORDS = 1 << 16


def build() -> Path:
    """Compile liboracle.so (gcc) if it is missing or older than its source."""
    src = HERE / "qx_oracle.c"
    if not LIB_PATH.exists() or LIB_PATH.stat().st_mtime < src.stat().st_mtime:
        subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB_PATH


_lib = None


def lib():
    global _lib
    if _lib is None:
        build()
        _lib = C.CDLL(str(LIB_PATH))
        _lib.qxo_step.restype = C.c_int
        _lib.qxo_decode.restype = C.c_int32
        _lib.qxo_rom_word.restype = C.c_uint32
        _lib.qxo_rom_word.argtypes = [C.c_uint32, C.c_uint32]
        _lib.qxo_machine_size.restype = C.c_int64
        _lib.qxo_machine_run.restype = C.c_int64
        _lib.qxo_machine_record.restype = C.c_int64
        _lib.qxo_trace_and_state.restype = C.c_int64
        _lib.qxo_fnv1a.restype = C.c_uint64
        _lib.qxo_state_checksum.restype = C.c_uint64
        _lib.qxo_tok_family.restype = C.c_int32
        _lib.qxo_vocab.restype = C.c_int32
    return _lib


def _p(a: np.ndarray, t):
    assert a.flags["C_CONTIGUOUS"], "arrays passed to the oracle must be contiguous"
    return a.ctypes.data_as(C.POINTER(t))


class _Forms(C.Structure):
    _fields_ = [("ptr", C.POINTER(C.c_int64)), ("idx", C.POINTER(C.c_int32)),
                ("w", C.POINTER(C.c_float))]


class _Graph(C.Structure):
    _fields_ = [
        ("D", C.c_int32), ("n_levels", C.c_int32), ("levels", C.POINTER(C.c_int32)),
        ("level_kind", C.POINTER(C.c_int8)),
        ("n_ffn", C.c_int32), ("ffn_level", C.POINTER(C.c_int32)),
        ("ffn_out", C.POINTER(C.c_int32)), ("ffn_uptr", C.POINTER(C.c_int64)),
        ("unit_coef", C.POINTER(C.c_float)), ("unit_a", _Forms), ("unit_b", _Forms),
        ("n_heads", C.c_int32), ("head_level", C.POINTER(C.c_int32)),
        ("head_qhot", C.POINTER(C.c_int32)), ("head_q", C.POINTER(C.c_int32)),
        ("head_k", C.POINTER(C.c_int32)), ("q_forms", _Forms), ("k_forms", _Forms),
        ("n_vh", C.c_int32), ("vh_head", C.POINTER(C.c_int32)), ("vh_v", C.POINTER(C.c_int32)),
        ("vh_z", C.POINTER(C.c_int32)), ("vh_nrows", C.POINTER(C.c_int32)),
        ("vh_has_beta", C.POINTER(C.c_uint8)), ("v_forms", _Forms), ("z_forms", _Forms),
        ("vh_a", _Forms), ("vh_beta", _Forms), ("vh_out_ptr", C.POINTER(C.c_int64)),
        ("out_col", C.POINTER(C.c_int32)), ("out_dim", C.POINTER(C.c_int32)),
        ("out_w", C.POINTER(C.c_float)),
    ]


class _Decoder(C.Structure):
    _fields_ = [("nf", C.c_int32), ("npay", C.c_int32), ("F", C.c_int32), ("rows", C.c_int32),
                ("nfam", C.c_int32), ("fam_dims", C.POINTER(C.c_int32)),
                ("pay_dims", C.POINTER(C.c_int32)), ("feat_dims", C.POINTER(C.c_int32)),
                ("fam_ids", C.POINTER(C.c_int64)), ("fam_row0", C.POINTER(C.c_int64)),
                ("fam_small", C.POINTER(C.c_uint8)), ("base", C.POINTER(C.c_float)),
                ("bits", C.POINTER(C.c_float)), ("table", C.POINTER(C.c_float))]


class _TPos(C.Structure):
    _fields_ = [("sub", C.c_int32), ("vh0", C.c_int32)]


class _Tables(C.Structure):
    _fields_ = [("pc", _TPos), ("count", _TPos), ("j", _TPos), ("vcnt", _TPos),
                ("regs", _TPos * 3), ("quo", _TPos * 4), ("rom", _TPos * 32),
                ("drom", _TPos * 16), ("bn1", _TPos * 4), ("bn2", _TPos * 4),
                ("ram", _TPos * 32), ("reg_cols", (C.c_int32 * 8) * 32)]


class State(C.Structure):
    """Registers x0..x31, PC anchor and n (PC = 0x40000 + 4 (anchor + n)), RAM words."""
    _fields_ = [("x", C.c_uint32 * 32), ("anchor", C.c_uint32), ("n", C.c_uint32),
                ("ram", C.c_uint32 * RAM_WORDS)]

    def checksum(self) -> int:
        return int(lib().qxo_state_checksum(C.byref(self)))

    def as_dict(self) -> dict:
        return {"x": list(self.x), "anchor": self.anchor, "n": self.n,
                "ram": np.ctypeslib.as_array(self.ram).copy()}


class Oracle:
    """The oracle for one compiled graph (a :class:`qwenputer_b200.graphfile.GraphData`)."""

    def __init__(self, g):
        self.g = g
        self.keep = []  # arrays the C structs point into
        L = lib()
        del L

        def arr(a, dt):
            a = np.ascontiguousarray(np.asarray(a, dt))
            self.keep.append(a)
            return a

        def forms(f):
            return _Forms(_p(arr(f.ptr, np.int64), C.c_int64), _p(arr(f.idx, np.int32), C.c_int32),
                          _p(arr(f.w, np.float32), C.c_float))

        i32, i64, f32 = C.c_int32, C.c_int64, C.c_float
        self.cg = _Graph(
            g.D, len(g.levels), _p(arr(g.levels, np.int32), i32),
            _p(arr(g.level_kind, np.int8), C.c_int8),
            len(g.ffn_level), _p(arr(g.ffn_level, np.int32), i32), _p(arr(g.ffn_out, np.int32), i32),
            _p(arr(g.ffn_uptr, np.int64), i64), _p(arr(g.unit_coef, np.float32), f32),
            forms(g.unit_a), forms(g.unit_b),
            len(g.head_level), _p(arr(g.head_level, np.int32), i32),
            _p(arr(g.head_qhot, np.int32), i32), _p(arr(g.head_q, np.int32), i32),
            _p(arr(g.head_k, np.int32), i32), forms(g.q_forms), forms(g.k_forms),
            len(g.vh_head), _p(arr(g.vh_head, np.int32), i32), _p(arr(g.vh_v, np.int32), i32),
            _p(arr(g.vh_z, np.int32), i32), _p(arr(g.vh_nrows, np.int32), i32),
            _p(arr(g.vh_has_beta, np.uint8), C.c_uint8), forms(g.v_forms), forms(g.z_forms),
            forms(g.vh_a), forms(g.vh_beta), _p(arr(g.vh_out_ptr, np.int64), i64),
            _p(arr(g.out_col, np.int32), i32), _p(arr(g.out_dim, np.int32), i32),
            _p(arr(g.out_w, np.float32), f32))
        self.head_levels = g.head_sublayers()
        self.V = np.asarray([len(g.vheads_at(lv)) for lv in self.head_levels], np.int32)
        self.cdec = _Decoder(
            len(g.fam_ids), g.emb_bits.shape[1], len(g.feat_dims), g.emb_table.shape[0],
            len(g.fam_dims), _p(arr(g.fam_dims, np.int32), i32), _p(arr(g.pay_dims, np.int32), i32),
            _p(arr(g.feat_dims, np.int32), i32), _p(arr(g.fam_ids, np.int64), i64),
            _p(arr(g.fam_row0, np.int64), i64), _p(arr(g.fam_small, np.uint8), C.c_uint8),
            _p(arr(g.emb_base, np.float32), f32), _p(arr(g.emb_bits, np.float32), f32),
            _p(arr(g.emb_table, np.float32), f32))
        self.fam_size = arr(g.fam_size, np.int64)
        self.tables = self._tables()

    def _tables(self) -> _Tables:
        g = self.g
        t = _Tables()
        hl = {lv: i for i, lv in enumerate(self.head_levels)}

        def pos(name):
            lv, vh0, _ = g.table_position(name)
            return _TPos(hl[lv], vh0)

        t.pc, t.count, t.j, t.vcnt = pos("pc"), pos("count"), pos("j"), pos("vcnt")
        for i, p in enumerate(("rs1", "rs2", "rd")):
            t.regs[i] = pos(f"regs.{p}")
        for i in range(4):
            t.quo[i] = pos(f"quo{i}")
            t.bn1[i] = pos(f"bn1.{i}")
            t.bn2[i] = pos(f"bn2.{i}")
        for i in range(32):
            t.rom[i] = pos(f"rom{i}")
            t.ram[i] = pos(f"ram{i}")
        for i in range(16):
            t.drom[i] = pos(f"drom{i}")
        for i in range(32):
            for j in range(8):
                t.reg_cols[i][j] = int(g.reg_cols[i, j])
        return t

    # ---- executor state -------------------------------------------------------------------
    def new_state(self, B: int) -> dict:
        D = self.g.D
        return {"x": np.zeros((B, D), np.float32),
                "hist": [np.zeros((B, 3, D), np.float32) for _ in self.head_levels],
                "S": [np.zeros((B, int(v), HD, HD), np.float32) for v in self.V]}

    def step(self, st: dict, x: np.ndarray | None = None, nthreads: int | None = None) -> np.ndarray:
        """One Executor2 step over every row: x [B, D] in place (st['x'] if x is None)."""
        x = st["x"] if x is None else x
        assert x.dtype == np.float32 and x.flags["C_CONTIGUOUS"]
        B = x.shape[0]
        hp = (C.POINTER(C.c_float) * len(st["hist"]))(*[_p(h, C.c_float) for h in st["hist"]])
        sp = (C.POINTER(C.c_float) * len(st["S"]))(*[_p(s, C.c_float) for s in st["S"]])
        nt = nthreads or os.cpu_count() or 1
        lib().qxo_step(C.byref(self.cg), C.c_int32(B), _p(x, C.c_float), hp, sp,
                       _p(self.V, C.c_int32), C.c_int32(nt))
        return x

    def decode(self, out: np.ndarray) -> tuple[np.ndarray, np.ndarray, int]:
        """FreeRun._step's decode: (tokens [B], next embeddings [B, D], rows with no valid code)."""
        B, D = out.shape
        tok = np.zeros(B, np.int64)
        xn = np.zeros((B, D), np.float32)
        bad = lib().qxo_decode(C.byref(self.cdec), C.c_int32(B), C.c_int32(D),
                               _p(np.ascontiguousarray(out, np.float32), C.c_float),
                               _p(tok, C.c_int64), _p(xn, C.c_float), _p(self.fam_size, C.c_int64))
        return tok, xn, int(bad)

    def snapshot(self, st: dict, row: int, m: "Machine") -> None:
        """core.snapshot + Executor2.load_init of machine m into batch row `row`."""
        views = [s[row] for s in st["S"]]
        for v in views:
            v[...] = 0
        sp = (C.POINTER(C.c_float) * len(views))(*[_p(v, C.c_float) for v in views])
        lib().qxo_snapshot(C.byref(self.tables), m.ptr, sp, _p(self.V, C.c_int32))

    def readback(self, st: dict, row: int) -> State:
        views = [np.ascontiguousarray(s[row]) for s in st["S"]]
        sp = (C.POINTER(C.c_float) * len(views))(*[_p(v, C.c_float) for v in views])
        out = State()
        lib().qxo_readback(C.byref(self.tables), sp, _p(self.V, C.c_int32), C.byref(out))
        return out

    def free_run(self, st: dict, first_tokens: list[int], n: int) -> np.ndarray:
        """FreeRun.run: from the first tokens' embeddings, n steps of step + decode; returns the
        [B, n] predicted tokens."""
        B = len(first_tokens)
        x = self.g.embed(first_tokens)
        out = np.zeros((B, n), np.int64)
        for t in range(n):
            self.step(st, x)
            tok, x, _ = self.decode(x)
            out[:, t] = tok
        return out


class Machine:
    """The traced RV32 machine (ref.Machine) of the C oracle."""

    def __init__(self, text, data=b"", data_base=0x100, rodata=b"", entry=0x40000):
        L = lib()
        self.buf = C.create_string_buffer(int(L.qxo_machine_size()))
        self.ptr = C.cast(self.buf, C.c_void_p)
        t = np.ascontiguousarray(np.asarray(text, np.uint32))
        d = np.frombuffer(bytes(data), np.uint8).copy()
        r = np.frombuffer(bytes(rodata), np.uint8).copy()
        L.qxo_machine_init(self.ptr, _p(t, C.c_uint32), C.c_int32(len(t)), _p(d, C.c_uint8),
                           C.c_int32(len(d)), C.c_uint32(data_base), _p(r, C.c_uint8),
                           C.c_int32(len(r)), C.c_uint32(entry))

    @classmethod
    def from_program(cls, prog) -> "Machine":
        return cls(prog.text, prog.data, prog.data_base, prog.rodata, prog.entry)

    def copy(self) -> "Machine":
        m = Machine.__new__(Machine)
        m.buf = C.create_string_buffer(self.buf.raw, len(self.buf))
        m.ptr = C.cast(m.buf, C.c_void_p)
        return m

    def run(self, max_tokens: int = 10 ** 6) -> np.ndarray:
        """Machine.run: GO, then records until HALT or at least max_tokens tokens."""
        cap = max_tokens + 256
        out = np.zeros(cap, np.int32)
        n = lib().qxo_machine_run(self.ptr, C.c_int64(max_tokens), _p(out, C.c_int32), C.c_int64(cap))
        assert n <= cap
        return out[:n].astype(np.int64)

    def trace_and_state(self, n: int) -> tuple[np.ndarray, State]:
        """(GO + the first n predicted tokens (shorter if the machine halts), the state after the
        last record completed within the first n tokens)."""
        toks = np.zeros(n + 1, np.int32)
        st = State()
        ln = lib().qxo_trace_and_state(self.ptr, C.c_int64(n), _p(toks, C.c_int32), C.byref(st))
        return toks[:ln].astype(np.int64), st

    def state(self) -> State:
        st = State()
        lib().qxo_machine_state(self.ptr, C.byref(st))
        return st


def rom_word(w: int, pc: int) -> int:
    return int(lib().qxo_rom_word(w, pc))


def fnv1a(words: np.ndarray, h: int = 0xcbf29ce484222325) -> int:
    w = np.ascontiguousarray(np.asarray(words, np.uint32))
    return int(lib().qxo_fnv1a(_p(w, C.c_uint32), C.c_int64(len(w)), C.c_uint64(h)))


def gdn_step(S, q, k, v, alpha, beta) -> np.ndarray:
    """The gated delta-rule step (in place on S [BH, dk, dv]); returns o [BH, dv]."""
    BH, dk, dv = S.shape
    o = np.zeros((BH, dv), np.float32)
    args = [np.ascontiguousarray(a, np.float32) for a in (q, k, v, alpha, beta)]
    assert S.dtype == np.float32 and S.flags["C_CONTIGUOUS"]
    lib().qxo_gdn_step(C.c_int64(BH), C.c_int32(dk), C.c_int32(dv), _p(S, C.c_float),
                       *[_p(a, C.c_float) for a in args], _p(o, C.c_float))
    return o
