"""The executor as the reference's callers see it, over the C ABI of include/qx.h.

``Executor`` keeps the surface of the reference's Triton executor
(``ERV/chipformer/rv/tritonexec.py:173-289``, ``Executor2``): ``Executor(c, batch, device)``,
``D``, ``B``, ``steps`` (one dict per sublayer; head sublayers expose ``"S"`` ``[B, V, 128, 128]``
fp32 device tensors mutated in place and ``"hist"``), ``load_init(row)``, ``reset(rows)``,
``embed(toks)`` and ``step(x)``; so ``chat.ExecRow``-style callers (clone / restore ``S`` and
``hist``, capture ``step`` in a CUDA graph) work unchanged.  ``FreeRun`` keeps the surface of
``ERV/chipformer/rv/fastexec.py:236-340`` (``load(row, first_token)``, ``run(n)``) with decode and
next embedding on the device inside the same persistent kernel.

Differences a caller can observe:
  * ``hist`` is ``[B, 3, n]`` over the ``n`` dims that sublayer's heads read at lags 1..3 (the
    only dims the history is kept for), not ``[B, 3, D]``; ``hist_dims[i]`` lists them;
  * a machine can be loaded without a live graph: ``load_machines(row0, programs)`` builds the
    head states on the device from program images (``core.snapshot``'s layout).

There is no CPU fallback: without libqx.so or a CUDA device every entry point raises.
"""

from __future__ import annotations

import ctypes as C
from pathlib import Path

import numpy as np

from . import graphfile
from .plan import compile_plan

import os

LIB_PATH = Path(os.environ.get("QX_LIBRARY") or Path(__file__).resolve().parent / "libqx.so")
HD = 128
_lib = None
_plans: dict = {}


class QxError(RuntimeError):
    pass


def lib():
    """libqx.so, loaded once; raises if it was not built (python -m qwenputer_b200.build)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise QxError(f"{LIB_PATH} is missing: build it with `python -m qwenputer_b200.build`")
        L = C.CDLL(str(LIB_PATH))
        L.qx_last_error.restype = C.c_char_p
        for name in ("qx_create", "qx_destroy", "qx_buffer", "qx_reset", "qx_load_machines",
                     "qx_step", "qx_run", "qx_set_tokens", "qx_readback", "qx_checksums",
                     "qx_errors", "qx_gdn_step", "qx_gdn_step_noalloc", "qx_info",
                     "qx_cluster_capacity", "qx_set_table_images"):
            getattr(L, name).restype = C.c_int
        L.qx_gdn_work_bytes.restype = C.c_size_t
        L.qx_gdn_work_bytes.argtypes = [C.c_int64]
        _lib = L
    return _lib


def check(status: int, what: str) -> None:
    if status != 0:
        raise QxError(f"{what}: status {status}: {lib().qx_last_error().decode()}")


class Machine(C.Structure):
    """qx_machine (include/qx.h)."""
    _fields_ = [("rom", C.c_void_p), ("rom_words", C.c_uint32), ("drom", C.c_void_p),
                ("drom_bytes", C.c_uint32), ("ram", C.c_void_p), ("x", C.c_uint32 * 32),
                ("anchor", C.c_uint32), ("n", C.c_uint32), ("bn", C.c_void_p)]


class State(C.Structure):
    """qx_state: registers, PC anchor / n (PC = 0x40000 + 4 (anchor + n)), RAM words."""
    _fields_ = [("x", C.c_uint32 * 32), ("anchor", C.c_uint32), ("n", C.c_uint32),
                ("ram", C.c_uint32 * 8192)]


class _DevArray:
    """A device buffer of the executor seen by torch without a copy."""

    def __init__(self, ptr: int, shape, typestr: str):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr,
                                         "data": (ptr, False), "version": 3, "strides": None}


def _torch():
    import torch

    if not torch.cuda.is_available():
        raise QxError("the executor needs a CUDA device; there is no CPU path")
    return torch


def load_graph(c=None) -> graphfile.GraphData:
    """A GraphData from: None (the standalone RV32IM core shipped with the package), a path, a
    GraphData, or a live chipformer graph (exported on the fly)."""
    if c is None:
        return graphfile.load_graph(graphfile.default_graph_path())
    if isinstance(c, graphfile.GraphData):
        return c
    if isinstance(c, (str, Path)):
        return graphfile.load_graph(c)
    return graphfile.export_graph(c)


def plan_for(g: graphfile.GraphData, cluster: int = 1, tc: bool = False, group: int = 32):
    key = (id(g), cluster, tc, group)
    if key not in _plans:
        _plans[key] = (g, compile_plan(g, cluster=cluster, tc=tc, group=group))
    return _plans[key][1]


def pick_group(batch: int, device: int) -> int:
    """Machines a CTA runs: the smallest group (4, 8, 16 or 32) whose CTAs, one per SM, the
    device holds at once, so that few machines per GPU still spread over the SMs with every CTA
    independent (4,096 machines on a 148-SM B200: 32; 512: 4)."""
    sms = _torch().cuda.get_device_properties(device).multi_processor_count
    for g in (4, 8, 16):
        if -(-batch // g) <= sms:
            return g
    return 32


def cluster_capacity(g: graphfile.GraphData, cluster: int, device: int) -> int:
    """Clusters of `cluster` token-kernel CTAs the device holds at once (qx_cluster_capacity)."""
    blob = plan_for(g, 1).blob()
    n = C.c_int32()
    check(lib().qx_cluster_capacity(blob, C.c_size_t(len(blob)), C.c_int32(device), C.c_int32(cluster),
                                    C.byref(n)), "qx_cluster_capacity")
    return int(n.value)


def pick_cluster(batch: int, g: graphfile.GraphData, device: int) -> int:
    """CTAs per group of 32 machines: the largest size (up to 8) whose clusters all fit on the
    device at once, so a small batch still spreads its work over the SMs (4,096 machines: 1)."""
    groups = (batch + 31) // 32
    for c in range(8, 1, -1):
        if cluster_capacity(g, c, device) >= groups:
            return c
    return 1


def program_image(prog, keep: list) -> Machine:
    """A qx_machine for a freshly loaded program (ref.Machine.from_program, ERV/chipformer/rv/
    ref.py:401-414): text at 0x40000, data at data_base, rodata at 0x20000, sp = 0x8000."""
    text = np.ascontiguousarray(np.asarray(prog.text, np.uint32))
    ram = np.zeros(8192 * 4, np.uint8)
    data = np.frombuffer(bytes(prog.data), np.uint8)
    ram[prog.data_base:prog.data_base + len(data)] = data[:max(0, 8192 * 4 - prog.data_base)]
    ramw = ram.view(np.uint32).copy()
    rod = np.frombuffer(bytes(getattr(prog, "rodata", b"")) or b"\0", np.uint8).copy()
    keep += [text, ramw, rod]
    m = Machine()
    m.rom, m.rom_words = text.ctypes.data, len(text)
    m.drom, m.drom_bytes = rod.ctypes.data, len(getattr(prog, "rodata", b""))
    m.ram = ramw.ctypes.data
    m.x[2] = 0x8000
    m.anchor = (prog.entry - 0x40000) >> 2
    m.n = 0
    m.bn = None
    return m


def state_image(prog, x, anchor: int, n: int, ram, keep: list) -> Machine:
    """A qx_machine for a machine in a given state (e.g. a firmware run to its park, as the text
    bridge starts it: ERV/chipformer/rv/bridge.py:106-111): the program's ROM / DROM, and the
    registers, PC (anchor, n) and 8,192 RAM words given."""
    m = program_image(prog, keep)
    ramw = np.ascontiguousarray(np.asarray(ram, np.uint32))
    assert ramw.shape == (8192,)
    keep.append(ramw)
    m.ram = ramw.ctypes.data
    for i in range(32):
        m.x[i] = int(x[i]) if i else 0
    m.anchor, m.n = int(anchor), int(n)
    return m


def snapshot_states(c, head_levels) -> list:
    """Executor2.load_init's host buffers (tritonexec.py:246-258): for each head sublayer level,
    a [V, 128, 128] fp32 array of the value heads' initial rows that the live graph's heads hold
    (``Head.init``, written by ``core.snapshot``), value heads in node order."""
    from chipformer.q35.ir import Head

    out = []
    for lv in head_levels:
        heads = [n for n in c.nodes if n.level == lv and isinstance(n, Head)]
        buf = np.zeros((sum(len(n.vheads()) for n in heads), HD, HD), np.float32)
        j = 0
        for n in heads:
            init = n.init or []
            for x in range(len(n.vheads())):
                for r, vec in (init[x] if x < len(init) else {}).items():
                    buf[j, r] = vec
                j += 1
        out.append(buf)
    return out


class Executor:
    """Executor2's surface (tritonexec.py:173-289) on the B200 kernel."""

    def __init__(self, c=None, batch: int = 1, device="cuda", cluster: int | None = None, tc: bool = False,
                 table_images: int | None = None, group: int | None = None):
        """``group``: machines one CTA runs (32, or 16 / 8 / 4 with a warp's lanes running that
        many fewer machines and 32 / group stream records side by side; default: pick_group, or 32
        when ``cluster`` or ``tc`` is given).  ``cluster``: CTAs (a thread-block cluster) sharing a
        group of 32 machines.  ``tc``: run the linear forms on the tensor cores (tcgen05 MMA
        phases) instead of the CUDA cores; the results are the same bits either way.  ``table_images``: machines running
        the same firmware share one copy of its read-only ROM / DROM tables, in that many image
        slots (qx_set_table_images); the head sublayers holding only those tables then expose
        ``S`` as [table_images, V, 128, 128] and ``table_image`` gives each machine's slot."""
        torch = _torch()
        self.g = load_graph(c)
        self.c = c
        self.B = int(batch)
        self.dev = torch.device(device)
        if self.dev.index is None:
            self.dev = torch.device("cuda", torch.cuda.current_device())
        if group is None:
            group = 32 if (cluster is not None or tc) else pick_group(self.B, self.dev.index)
        self.group = int(group)
        if cluster is None:
            cluster = 1 if self.group < 32 else pick_cluster(self.B, self.g, self.dev.index)
        self.cluster = int(cluster)
        self.tc = bool(tc)
        self.plan = plan_for(self.g, self.cluster, self.tc, self.group)
        self.D = int(self.g.D)
        blob = self.plan.blob()
        self._blob = C.create_string_buffer(blob, len(blob))
        h = C.c_void_p()
        with torch.cuda.device(self.dev):
            check(lib().qx_create(self._blob, C.c_size_t(len(blob)), C.c_int32(self.B),
                                  C.c_int32(self.dev.index), C.byref(h)), "qx_create")
        self.h = h
        self.table_images = int(table_images) if table_images else 0
        if self.table_images:
            check(lib().qx_set_table_images(self.h, C.c_int32(self.table_images)), "qx_set_table_images")
        self.x = self._buffer(0, 0, (self.B, self.D), "<f4")
        self.err = self._buffer(3, 0, (self.B,), "<u4")
        self.hash = self._buffer(4, 0, (self.B,), "<u8")
        self.count = self._buffer(5, 0, (self.B,), "<i8")
        self.halt_at = self._buffer(6, 0, (self.B,), "<i8")
        self.state_bytes = self._buffer(7, 0, (1,), "<u8")
        self.y = torch.zeros(self.B, self.D, device=self.dev)  # Executor2.y (unused here)
        self.steps, self.hist_dims = [], []
        hl = 0
        for lv, kind in zip(self.g.levels, self.g.level_kind):
            if kind == 0:
                self.steps.append({"kind": "ffn", "level": int(lv)})
                continue
            V = len(self.g.vheads_at(int(lv)))
            ne = max(1, len(self.plan.lag_dims[int(lv)]))
            bpad = (self.B + 31) // 32 * 32
            copies = self._buffer_bytes(1, hl) // (V * HD * HD * 4)  # B, or the image slots (shared)
            S = self._buffer(1, hl, (copies, V, HD, HD), "<f4")
            H = self._buffer(2, hl, (3, ne, bpad), "<f4").permute(2, 0, 1)[:self.B]
            self.steps.append({"kind": "head", "level": int(lv), "V": V, "S": S, "hist": H,
                               "shared": bool(self.table_images) and self._shared(hl),
                               "heads": [str(self.g.head_name[h]) for h in self.g.heads_at(int(lv))]})
            self.hist_dims.append(self.plan.lag_dims[int(lv)])
            hl += 1
        self.feat_ids = [int(d) for d in self.g.feat_dims[1:]]
        self.table_image = self._buffer(8, 0, (self.B,), "<i4") if self.table_images else None

    def info(self, what: int) -> int:
        """qx_info: 0 cluster size, 1 clusters the device holds at once, 2 CTAs a launch, 3 smem."""
        v = C.c_int64()
        check(lib().qx_info(self.h, C.c_int32(what), C.byref(v)), "qx_info")
        return int(v.value)

    def _buffer_bytes(self, kind: int, i: int) -> int:
        p, n = C.c_void_p(), C.c_size_t()
        check(lib().qx_buffer(self.h, C.c_int32(kind), C.c_int32(i), C.byref(p), C.byref(n)), "qx_buffer")
        return int(n.value)

    def _shared(self, hl: int) -> bool:
        """Whether head sublayer hl holds only ROM / DROM tables (shared with table_images)."""
        from .plan import TABLE_ORDER

        names = [n for n in TABLE_ORDER if n.startswith("rom") or n.startswith("drom")]
        lv = self.g.head_sublayers()[hl]
        return sum(self.g.table_position(n)[2] for n in names if self.g.table_position(n)[0] == lv) == \
            len(self.g.vheads_at(lv))

    def _buffer(self, kind: int, i: int, shape, typestr: str):
        torch = _torch()
        p, n = C.c_void_p(), C.c_size_t()
        check(lib().qx_buffer(self.h, C.c_int32(kind), C.c_int32(i), C.byref(p), C.byref(n)),
              "qx_buffer")
        return torch.as_tensor(_DevArray(p.value, shape, typestr), device=self.dev)

    def __del__(self):
        h = getattr(self, "h", None)
        if h is not None and _lib is not None:
            _lib.qx_destroy(h)
            self.h = None

    def _stream(self):
        torch = _torch()
        return C.c_void_p(torch.cuda.current_stream(self.dev).cuda_stream)

    # ---- Executor2 surface -----------------------------------------------------------------
    def load_init(self, row: int = 0):
        """The heads' initial states of the live graph (the snapshot it now holds) into batch
        row ``row`` (tritonexec.py:246-258).  Needs the executor built from a live graph."""
        torch = _torch()
        if self.c is None or isinstance(self.c, (str, Path, graphfile.GraphData)):
            raise QxError("load_init reads the live graph's Head.init; use load_machines instead")
        bufs = snapshot_states(self.c, [st["level"] for st in self.steps if st["kind"] == "head"])
        for st, buf in zip([st for st in self.steps if st["kind"] == "head"], bufs):
            st["S"][row].copy_(torch.from_numpy(buf))

    def reset(self, rows=None):
        """Fresh lag histories for the rows (tritonexec.py:260-263)."""
        if rows is None:
            check(lib().qx_reset(self.h, 0, self.B, self._stream()), "qx_reset")
            return
        for r in ([rows] if isinstance(rows, int) else list(rows)):
            check(lib().qx_reset(self.h, int(r), 1, self._stream()), "qx_reset")

    def embed(self, toks):
        """[n, D] fp32 embeddings on the device (tritonexec.py:265-270)."""
        torch = _torch()
        return torch.from_numpy(self.g.embed([int(t) for t in toks])).to(self.dev)

    def step(self, x):
        """One position for every row: x [B, D] fp32 (the embeddings in) becomes the residual
        after every node, in place (tritonexec.py:272-289)."""
        assert x.dtype == _torch().float32 and x.is_contiguous() and tuple(x.shape) == (self.B, self.D)
        check(lib().qx_step(self.h, C.c_void_p(x.data_ptr()), self._stream()), "qx_step")
        return x

    # ---- machine images / state ------------------------------------------------------------
    def load_machines(self, row0: int, programs, states=None) -> None:
        """core.snapshot + load_init of program images into rows row0.. (on the device): fresh
        programs, or (``states``: one (x, anchor, n, ram) per program) machines in those states."""
        keep: list = []
        if states is None:
            imgs = (Machine * len(programs))(*[program_image(p, keep) for p in programs])
        else:
            imgs = (Machine * len(programs))(*[state_image(p, *st, keep) for p, st in zip(programs, states)])
        check(lib().qx_load_machines(self.h, C.c_int32(row0), C.c_int32(len(programs)), imgs,
                                     self._stream()), "qx_load_machines")

    def readback(self, row: int) -> State:
        st = State()
        check(lib().qx_readback(self.h, C.c_int32(row), C.byref(st), self._stream()), "qx_readback")
        return st

    def checksums(self):
        """[B] uint64 (as int64 tensor) FNV-1a 64 state checksums, on the device."""
        torch = _torch()
        out = torch.empty(self.B, dtype=torch.int64, device=self.dev)
        check(lib().qx_checksums(self.h, C.c_void_p(out.data_ptr()), self._stream()), "qx_checksums")
        return out

    def errors(self) -> int:
        v = C.c_uint32()
        check(lib().qx_errors(self.h, C.byref(v), self._stream()), "qx_errors")
        return int(v.value)

    # ---- free running ----------------------------------------------------------------------
    def set_tokens(self, row0: int, toks) -> None:
        t = np.ascontiguousarray(np.asarray(toks, np.int32))
        check(lib().qx_set_tokens(self.h, C.c_int32(row0), C.c_int32(len(t)),
                                  t.ctypes.data_as(C.POINTER(C.c_int32)), self._stream()),
              "qx_set_tokens")

    def run(self, n_tokens: int, tokens=None) -> None:
        """n_tokens free-running steps of every row (tokens: a [n_tokens, B] int32 CUDA tensor
        receiving the generated ids, or None)."""
        p = C.c_void_p(0 if tokens is None else tokens.data_ptr())
        if tokens is not None:
            assert tokens.dtype == _torch().int32 and tuple(tokens.shape) == (n_tokens, self.B)
        check(lib().qx_run(self.h, C.c_int32(n_tokens), p, self._stream()), "qx_run")


class FreeRun:
    """FreeRun's surface (fastexec.py:236-340): every predicted token is the next input; the
    decode and the next embedding run inside the executor's kernel."""

    def __init__(self, c=None, batch: int = 1, device="cuda"):
        self.ex = Executor(c, batch, device)
        self.B = batch

    def load(self, row: int, first_token: int):
        """Row ``row`` starts from the graph's current snapshot, then ``first_token``."""
        self.ex.load_init(row)
        self.ex.reset([row])
        self.ex.set_tokens(row, [first_token])

    def load_program(self, row: int, prog, first_token: int):
        self.ex.load_machines(row, [prog])
        self.ex.reset([row])
        self.ex.set_tokens(row, [first_token])

    def run(self, n_steps: int) -> np.ndarray:
        """[B, n_steps] generated tokens."""
        torch = _torch()
        out = torch.zeros(n_steps, self.B, dtype=torch.int32, device=self.ex.dev)
        self.ex.run(n_steps, out)
        torch.cuda.synchronize(self.ex.dev)
        return out.cpu().numpy().T.astype(np.int64)


def gdn_check_args(S, q, k, v, alpha, beta, o=None, work=None) -> int:
    """Validates the tensors of one gated delta-rule step and returns BH: S [BH, 128, 128], q / k /
    v (and o) [BH, 128], alpha / beta [BH], all fp32, contiguous, on S's CUDA device; work, when
    given, a byte buffer of at least qx_gdn_work_bytes(BH).  Raises before anything is launched."""
    import torch

    if S.dim() != 3 or tuple(S.shape[1:]) != (HD, HD):
        raise ValueError(f"gdn_step: S must be [BH, {HD}, {HD}], got {tuple(S.shape)}")
    BH = int(S.shape[0])
    want = {"q": (q, (BH, HD)), "k": (k, (BH, HD)), "v": (v, (BH, HD)), "alpha": (alpha, (BH,)),
            "beta": (beta, (BH,))}
    if o is not None:
        want["o"] = (o, (BH, HD))
    every = {"S": (S, tuple(S.shape)), **want}
    for name, (t, shape) in every.items():
        if tuple(t.shape) != shape:
            raise ValueError(f"gdn_step: {name} must be {list(shape)}, got {list(t.shape)}")
        if t.dtype != torch.float32 or not t.is_contiguous():
            raise ValueError(f"gdn_step: {name} must be contiguous float32")
    for name, (t, _) in every.items():
        if t.device != S.device or t.device.type != "cuda":
            raise ValueError(f"gdn_step: {name} must be on S's CUDA device ({S.device}), got {t.device}")
    if work is not None:
        need = 8 + 4 * BH  # qx_gdn_work_bytes: count, error word, one index per head
        if work.device != S.device or not work.is_contiguous() or work.numel() * work.element_size() < need:
            raise ValueError(f"gdn_step: work must be a contiguous buffer of >= {need} bytes on {S.device}")
    return BH


def gdn_step(S, q, k, v, alpha, beta, o=None, work=None):
    """One gated delta-rule decode step on [BH, 128, 128] fp32 states (in place); returns o.
    The step's error word is work[1] (uint32; see gdn_error)."""
    torch = _torch()
    BH = gdn_check_args(S, q, k, v, alpha, beta, o, work)
    with torch.cuda.device(S.device):
        if o is None:
            o = torch.empty(BH, HD, device=S.device)
        if work is None:
            work = torch.empty(int(lib().qx_gdn_work_bytes(BH)), dtype=torch.uint8, device=S.device)
        stream = C.c_void_p(torch.cuda.current_stream(S.device).cuda_stream)
        check(lib().qx_gdn_step(C.c_int64(BH), *[C.c_void_p(t.data_ptr()) for t in (S, q, k, v, alpha, beta, o, work)],
                                stream), "qx_gdn_step")
    return o


def gdn_error(work) -> int:
    """The error word of the last step run with this work buffer (synchronises): 0, or
    QX_ERR_DEVICE_FLAG (5) when a bounded wait of the full-matrix path gave up (the states of
    that step are then undefined)."""
    return int(work[4:8].cpu().numpy().view(np.uint32)[0])
