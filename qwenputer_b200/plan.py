"""Plan compiler: a compiled graph (graphfile.GraphData) -> the per-token program of the CUDA
executor (the blob format of include/qx.h).

The reference lowers each sublayer into CSR tables once and launches one Triton kernel per
sublayer and machine (ERV/chipformer/rv/tritonexec.py:176-244, 272-289).  This compiler instead
produces one program that a persistent CTA runs for 32 machines at a time (one per lane), with
the residual stream of those machines resident in shared memory:

* residual slots: every dim gets an X row only over its live range (birth .. last use), so the
  2,679 dims fit in ~1,400 rows; rows are 33 floats (32 lanes + 1 pad: conflict-free whether a
  warp walks machines or rows);
* linear forms: the non-constant part of every projection is deduplicated per phase group and
  evaluated once into a scratch row; the constant part (the ONE dim's coefficient) is applied
  where the form is used (``F + c * x0``), so units that differ only in their threshold share
  a form;
* key heads: the terms every channel of a key head shares (its head-select literals) form one
  "common" form per head; the per-channel remainders are shared across heads (the row-address
  literals of the RAM, ROM and DROM heads), cutting the head projections ~6x;
* lag history: only (lag, dim) pairs the heads read are kept, staged into scratch rows at the
  start of their head sublayer (the ``_lag_load`` of tritonexec.py:74-79);
* dims both written and read inside one sublayer (``into`` outputs) are accumulated into a
  temporary row and added at the sublayer's end, so every read sees the sublayer's input, as
  the reference's separate output buffer guarantees (tritonexec.py:151-170).

Form, unit and key-head work is serialised into one stream of 16-byte quads, split into
contiguous per-warp ranges balanced at compile time (longest first); the kernel streams each
warp's range through shared memory with asynchronous copies.

Stream records (all fields little-endian uint32; "row" fields are shared-memory byte offsets,
row * 132, so the kernel adds them to its lane's base; the row after the last one is kept at
zero and stands for "no form"):
  form      [dst, n entry quads, 0, 0] + entry quads of two entries [row, w, row, w] (fp32 w)
  FFN node  [out, n groups, n quads, 0] + per group of units sharing their (a, b) forms:
              constant a: [a, b, n, 0] + (n + 1) / 2 quads [k, cb, k, cb], k = coef * ca, each
                          unit k x0 relu(F[b] + cb x0) (a padding unit has k = 0)
              a form:     [a, b, n | 1 << 31, 0] + n quads [coef, ca, cb, 0], each unit
                          coef (F[a] + ca x0) relu(F[b] + cb x0)
            (a node may be split into several records that add into the same row)
  key head  [slot | qhot << 16, k common, q common, nk | nq << 16], [k lag-ONE row, q lag-ONE
            row, 0, 0], then nk key-channel quads and nq query-channel quads
            [row | exists << 31, c0, c1, 0]: channel = relu(F[row] + (exists ? F[common] : 0)
            + c0 x0 + c1 x0(t - lag))
"""

from __future__ import annotations

import collections
import heapq
import struct
from collections import defaultdict

import numpy as np

from .graphfile import HD, ONE, GraphData

NONE = 0xFFFF
NONE32 = 0xFFFFFFFF
ROW_PAD = 33
MAGIC = 0x314E414C50585151
VERSION = 18
# machines one CTA runs (its group): 32 (a lane per machine) or, for few machines per GPU, 16, 8
# or 4 -- then a warp's lanes are WAYS = 32 / group record slots of `group` machines each, and the
# stream of a phase comes in lines of WAYS quads (one per slot) whose records the plan compiler
# pads to a common shape (bundles); a residual row is group + 1 floats
GROUPS = (32, 16, 8, 4)
NW_DEFAULT = 16
RING_QUADS = 32  # quads per half of a warp's stream ring
PH = dict(ZERO=1, LOADX=2, STAGE=3, FORMS=4, UNITS=5, KSEL=6, VH=7, APPLY=8, WRITEOUT=9,
          DECODE=10, END=11, VHRUN=12, VHSUM=13, MMA=14)
NOSYNC = 0x100  # phase kind flag: no barrier after the phase
# stream pieces: a header quad [x, y, z, n | flags << 24] and n <= PIECE_MAX - 1 body quads, never
# crossing a ring chunk of RING_QUADS quads (counted from the warp's range start); a record longer
# than a piece continues in the next pieces of the same warp.  In a bundled plan (group < 32) the
# same holds for lines of WAYS quads: a piece is a header line and n body lines, a ring chunk
# RING_QUADS lines; R_NOP marks a padding record of a bundle (it stores nothing), R_SPLIT a bundle
# that is one long form pair split over the record slots (line j holds its terms j * WAYS ..
# j * WAYS + WAYS - 1; the slots' partial sums meet in a warp reduction, slot 0 stores)
PIECE_MAX = 16
R_FIRST, R_LAST, R_STORE, R_QUERY, R_MERGE, R_NOP, R_SPLIT, R_SKIP = 1, 2, 4, 8, 0x10, 0x20, 0x40, 0x80
# form pairs of a bundled plan at least this long are split over the record slots
FORM_SPLIT_MIN = {1: 1 << 30, 2: 24, 4: 24, 8: 24}
# value heads a VH phase lists: its worklist of (value head, machine) records, 8 bytes each,
# lives in the stream rings (NW x 2 x RING_QUADS x 16 bytes = 2048 records for 16 warps); with a
# cluster the rings also hold the CTA's output deltas (one row per output row of the phase)
VH_CHUNK = 64
DELTA_ROWS = 128  # output rows one value-head phase may sum into (the group's delta buffer)
UNIT_CHUNK = 64  # FFN nodes with more units are split into records of at most this many
# key / query records of a cluster plan are split into parts of at most this many channels (by
# cluster size), each on its own warp; the parts merge into the slots with atomic maxima of
# packed selection words (a positive channel's value bits above bit 7, 127 - channel below)
KSEL_PART = {1: 128, 2: 64, 3: 48, 4: 32, 5: 32, 6: 24, 7: 24, 8: 16}
# the same for bundled plans, by record slots a warp (WAYS): the key-select phase of a group
# spreads over more slots when each part is shorter
KSEL_PART_WAYS = {1: 128, 2: 64, 4: 16, 8: 16}
# FFN nodes of a bundled plan split into records of at most this many units
UNIT_CHUNK_WAYS = {1: 64, 2: 64, 4: 32, 8: 32}
SEC = ["RUN_PROG", "STEP_PROG", "ROWS", "PAIRS", "STREAM", "VHSUM_ROWS", "WARP_PTR", "STAGES",
       "VHEADS", "VFORM", "ZFORM", "OUT_ROW", "OUT_W", "HL_V", "HL_NE", "FAM_ROW", "PAY_ROW",
       "FEAT_ROW", "FAM_IDS", "FAM_SIZE", "FAM_ROW0", "EMB_BASE", "EMB_BITS", "EMB_TABLE",
       "TABLES", "REG_COLS", "FAM_TOUCH_PTR", "FAM_TOUCH", "MMA_PHASES", "MMA_TILES", "TILEDATA",
       "FEAT_DIM", "CODE_ROW", "TEXT_WORDS", "TEXT_BASE", "TEXT_BITS", "PRINTABLE", "TEXT_TOUCH",
       "MERGED_INFO"]
N_SEC = 48  # section slots in the header
TABLE_ORDER = (["pc", "count", "j", "vcnt", "regs.rs1", "regs.rs2", "regs.rd"]
               + [f"quo{i}" for i in range(4)] + [f"rom{i}" for i in range(32)]
               + [f"drom{i}" for i in range(16)] + [f"bn1.{i}" for i in range(4)]
               + [f"bn2.{i}" for i in range(4)] + [f"ram{i}" for i in range(32)])
SMEM_MAX = 232448  # dynamic shared memory one B200 CTA may opt into (227 KB)
# bundled plans: shared memory for plan tables the token loop reads (the running phase program,
# the warp ranges, value heads, zero-row lists, delta-sum rows, lag stages: those that fit, in
# that order), by group: as much as leaves the plan its fewest phases
TABLE_BYTES = {32: 0, 16: 24576, 8: 36864, 4: 24576}
# tensor-core form phases (PH["MMA"]): F[form, machine] = sum W[form, k] X[k, machine] on tcgen05
# as M = 128 forms (a form block) x N = 32 machines x K = 16 source rows (a K block) tiles, bf16
# operands (every weight and every value a form reads is bf16-exact) and fp32 accumulators in
# tensor memory; the phase's source rows are staged as bf16 into the stream rings (1 KB per K
# block, so at most MMA_MAX_KB), the accumulators of at most MMA_MAX_FB form blocks live in
# tensor-memory columns [0, 256)
MMA_M, MMA_K = 128, 16
MMA_MAX_KB = 16
MMA_MAX_FB = 8
FLAG_MMA = 1  # header flag: the plan has tensor-core form phases
FLAG_MERGED = 2  # header flag: merged readout (code-dim signs, text tokens; MERGED_INFO)
# header flag: value-head outputs add straight into the residual rows (shared-memory reductions;
# plans of one CTA a group): OUT_ROW / out4 hold residual rows and no VHSUM phase exists
FLAG_DIRECT_OUT = 4
DEFERRED = 0x80000000  # FEAT_ROW flag: the feature is loaded where it is first used (low bits: dim)

DT = {
    "phase": np.dtype([("kind", "<u4"), ("a", "<u4"), ("b", "<u4"), ("c", "<u4")]),
    "stage": np.dtype([("e", "<u4"), ("x_row", "<u4"), ("ml", "<u4"), ("s0", "<u4"),
                       ("s1", "<u4"), ("s2", "<u4")]),
    "vhead": np.dtype([("hl", "<u4"), ("vh", "<u4"), ("col", "<u4"), ("slot", "<u2"),
                       ("nrows", "<u2"), ("a_row", "<u4"), ("b_row", "<u4"), ("ca", "<f4"),
                       ("cb", "<f4"), ("bconst", "<f4"), ("nout", "<u4"), ("out4", "<u4", (4,))]),
    "colform": np.dtype([("row", "<u4"), ("pad", "<u2"), ("live", "<u2"), ("c", "<f4")]),
    "mma": np.dtype([("n_kb", "<u4"), ("kr0", "<u4"), ("n_fb", "<u4"), ("dst0", "<u4"), ("t0", "<u4"),
                     ("t1", "<u4"), ("pad0", "<u4"), ("pad1", "<u4")]),
    "tile": np.dtype([("data", "<u4"), ("fb", "<u4"), ("kb", "<u4"), ("acc", "<u4")]),
}
HEADER = struct.Struct("<QII" + "I" * 18 + "48Q48Q")


def row_pad(group: int) -> int:
    """Floats per residual row: the group's machines plus one (conflict-free both when lanes walk
    machines and when they walk rows)."""
    return group + 1


def smem_extra_bytes(ksel_slots: int, qhot: int, nw: int, group: int = 32) -> int:
    """Shared memory after the rows: the zero row, key-select slots, the decode area, a counter
    block and the per-warp stream rings (two halves of RING_QUADS lines of 32 / group quads)."""
    return (row_pad(group) * 4 + ksel_slots * 32 * (1 + qhot) * 4 + 32 * 18 * 4 + 64 + 16
            + nw * 2 * RING_QUADS * 16 * (32 // group) + TABLE_BYTES[group])


def _bf16_bits(w: float) -> int:
    u = int(np.float32(w).view(np.uint32))
    if u & 0xFFFF:
        raise ValueError(f"weight {w!r} is not exact in bf16; the packed form format needs it")
    return u >> 16


def _fbits(x: float) -> int:
    return int(np.float32(x).view(np.uint32))


def split_form(forms, i: int, D: int) -> tuple[tuple, float]:
    """(non-constant terms, constant) of form i: the constant is the coefficient of ONE at
    lag 0 (x0 = 1 on every chip token); lagged ONE terms stay terms."""
    idx, w = forms.row(i)
    const = 0.0
    terms = []
    for k, v in zip(idx.tolist(), w.tolist()):
        lag, d = divmod(k, D)
        if lag == 0 and d == ONE:
            const += v
        else:
            terms.append(((lag, d), v))
    return tuple(sorted(terms)), float(np.float32(const))


class RowsExhausted(AssertionError):
    """The residual slots do not leave enough scratch rows in shared memory."""


class Plan:
    """The compiled program (numpy arrays per section) and its statistics."""

    def __init__(self):
        self.sec: dict[str, np.ndarray] = {}
        self.hdr: dict[str, int] = {}
        self.stats: dict = {}

    def blob(self) -> bytes:
        offs, cnts, parts = [0] * N_SEC, [0] * N_SEC, []
        pos = (HEADER.size + 255) // 256 * 256
        for i, name in enumerate(SEC):
            a = np.ascontiguousarray(self.sec[name])
            offs[i], cnts[i] = pos, len(a)
            b = a.tobytes()
            parts.append((pos, b))
            pos = (pos + len(b) + 255) // 256 * 256
        h = self.hdr
        head = HEADER.pack(MAGIC, VERSION, h["D"], h["n_slots"], h["n_scratch"], h["nw"],
                           h["n_head_levels"], h["one_row"], h["n_ksel_slots"], h["qhot_max"],
                           h["n_fam"], h["n_pay"], h["n_feat"], h["n_emb_rows"], h["n_families"],
                           h["vocab"], h["n_born0"], h["cluster"], h.get("flags", 0),
                           h.get("group", 32), h.get("table_bytes", 0), *offs, *cnts)
        out = bytearray(pos)
        out[:len(head)] = head
        for p, b in parts:
            out[p:p + len(b)] = b
        return bytes(out)


def compile_plan(g: GraphData, smem_rows: int | None = None, nw: int = NW_DEFAULT,
                 ksel_slots: int | None = None, cluster: int = 1, tc: bool = False,
                 defer: bool | None = None, ksel_part: int | None = None, group: int = 32) -> Plan:
    """The phase program and stream of the graph, for CTAs of ``nw`` warps; one group of 32
    machines runs on a cluster of ``cluster`` CTAs, so stream records are balanced over
    nw * cluster warps.  ``tc``: linear forms run as tensor-core phases (tcgen05) instead of
    stream records on the CUDA cores (every CTA of a cluster then computes all of them).
    ``group`` < 32: one CTA runs that many machines and a warp WAYS = 32 / group records side by
    side (bundles of records padded to one shape, lines of WAYS quads); no cluster, no tensor cores.
    ``defer`` (default: merged graphs): a token feature gets its row only from the sublayer that
    first uses it, loaded there from the executor's x (where the decode writes it), so that the
    rows of features used late are free before; ``ksel_slots`` (default 16, fewer when the rows
    do not fit otherwise): key heads one key-select phase serves; ``ksel_part`` (default by
    cluster size, KSEL_PART, or by record slots, KSEL_PART_WAYS): channels per part of a key or
    query record."""
    if defer is None:
        defer = g.merged
    if ksel_slots is None:
        for k in (16, 12, 8):
            try:
                return compile_plan(g, smem_rows, nw, k, cluster, tc, defer, ksel_part, group)
            except RowsExhausted:
                if k == 8:
                    raise
    assert 1 <= cluster <= 8, cluster
    assert group in GROUPS, group
    ways = 32 // group
    assert ways == 1 or (cluster == 1 and not tc), "bundled plans run on one CTA, on the CUDA cores"
    if ksel_part is None:
        ksel_part = KSEL_PART[cluster] if ways == 1 else KSEL_PART_WAYS[ways]
    assert 1 <= ksel_part <= 128
    unit_chunk = UNIT_CHUNK if ways == 1 else UNIT_CHUNK_WAYS[ways]
    # value-head outputs: straight into the residual rows on one CTA, through L2 delta rows on a
    # cluster (whose copies each fold them in)
    direct_out = cluster == 1
    # the kernel takes the ONE dim as 1 on every machine: no sublayer may write it
    assert ONE not in set(int(d) for d in g.ffn_out) and ONE not in set(int(d) for d in g.out_dim)
    ring_bytes = nw * 2 * RING_QUADS * 16 * ways
    qhot = int(g.head_qhot.max())
    assert qhot <= 4, "queries may read at most 4 rows"
    rp = row_pad(group)
    if smem_rows is None:
        smem_rows = (SMEM_MAX - smem_extra_bytes(ksel_slots, qhot, nw, group)) // (rp * 4)
    D = g.D
    levels = [int(x) for x in g.levels]
    kinds = [int(k) for k in g.level_kind]
    head_levels = [lv for lv, k in zip(levels, kinds) if k == 1]
    hl_index = {lv: i for i, lv in enumerate(head_levels)}
    INF = 10 ** 9
    stats = defaultdict(float)

    # ---- per level: forms (non-constant parts + constants), reads, writes ---------------------
    ffn_nodes = defaultdict(list)
    for n in range(len(g.ffn_level)):
        ffn_nodes[int(g.ffn_level[n])].append(n)
    unit_a = [split_form(g.unit_a, u, D) for u in range(g.unit_a.n)]
    unit_b = [split_form(g.unit_b, u, D) for u in range(g.unit_b.n)]
    qf = [split_form(g.q_forms, i, D) for i in range(g.q_forms.n)]
    kf = [split_form(g.k_forms, i, D) for i in range(g.k_forms.n)]
    vf = [split_form(g.v_forms, i, D) for i in range(g.v_forms.n)]
    zf = [split_form(g.z_forms, i, D) for i in range(g.z_forms.n)]
    af = [split_form(g.vh_a, i, D) for i in range(g.vh_a.n)]
    bf = [split_form(g.vh_beta, i, D) for i in range(g.vh_beta.n)]

    reads = defaultdict(set)  # level -> {(lag, dim)}
    writes = defaultdict(set)  # level -> {dim}
    for lv in levels:
        for n in ffn_nodes.get(lv, []):
            writes[lv].add(int(g.ffn_out[n]))
            for u in range(int(g.ffn_uptr[n]), int(g.ffn_uptr[n + 1])):
                for t, _ in unit_a[u][0] + unit_b[u][0]:
                    reads[lv].add(t)
        for h in g.heads_at(lv):
            for c in range(HD):
                for tab, fs in ((g.head_q, qf), (g.head_k, kf)):
                    if tab[h, c] >= 0:
                        for t, _ in fs[tab[h, c]][0]:
                            reads[lv].add(t)
            for j in g.vheads_of(h):
                for c in range(HD):
                    for tab, fs in ((g.vh_v, vf), (g.vh_z, zf)):
                        if tab[j, c] >= 0:
                            for t, _ in fs[tab[j, c]][0]:
                                reads[lv].add(t)
                for t, _ in af[j][0] + bf[j][0]:
                    reads[lv].add(t)
                for e in range(int(g.vh_out_ptr[j]), int(g.vh_out_ptr[j + 1])):
                    writes[lv].add(int(g.out_dim[e]))

    # ---- liveness and residual slots ----------------------------------------------------------
    feat = [int(d) for d in g.feat_dims]
    birth, last = {}, {}
    for d in feat:
        birth[d] = 0
        last[d] = 0
    for lv in levels:
        for d in writes[lv]:
            birth[d] = min(birth.get(d, INF), lv)
            last[d] = max(last.get(d, 0), lv)
    for lv in levels:
        for lag, d in reads[lv]:
            # a dim read before its first write holds its input value (0) until then
            birth[d] = min(birth.get(d, INF), lv)
            last[d] = max(last.get(d, 0), lv)
    for d in list(g.fam_dims) + list(g.pay_dims) + [int(x) for x in g.code_dims] + [ONE]:
        birth.setdefault(int(d), 0)
        last[int(d)] = INF
    deferred = set()
    if defer:
        # a feature's first use (a read, or a write that adds to its input value) decides where
        # it is loaded; features first used by the first sublayer stay born with the token
        first_use = {}
        for lv in levels:
            for d in writes[lv] | {dd for _, dd in reads[lv]}:
                first_use.setdefault(d, lv)
        for d in feat:
            if d != ONE and d in first_use and first_use[d] > levels[0]:
                birth[d] = first_use[d]
                deferred.add(d)
    last_write = {}
    for lv in levels:
        for d in writes[lv]:
            last_write[d] = lv
    temps = {}  # (level, dim) -> pseudo id of its temporary row
    for lv in levels:
        for d in sorted(writes[lv] & {dd for lag, dd in reads[lv] if lag == 0}):
            key = ("T", lv, d)
            temps[(lv, d)] = key
            birth[key] = lv
            last[key] = lv
    items = sorted(birth, key=lambda k: (birth[k], str(k)))
    slot = {}
    free: list[int] = []
    active: list[tuple[int, int]] = []
    n_slots = 0
    for k in items:
        b = birth[k]
        while active and active[0][0] < b:
            _, s = heapq.heappop(active)
            heapq.heappush(free, s)
        if free:
            s = heapq.heappop(free)
        else:
            s, n_slots = n_slots, n_slots + 1
        slot[k] = s
        heapq.heappush(active, (last[k], s))
    n_scratch = smem_rows - n_slots
    if n_scratch < 64:
        raise RowsExhausted(f"{n_slots} residual slots leave too little scratch")
    occupied = defaultdict(set)
    for k in items:
        for lv in levels:
            if birth[k] <= lv <= last[k]:
                occupied[lv].add(slot[k])
    free_rows = {lv: [r for r in range(smem_rows) if r not in occupied[lv]] for lv in levels}
    zero_row = smem_rows  # an extra row the kernel keeps at zero (reads of "no form")

    def W(r: int) -> int:
        """Shared-memory byte offset of a row (rows are row_pad(group) floats apart)."""
        return r * rp * 4

    ZW = W(zero_row)
    one_w = W(slot[ONE])

    # ---- builders -----------------------------------------------------------------------------
    rows_l: list[int] = []
    pairs_l: list[tuple[int, int]] = []
    stream: list[tuple[int, int, int, int]] = []
    warp_ptr_l: list[int] = []
    nnz_l: list[int] = []
    vhsum_l: list[int] = []  # residual rows (byte offsets) the cluster's output deltas add into
    stages_l, vheads_l, vform_l, zform_l, out_row_l, out_w_l = [], [], [], [], [], []

    def entry_quads(terms, rowmap) -> list[tuple]:
        ents = [(W(rowmap(t)), _fbits(w)) for t, w in terms]
        if len(ents) % 2:
            ents.append((ZW, 0))  # the zero row times +0
        return [(ents[i][0], ents[i][1], ents[i + 1][0], ents[i + 1][1]) for i in range(0, len(ents), 2)]

    def pack_terms(terms, rowmap) -> tuple[int, int]:
        """Packed entries of a lazily evaluated column form (NNZ array, 4-aligned)."""
        start = len(nnz_l)
        for q in entry_quads(terms, rowmap):
            nnz_l.extend(q)
        return start, (len(nnz_l) - start) // 4

    nwv = nw * cluster  # warps of a machine group: every warp of its cluster

    def balance(costs: list[float]) -> list[list[int]]:
        """Longest-first assignment of items to the group's nwv warps."""
        loads = [(0.0, w) for w in range(nwv)]
        heapq.heapify(loads)
        per = [[] for _ in range(nwv)]
        for i in sorted(range(len(costs)), key=lambda i: -costs[i]):
            ld, w = heapq.heappop(loads)
            per[w].append(i)
            heapq.heappush(loads, (ld + costs[i], w))
        tot = sum(costs)
        if tot:
            stats["imbalance_sum"] += max(l for l, _ in loads) - tot / nwv
            stats["balanced_sum"] += tot / nwv
        return per

    def pieces(x: int, y: int, z: int, body: list[tuple], flags: int = 0, step: int = 1) -> list[list[tuple]]:
        """A record as pieces of at most PIECE_MAX quads (header + body); `step`: body quads
        that must stay together.  The first piece carries R_FIRST, the last R_LAST."""
        out, i = [], 0
        cap = (PIECE_MAX - 1) // step * step
        npc = max(1, -(-len(body) // cap))
        cap = -(-len(body) // npc // step) * step or cap  # even pieces
        while True:
            part = body[i:i + cap]
            fl = flags | (R_FIRST if i == 0 else 0) | (R_LAST if i + cap >= len(body) else 0)
            out.append([(x, y, z, len(part) | fl << 24)] + part)
            i += cap
            if i >= len(body):
                return out

    def zip_lanes(lane_recs: list[list[list[tuple]]]) -> list[list[tuple]]:
        """WAYS records of one shape (pieces of equal lengths) as one bundle: its piece k holds,
        line by line, one quad of every record's piece k (record slot s = quad s of a line)."""
        out = []
        for k in range(len(lane_recs[0])):
            n = len(lane_recs[0][k])
            assert all(len(lr) == len(lane_recs[0]) and len(lr[k]) == n for lr in lane_recs)
            out.append([lr[k][j] for j in range(n) for lr in lane_recs])
        return out

    def stream_phase(kind: int, records: list[list[list[tuple]]], costs: list[float], prog, a=0, b=0):
        """Emit per-warp quad ranges of the records (each a list of pieces; in a bundled plan a
        record is a bundle of WAYS records) as one phase: a piece that would cross a ring chunk
        is moved to the next chunk behind an R_SKIP header line."""
        per = balance(costs)
        wp = len(warp_ptr_l)
        warp_ptr_l.append(len(stream))
        chunk = RING_QUADS * ways
        for w in range(nwv):
            start = len(stream)
            for i in per[w]:
                for pc in records[i]:
                    assert len(pc) <= PIECE_MAX * ways and len(pc) % ways == 0
                    room = chunk - (len(stream) - start) % chunk
                    if len(pc) > room:
                        stream.extend([(0, 0, 0, R_SKIP << 24)] * ways)
                        stream.extend([(0, 0, 0, 0)] * (room - ways))
                        stats["pad_quads"] += room
                    stream.extend(pc)
            warp_ptr_l.append(len(stream))
        prog.append((kind, a, b, wp))

    def bundles(items: list, shape) -> list[list]:
        """Items in bundles of WAYS, similar shapes together (one bundle per item when WAYS = 1,
        in the given order)."""
        if ways == 1:
            return [[it] for it in items]
        order = sorted(items, key=shape, reverse=True)
        return [order[i:i + ways] for i in range(0, len(order), ways)]

    def forms_phase(form_list: list[tuple], dst_rows: list[int], rowmap, prog):
        """Forms in pairs of similar length: pieces [dst A, dst B, 0, n | flags] + n quads
        [row, w of A, row, w of B] (the shorter padded with the zero row times +0), so a warp
        runs two independent sums; an odd last form pairs with an empty one into the zero row."""
        recs, costs = [], []
        items = sorted(zip(form_list, dst_rows), key=lambda fd: -len(fd[0]))
        prs = []
        for i in range(0, len(items), 2):
            ta, da = items[i]
            tb, db = items[i + 1] if i + 1 < len(items) else ((), None)
            ea = [(W(rowmap(t)), _fbits(w)) for t, w in ta]
            eb = [(W(rowmap(t)), _fbits(w)) for t, w in tb]
            prs.append((ea, eb, W(da), W(db) if db is not None else ZW))
            stats["form_nnz"] += len(ta) + len(tb)
        split = [pr for pr in prs if max(len(pr[0]), len(pr[1])) >= FORM_SPLIT_MIN[ways]]
        prs = [pr for pr in prs if max(len(pr[0]), len(pr[1])) < FORM_SPLIT_MIN[ways]]
        for ea, eb, xa, xb in split:
            # one pair over the WAYS slots: slot s takes terms s, s + WAYS, ... (zero-padded)
            n = -(-max(len(ea), len(eb)) // ways)
            ea = ea + [(ZW, 0)] * (n * ways - len(ea))
            eb = eb + [(ZW, 0)] * (n * ways - len(eb))
            lanes = [pieces(xa, xb, 0, [(ea[j * ways + k][0], ea[j * ways + k][1], eb[j * ways + k][0],
                                          eb[j * ways + k][1]) for j in range(n)], R_SPLIT)
                     for k in range(ways)]
            recs.append(zip_lanes(lanes))
            costs.append(4 * n + 14 * len(recs[-1]) + 12)
            stats["split_pairs"] += 1
        for bd in bundles(prs, lambda pr: max(len(pr[0]), len(pr[1]))):
            n = max(max(len(ea), len(eb)) for ea, eb, _, _ in bd)
            lanes = []
            for k in range(ways):
                # a bundle's padding record: zero-weight entries on the zero row, stores nothing
                ea, eb, xa, xb = bd[k] if k < len(bd) else ([], [], ZW, ZW)
                ea = ea + [(ZW, 0)] * (n - len(ea))
                eb = eb + [(ZW, 0)] * (n - len(eb))
                body = [(ea[j][0], ea[j][1], eb[j][0], eb[j][1]) for j in range(n)]
                lanes.append(pieces(xa, xb, 0, body, 0 if k < len(bd) else R_NOP))
            recs.append(lanes[0] if ways == 1 else zip_lanes(lanes))
            costs.append(4 * n + 14 * len(recs[-1]))
            stats["bundle_pad_quads"] += sum(n - max(len(ea), len(eb)) for ea, eb, _, _ in bd) + n * (ways - len(bd))
        stream_phase(PH["FORMS"], recs, costs, prog)

    mma_l: list[tuple] = []
    tiles_l: list[tuple] = []
    tiledata_l: list[np.ndarray] = []

    def bf16_exact(w: float) -> bool:
        return (int(np.float32(w).view(np.uint32)) & 0xFFFF) == 0

    def mma_phase(form_list: list[tuple], dst_rows: list[int], rowmap, prog) -> None:
        """Forms on the tensor cores: split (in the given order) into MMA phases of at most
        MMA_MAX_KB K blocks of source rows and MMA_MAX_FB form blocks; per phase its source rows
        (K blocks of MMA_K, padded with the zero row), the form blocks' destination rows (padded
        with NONE32), and one bf16 A tile [MMA_M forms x MMA_K rows] per occupied (form block,
        K block), the first tile of each form block starting its accumulator."""
        if not all(bf16_exact(w) for ft in form_list for _, w in ft):
            forms_phase(form_list, dst_rows, rowmap, prog)  # a weight bf16 cannot hold
            return
        subs, cur, cur_rows = [], [], set()
        for ft, dr in zip(form_list, dst_rows):
            rs = {rowmap(t) for t, _ in ft}
            if cur and (len(cur_rows | rs) > MMA_MAX_KB * MMA_K or len(cur) >= MMA_MAX_FB * MMA_M):
                subs.append(cur)
                cur, cur_rows = [], set()
            cur.append((ft, dr))
            cur_rows |= rs
        if cur:
            subs.append(cur)
        for sub in subs:
            src = sorted({rowmap(t) for ft, _ in sub for t, _ in ft})
            kidx = {r: i for i, r in enumerate(src)}
            n_kb = -(-len(src) // MMA_K)
            rows_l.extend([0] * (-len(rows_l) % 4))  # K blocks start 16-byte aligned (uint4 loads)
            kr0 = len(rows_l)
            rows_l.extend(W(r) for r in src)
            rows_l.extend([ZW] * (n_kb * MMA_K - len(src)))
            n_fb = -(-len(sub) // MMA_M)
            dst0 = len(rows_l)
            rows_l.extend(W(dr) for _, dr in sub)
            rows_l.extend([NONE32] * (n_fb * MMA_M - len(sub)))
            t0 = len(tiles_l)
            for fb in range(n_fb):
                blocks: dict[int, np.ndarray] = {}
                for i, (ft, _) in enumerate(sub[fb * MMA_M:(fb + 1) * MMA_M]):
                    for t, w in ft:
                        k = kidx[rowmap(t)]
                        tile = blocks.setdefault(k // MMA_K, np.zeros((MMA_M, MMA_K), np.uint16))
                        assert tile[i, k % MMA_K] == 0, "two terms of one form on one row"
                        tile[i, k % MMA_K] = _bf16_bits(w)
                for j, kb in enumerate(sorted(blocks)):
                    tiles_l.append((len(tiledata_l), fb, kb, 0 if j == 0 else 1))
                    tiledata_l.append(blocks[kb])
            mma_l.append((n_kb, kr0, n_fb, dst0, t0, len(tiles_l), 0, 0))
            prog.append((PH["MMA"], len(mma_l) - 1, 0, 0))
            stats["form_nnz"] += sum(len(ft) for ft, _ in sub)
            stats["mma_tiles"] += len(tiles_l) - t0
            stats["mma_phases"] += 1

    def run_forms(form_list, dst_rows, rowmap, prog) -> None:
        (mma_phase if tc else forms_phase)(form_list, dst_rows, rowmap, prog)

    def tc_order(forms: dict, rowmap) -> dict:
        """In tensor-core mode, forms ordered by their source rows (forms with like rows share
        A tiles; consecutive forms get consecutive destination rows); else as given."""
        if not tc:
            return forms
        order = sorted(forms, key=lambda f: tuple(sorted(rowmap(t) for t, _ in f)))
        return {f: i for i, f in enumerate(order)}

    def xrow(lv, d):
        return slot[temps[(lv, d)]] if (lv, d) in temps else slot[d]

    run_prog: list[tuple] = []
    step_prog: list[tuple] = []
    hl_ne = []
    group_stats = []

    born0 = sorted(k for k in birth if birth[k] == 0 and not isinstance(k, tuple))
    assert not pairs_l  # the run-mode prologue / epilogue are PAIRS[0 : n_born0]
    pairs_l.extend((W(slot[d]), d) for d in born0)
    step_prog.append((PH["LOADX"], 0, len(born0), 0))

    for lv, kind in zip(levels, kinds):
        born_all = sorted(d for d in birth if not isinstance(d, tuple) and birth[d] == lv and lv > 0)
        # deferred features born here are read by this sublayer's first phase: loaded (from x,
        # in both modes) behind a barrier of their own
        born_f = [d for d in born_all if d in deferred]
        born = [d for d in born_all if d not in deferred]
        if born_f:
            p0 = len(pairs_l)
            pairs_l.extend((W(slot[d]), d) for d in born_f)
            run_prog.append((PH["LOADX"], p0, len(born_f), 0))
            step_prog.append((PH["LOADX"], p0, len(born_f), 0))
            stats["deferred_loads"] += len(born_f)
        tmp = sorted(slot[k] for (l2, d), k in temps.items() if l2 == lv)
        r0 = len(rows_l)
        rows_l.extend(W(slot[d]) for d in born)
        rows_l.extend(W(t) for t in tmp)
        # newborn and temporary rows are neither read nor written by the sublayer's first phase
        # (a stage or form phase): their zeroing needs no barrier of its own
        if born or tmp:
            run_prog.append((PH["ZERO"] | NOSYNC, r0, len(born) + len(tmp), 0))
        if tmp:
            step_prog.append((PH["ZERO"] | NOSYNC, r0 + len(born), len(tmp), 0))
        if born:
            p0 = len(pairs_l)
            pairs_l.extend((W(slot[d]), d) for d in born)
            step_prog.append((PH["LOADX"] | NOSYNC, p0, len(born), 0))
        body: list[tuple] = []
        free = free_rows[lv]
        if kind == 0:
            # ---------- FFN sublayer: groups of nodes whose distinct forms fit the scratch ----
            nodes = ffn_nodes[lv]
            groups, cur, cur_forms = [], [], {}
            for n in nodes:
                nf = {}
                for u in range(int(g.ffn_uptr[n]), int(g.ffn_uptr[n + 1])):
                    for fm in (unit_a[u][0], unit_b[u][0]):
                        if fm:
                            nf[fm] = 1
                new = [f for f in nf if f not in cur_forms]
                if cur and len(cur_forms) + len(new) > len(free):
                    groups.append((cur, cur_forms))
                    cur, cur_forms = [], {}
                    new = list(nf)
                cur.append(n)
                for f in new:
                    cur_forms[f] = len(cur_forms)
            if cur:
                groups.append((cur, cur_forms))
            for gnodes, gforms in groups:
                assert len(gforms) <= len(free), f"sublayer {lv}: a node needs too many forms"
                gforms = tc_order(gforms, lambda t: slot[t[1]])
                flist = list(gforms)
                run_forms(flist, [free[i] for i in range(len(flist))], lambda t: slot[t[1]], body)
                frow = {f: W(free[i]) for f, i in gforms.items()}
                # units as flat quads (ONE is 1 for every machine: no sublayer writes it):
                #   constant a:  [F[b] row, k, cb, 0]          k = coef * ca rounded as the
                #                                               reference rounds coef * a
                #   a form a:    [F[a] row, F[b] row, coef, ca], [cb, 0, 0, 0]
                # a node's units go out as records of at most UNIT_CHUNK units (warps balance them)
                parts = []  # (out row, const quads, has-a quad pairs)
                for n in gnodes:
                    out = W(xrow(lv, int(g.ffn_out[n])))
                    cq, hq = [], []
                    for u in range(int(g.ffn_uptr[n]), int(g.ffn_uptr[n + 1])):
                        (ta, ca), (tb, cb) = unit_a[u], unit_b[u]
                        rb = frow[tb] if tb else ZW
                        cf = float(g.unit_coef[u])
                        if ta:
                            hq.append(((frow[ta], rb, _fbits(cf), _fbits(ca)), (_fbits(cb), 0, 0, 0)))
                        else:
                            cq.append((rb, _fbits(np.float32(cf) * np.float32(ca)), _fbits(cb), 0))
                    units_all = [("c", q) for q in cq] + [("h", q) for q in hq]
                    for c0 in range(0, max(len(units_all), 1), unit_chunk):
                        chunk = units_all[c0:c0 + unit_chunk]
                        parts.append((out, [q for k, q in chunk if k == "c"], [q for k, q in chunk if k == "h"]))
                    stats["units"] += int(g.ffn_uptr[n + 1] - g.ffn_uptr[n])
                    stats["unit_groups"] += 0
                # a row that only one record of the phase adds into is updated with a plain
                # read-add-store (R_STORE); rows several records meet take atomic adds
                nrec = collections.Counter(out for out, _, _ in parts)

                def unit_pieces(out, cq, hq, fl0):
                    body_q = cq + [q for pair in hq for q in pair]
                    pcs, i = [], 0
                    while True:
                        e = min(i + PIECE_MAX - 1, len(body_q))
                        if e > len(cq) and (e - len(cq)) % 2:
                            e -= 1  # a unit's two quads stay in one piece
                        nc = max(0, min(e, len(cq)) - i)
                        fl = fl0 | (R_FIRST if i == 0 else 0) | (R_LAST if e >= len(body_q) else 0)
                        pcs.append([(out, nc, 0, (e - i) | fl << 24)] + body_q[i:e])
                        i = e
                        if i >= len(body_q):
                            return pcs

                recs, costs = [], []
                # bundles share their pieces' shape: constant-gate units padded with k = 0 on the
                # zero row, units with an a form with coef = 0 (both add +0)
                for bd in bundles(parts, lambda pt: (len(pt[2]), len(pt[1]))):
                    ncq = max(len(cq) for _, cq, _ in bd)
                    nhq = max(len(hq) for _, _, hq in bd)
                    lanes = []
                    for k in range(ways):
                        out, cq, hq = bd[k] if k < len(bd) else (ZW, [], [])
                        fl0 = (R_STORE if nrec[out] == 1 else 0) if k < len(bd) else R_NOP
                        cq = cq + [(ZW, 0, 0, 0)] * (ncq - len(cq))
                        hq = hq + [((ZW, ZW, 0, 0), (0, 0, 0, 0))] * (nhq - len(hq))
                        lanes.append(unit_pieces(out, cq, hq, fl0))
                    recs.append(lanes[0] if ways == 1 else zip_lanes(lanes))
                    costs.append(4 * ncq + 9 * nhq + 12 * len(recs[-1]))
                    stats["bundle_pad_quads"] += sum(ncq - len(cq) + 2 * (nhq - len(hq)) for _, cq, hq in bd) + (ncq + 2 * nhq) * (ways - len(bd))
                stream_phase(PH["UNITS"], recs, costs, body)
            group_stats.append((lv, "ffn", len(groups)))
        else:
            # ---------- head sublayer ---------------------------------------------------------
            hi = hl_index[lv]
            lag_pairs = sorted({t for t in reads[lv] if t[0] > 0})
            # lagged ONE terms of key / query channels become per-channel constants times the
            # staged ONE: make sure those stage rows exist
            for h in g.heads_at(lv):
                for tab, fs in ((g.head_k, kf), (g.head_q, qf)):
                    for c in range(HD):
                        if tab[h, c] >= 0:
                            for (lag, d), _ in fs[tab[h, c]][0]:
                                if d == ONE and lag > 0 and (lag, ONE) not in lag_pairs:
                                    lag_pairs.append((lag, ONE))
            lag_pairs = sorted(set(lag_pairs))
            lag_dims = sorted({d for _, d in lag_pairs})
            stage_row = {t: free[i] for i, t in enumerate(lag_pairs)}
            hl_ne.append(len(lag_dims))
            if lag_dims:
                s0 = len(stages_l)
                for e, d in enumerate(lag_dims):
                    ml = max(lag for lag, dd in lag_pairs if dd == d)
                    st = [W(stage_row[(lag, d)]) if (lag, d) in stage_row else NONE32 for lag in (1, 2, 3)]
                    stages_l.append((e, W(slot[d]), ml, *st))
                body.append((PH["STAGE"], s0, len(lag_dims), hi))
            ffree = free[len(lag_pairs):]
            cap = len(ffree)

            def rowmap(t, lv=lv):
                return slot[t[1]] if t[0] == 0 else stage_row[t]

            def head_forms(h):
                """Per key / query: (common terms, lag of the lagged-ONE constant,
                {channel: (resid terms, c0, c1)}).  The common terms are those all (>= 4)
                channels of the head share; a lagged ONE term becomes the constant c1."""
                out = {}
                for nm, tab, fs in (("k", g.head_k, kf), ("q", g.head_q, qf)):
                    chans = {}
                    lags = set()
                    for c in range(HD):
                        if tab[h, c] < 0:
                            continue
                        t, c0 = fs[tab[h, c]]
                        ones = [(lag, w) for (lag, d), w in t if d == ONE and lag > 0]
                        assert len(ones) <= 1
                        c1 = ones[0][1] if ones else 0.0
                        if ones:
                            lags.add(ones[0][0])
                        chans[c] = (tuple(x for x in t if not (x[0][1] == ONE and x[0][0] > 0)), c0, c1)
                    assert len(lags) <= 1, "one lag of the ONE dim per head"
                    common = set()
                    if len(chans) >= 4:
                        common = set(next(iter(chans.values()))[0])
                        for t, _, _ in chans.values():
                            common &= set(t)
                    res = {c: (tuple(x for x in t if x not in common), c0, c1)
                           for c, (t, c0, c1) in chans.items()}
                    out[nm] = (tuple(sorted(common)), lags.pop() if lags else 0, res)
                return out

            heads = g.heads_at(lv)
            vhs_level = g.vheads_at(lv)
            hf = {h: head_forms(h) for h in heads}
            groups, cur, cur_forms = [], [], {}
            for h in heads:
                nf = {}
                for nm in ("k", "q"):
                    com, _, res = hf[h][nm]
                    if com:
                        nf[com] = 1
                    for t, _, _ in res.values():
                        if t:
                            nf[t] = 1
                for j in g.vheads_of(h):
                    for fs in (af, bf):
                        if fs[j][0]:
                            nf[fs[j][0]] = 1
                    for c in range(HD):
                        for tab, fs in ((g.vh_v, vf), (g.vh_z, zf)):
                            if tab[j, c] >= 0 and fs[tab[j, c]][0]:
                                nf[fs[tab[j, c]][0]] = 1
                new = [f for f in nf if f not in cur_forms]
                if cur and (len(cur_forms) + len(new) > cap or len(cur) >= ksel_slots):
                    groups.append((cur, cur_forms))
                    cur, cur_forms = [], {}
                    new = list(nf)
                cur.append(h)
                for f in new:
                    cur_forms[f] = len(cur_forms)
            if cur:
                groups.append((cur, cur_forms))
            for gheads, gforms in groups:
                assert len(gforms) <= cap, f"sublayer {lv}: a key head needs too many forms"
                gforms = tc_order(gforms, rowmap)
                flist = list(gforms)
                frow = {f: W(ffree[i]) for f, i in gforms.items()}
                if flist:
                    run_forms(flist, [ffree[i] for i in range(len(flist))], rowmap, body)
                # a key head is two records, on any warps: key pieces [slot | qhot << 16, common
                # row, lag-ONE row, n | flags] and query pieces (R_QUERY); channel quads [row, c0,
                # c1, 1.0 if the common form applies else 0]
                specs = []
                one_f = _fbits(1.0)
                for sl, h in enumerate(gheads):
                    for nm, qf_flag in (("k", 0), ("q", R_QUERY)):
                        com, lag, res = hf[h][nm]
                        com_row = frow[com] if com else ZW
                        one_row = W(stage_row[(lag, ONE)]) if lag else ZW
                        # channels past the last present one (zero rows, all weights 0) can
                        # never be selected or count as positive: they are not emitted
                        chans = []
                        if res:
                            for c in range(max(res) + 1):
                                if c in res:
                                    t, c0, c1 = res[c]
                                    chans.append((frow[t] if t else ZW, _fbits(c0), _fbits(c1), one_f if com else 0))
                                else:
                                    chans.append((ZW, 0, 0, 0))
                        # a record longer than ksel_part channels goes out as parts of even
                        # length (header x: slot | qhot << 16 | first channel << 24), each on
                        # any warp, merged into the slot (R_MERGE)
                        npart = max(1, -(-len(chans) // ksel_part))
                        plen = -(-len(chans) // npart) if chans else 0
                        for lo in range(0, max(len(chans), 1), max(plen, 1)):
                            part = chans[lo:lo + plen]
                            fl = qf_flag | (R_MERGE if npart > 1 else 0)
                            specs.append((sl | int(g.head_qhot[h]) << 16 | lo << 24, com_row, one_row, part, fl))
                        stats["kq_channels"] += len(chans)
                        stats["kq_parts"] += npart
                # bundles hold keys or queries only (their channel loops differ); padding
                # channels on the zero row never count as positive, padding records store nothing
                recs, costs = [], []
                kq_bundles = []
                if ways == 1:
                    kq_bundles = [[sp] for sp in specs]
                else:
                    for qk in (0, R_QUERY):
                        kq_bundles += bundles([sp for sp in specs if sp[4] & R_QUERY == qk], lambda sp: len(sp[3]))
                for bd in kq_bundles:
                    n = max(len(sp[3]) for sp in bd)
                    lanes = []
                    for k in range(ways):
                        x, com_row, one_row, part, fl = bd[k] if k < len(bd) else (
                            bd[0][0] & 0xFF0000, ZW, ZW, [], (bd[0][4] & R_QUERY) | R_NOP)
                        part = part + [(ZW, 0, 0, 0)] * (n - len(part))
                        lanes.append(pieces(x, com_row, one_row, part, fl))
                    recs.append(lanes[0] if ways == 1 else zip_lanes(lanes))
                    key = not bd[0][4] & R_QUERY
                    costs.append((12 if key else 18) * n + 12 * len(recs[-1])
                                 + (40 * cluster if bd[0][4] & R_MERGE else 0))
                    stats["bundle_pad_quads"] += sum(n - len(sp[3]) for sp in bd) + n * (ways - len(bd))
                stream_phase(PH["KSEL"], recs, costs, body)
                v0 = len(vheads_l)
                for sl, h in enumerate(gheads):
                    for j in g.vheads_of(h):
                        col = len(out_row_l)
                        for c in range(HD):
                            for tab, fs, dstl in ((g.vh_v, vf, vform_l), (g.vh_z, zf, zform_l)):
                                if tab[j, c] >= 0:
                                    t, cc = fs[tab[j, c]]
                                    dstl.append((frow[t] if t else ZW, 0, 1, cc))
                                else:
                                    dstl.append((ZW, 0, 0, 0.0))
                        orow = [NONE32] * HD
                        ow = [0.0] * HD
                        for e in range(int(g.vh_out_ptr[j]), int(g.vh_out_ptr[j + 1])):
                            c = int(g.out_col[e])
                            if float(g.out_w[e]) != 0.0:
                                orow[c] = W(xrow(lv, int(g.out_dim[e])))
                                ow[c] = float(g.out_w[e])
                        out_row_l.extend(orow)
                        out_w_l.extend(ow)
                        ta, ca = af[j]
                        tb, cb = bf[j]
                        vheads_l.append((hi, vhs_level.index(j), col, sl, int(g.vh_nrows[j]),
                                         frow[ta] if ta else ZW, frow[tb] if tb else ZW,
                                         ca, cb, 0.0 if g.vh_has_beta[j] else 1.0))
                # value-head outputs are summed into the group's delta rows in global memory
                # (one row per distinct output row of the phase, DELTA_ROWS at most, byte offset
                # j * 128: 32 machines x fp32) by L2 atomic adds; a VHSUM phase adds them into
                # the residual rows (of every copy, on a cluster)
                def fits(nh, nr):
                    return nh <= VH_CHUNK and nh * 32 * 8 <= ring_bytes and (direct_out or nr <= DELTA_ROWS)

                c0 = v0
                while c0 < len(vheads_l):
                    rows: list[int] = []
                    c1 = c0
                    while c1 < len(vheads_l):
                        col = vheads_l[c1][2]
                        new = [r for r in dict.fromkeys(out_row_l[col:col + HD]) if r != NONE32 and r not in rows]
                        if not fits(c1 - c0 + 1, len(rows) + len(new)):
                            break
                        rows += new
                        c1 += 1
                    assert c1 > c0, "one value head has more output rows than the delta buffer"
                    if direct_out:
                        # one CTA a group: the outputs add into the residual rows themselves
                        body.append((PH["VH"], c0, c1, 0))
                        body.append((PH["VHRUN"], c0, c1, 0))
                        c0 = c1
                        continue
                    dpos = {r: i * 128 for i, r in enumerate(rows)}
                    for v in range(c0, c1):
                        col = vheads_l[v][2]
                        for c in range(col, col + HD):
                            if out_row_l[c] != NONE32:
                                out_row_l[c] = dpos[out_row_l[c]]
                    body.append((PH["VH"], c0, c1, len(rows)))  # list the machines' row work
                    body.append((PH["VHRUN"], c0, c1, len(rows)))  # serve it
                    body.append((PH["VHSUM"], len(vhsum_l), len(rows), 0))
                    vhsum_l.extend(rows)
                    c0 = c1
            group_stats.append((lv, "head", len(groups)))
        apply_pairs = [(W(slot[d]), W(slot[k])) for (l2, d), k in temps.items() if l2 == lv]
        tail = []
        if apply_pairs:
            p0 = len(pairs_l)
            pairs_l.extend(apply_pairs)
            tail.append((PH["APPLY"], p0, len(apply_pairs), 0))
        run_prog += body + tail
        step_prog += body + tail
        wo = sorted(d for d, l2 in last_write.items() if l2 == lv)
        if wo:
            p0 = len(pairs_l)
            pairs_l.extend((W(slot[d]), d) for d in wo)
            step_prog.append((PH["WRITEOUT"], p0, len(wo), 0))
    run_prog.append((PH["DECODE"], 0, 0, 0))
    run_prog.append((PH["END"], 0, 0, 0))
    step_prog.append((PH["END"], 0, 0, 0))
    # tensor-core phases commit once per round of up to 16 tiles to one mbarrier: record per phase
    # the commits of a token before it (pad0) and a token's total (pad1), whose parities give the
    # barrier phase the kernel waits on (both programs run the same MMA phases in the same order)
    assert [p for p in run_prog if p[0] == PH["MMA"]] == [p for p in step_prog if p[0] == PH["MMA"]]
    # the key-select slots are read by the VH phase after their KSEL phase and cleared by the VH
    # serving phase after it, so every KSEL phase is followed by VH, then VHRUN, before the next
    for prog in (run_prog, step_prog):
        ks = [p[0] & 0xFF for p in prog if p[0] & 0xFF in (PH["KSEL"], PH["VH"], PH["VHRUN"])]
        assert all(ks[i:i + 3] == [PH["KSEL"], PH["VH"], PH["VHRUN"]] for i in range(0, len(ks), 3)), ks
    commits = 0
    for i, mp in enumerate(mma_l):
        mma_l[i] = mp[:6] + (commits, 0)
        commits += -(-(mp[5] - mp[4]) // 16)
    mma_l[:] = [mp[:7] + (commits,) for mp in mma_l]

    # ---- sections -----------------------------------------------------------------------------
    def arr(lst, dt):
        dt = DT[dt]
        a = np.zeros(max(1, len(lst)), dt)
        for i, v in enumerate(lst):
            a[i] = v
        return a

    P = Plan()
    s = P.sec
    s["RUN_PROG"] = arr(run_prog, "phase")
    s["STEP_PROG"] = arr(step_prog, "phase")
    s["ROWS"] = np.asarray(rows_l or [0], np.uint32)
    s["PAIRS"] = np.asarray(pairs_l or [(0, 0)], np.uint32).reshape(-1, 2)
    s["STREAM"] = np.asarray(stream or [(0, 0, 0, 0)], np.uint32).reshape(-1, 4)
    assert not nnz_l
    s["VHSUM_ROWS"] = np.asarray(vhsum_l or [0], np.uint32)
    s["WARP_PTR"] = np.asarray(warp_ptr_l or [0], np.uint32)
    s["STAGES"] = arr(stages_l, "stage")
    # value heads with at most 4 distinct output rows: OUT_ROW holds indices into out4, and the
    # kernel sums each row's columns across the warp before one add per row
    vh_full = []
    for v in vheads_l:
        col = v[2]
        rows = [r for r in dict.fromkeys(out_row_l[col:col + HD]) if r != NONE32]
        if len(rows) <= 4:
            for c in range(col, col + HD):
                if out_row_l[c] != NONE32:
                    out_row_l[c] = rows.index(out_row_l[c])
            vh_full.append(tuple(v) + (len(rows), tuple(rows + [0] * (4 - len(rows)))))
            stats["vh_out4"] += 1
        else:
            vh_full.append(tuple(v) + (0xFF, (0, 0, 0, 0)))
    s["VHEADS"] = arr(vh_full, "vhead")
    s["VFORM"] = arr(vform_l, "colform")
    s["ZFORM"] = arr(zform_l, "colform")
    s["OUT_ROW"] = np.asarray(out_row_l, np.uint32)
    s["OUT_W"] = np.asarray(out_w_l, np.float32)
    s["HL_V"] = np.asarray([len(g.vheads_at(lv)) for lv in head_levels], np.uint32)
    s["HL_NE"] = np.asarray([max(1, n) for n in hl_ne], np.uint32)
    s["FAM_ROW"] = np.asarray([W(slot[int(d)]) for d in g.fam_dims] or [0], np.uint32)
    s["PAY_ROW"] = np.asarray([W(slot[int(d)]) for d in g.pay_dims] or [0], np.uint32)
    s["FEAT_ROW"] = np.asarray([(DEFERRED | d) if d in deferred else W(slot[d]) for d in feat], np.uint32)
    s["FEAT_DIM"] = np.asarray(feat, np.uint32)
    # merged readout and text tokens
    merged = g.merged
    s["CODE_ROW"] = np.asarray([W(slot[int(d)]) for d in g.code_dims] or [0], np.uint32)
    s["TEXT_WORDS"] = np.ascontiguousarray(g.text_words if merged else np.zeros((1, 5), np.uint32)).reshape(-1)
    s["TEXT_BASE"] = np.asarray(g.text_base if merged else np.zeros(1), np.float32)
    s["TEXT_BITS"] = np.ascontiguousarray(g.text_bits if merged else np.zeros((1, 1)), np.float32).reshape(-1)
    s["PRINTABLE"] = np.asarray(g.printable if merged else [0], np.int32)
    if merged:
        tt = np.flatnonzero((np.asarray(g.text_base) != 0) | (np.asarray(g.text_bits) != 0).any(axis=0))
    else:
        tt = np.zeros(0, np.int64)
    s["TEXT_TOUCH"] = np.asarray(tt if len(tt) else [0], np.uint32)
    s["MERGED_INFO"] = np.asarray([int(g.q_fid[0]) if merged else 0, len(g.text_words) if merged else 0,
                                   len(g.printable) if merged else 0, len(tt), len(g.code_dims),
                                   g.text_bits.shape[0] if merged else 0, 0, 0], np.uint32)
    s["FAM_IDS"] = np.asarray(g.fam_ids, np.int32)
    s["FAM_SIZE"] = np.asarray(g.fam_size, np.int32)
    s["FAM_ROW0"] = np.asarray([int(r) if sm else -1 for r, sm in zip(g.fam_row0, g.fam_small)],
                               np.int32)
    s["EMB_BASE"] = np.ascontiguousarray(g.emb_base, np.float32).reshape(-1)
    s["EMB_BITS"] = np.ascontiguousarray(g.emb_bits, np.float32).reshape(-1)
    s["EMB_TABLE"] = np.ascontiguousarray(g.emb_table, np.float32).reshape(-1)
    tabs = []
    for name in TABLE_ORDER:
        lv, vh0, _ = g.table_position(name)
        tabs.append((hl_index[lv], vh0))
    s["TABLES"] = np.asarray(tabs, np.uint32).reshape(-1)
    s["REG_COLS"] = np.asarray(g.reg_cols, np.int32).reshape(-1)
    # per family built from payload bits: the feature indices its embeddings can make nonzero
    # (the base row's or any bit row's nonzeros); every other feature of such a token is 0
    eb = np.asarray(g.emb_bits, np.float32).reshape(len(g.fam_ids), -1, len(feat))
    ebase = np.asarray(g.emb_base, np.float32).reshape(len(g.fam_ids), len(feat))
    tptr, touch = [0], []
    for f in range(len(g.fam_ids)):
        nz = np.flatnonzero((ebase[f] != 0) | (eb[f] != 0).any(axis=0))
        touch.extend(int(x) for x in nz)
        tptr.append(len(touch))
    s["FAM_TOUCH_PTR"] = np.asarray(tptr, np.uint32)
    s["FAM_TOUCH"] = np.asarray(touch or [0], np.uint32)
    s["MMA_PHASES"] = arr(mma_l, "mma")
    s["MMA_TILES"] = arr(tiles_l, "tile")
    s["TILEDATA"] = (np.stack(tiledata_l).reshape(-1) if tiledata_l else np.zeros(MMA_M * MMA_K, np.uint16))
    P.hdr = dict(D=D, n_slots=n_slots, n_scratch=n_scratch, nw=nw, n_head_levels=len(head_levels),
                 one_row=one_w, n_ksel_slots=ksel_slots, qhot_max=qhot,
                 n_fam=len(g.fam_dims), n_pay=len(g.pay_dims), n_feat=len(feat),
                 n_emb_rows=int(g.emb_table.shape[0]), n_families=len(g.fam_ids),
                 vocab=int(g.vocab), n_born0=len(born0), cluster=cluster,
                 flags=(FLAG_MMA if mma_l else 0) | (FLAG_MERGED if merged else 0)
                 | (FLAG_DIRECT_OUT if direct_out else 0), group=group,
                 table_bytes=TABLE_BYTES[group])
    stats["n_slots"] = n_slots
    stats["ksel_slots"] = ksel_slots
    stats["deferred_features"] = len(deferred)
    stats["n_scratch"] = n_scratch
    stats["phases_run"] = len(run_prog)
    stats["barriers_run"] = sum(1 for k, *_ in run_prog if not k & NOSYNC and k != PH["END"])
    stats["stream_quads"] = len(stream)
    stats["weight_bytes"] = int(s["STREAM"].nbytes + s["STAGES"].nbytes + s["VHEADS"].nbytes
                                + s["RUN_PROG"].nbytes + s["WARP_PTR"].nbytes
                                + (s["TILEDATA"].nbytes + s["MMA_TILES"].nbytes + s["MMA_PHASES"].nbytes
                                   if mma_l else 0))
    stats["imbalance"] = (stats["imbalance_sum"] / stats["balanced_sum"]) if stats["balanced_sum"] else 0
    stats["groups"] = group_stats
    P.stats = dict(stats)
    P.slot = slot
    P.head_levels = head_levels
    P.lag_dims = {lv: sorted({d for lag, d in reads[lv] if lag > 0}) for lv in head_levels}
    return P
