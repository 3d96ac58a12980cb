"""The compiled-layer graph as a self-contained file.

The reference compiles its RV32IM machine into a ``chipformer.q35.ir.Graph`` (``ERV/chipformer/
q35/ir.py:121-244``; built by ``ERV/chipformer/rv/core.py:299-1171``).  Its executors lower that
graph at construction time (``ERV/chipformer/rv/tritonexec.py:176-244``) and build the output-code
decode tables of free-running generation (``ERV/chipformer/rv/fastexec.py:254-283``).  Neither the
graph builder nor its token-feature lambdas can travel to a machine without the reference, so this
module writes everything the executor consumes into one ``.npz``:

* every FFN node with its units ``coef * a * relu(b)`` (a / b as sparse linear forms), in
  ``c.nodes`` order, so that units keep the order ``Executor2`` gives them;
* every Gated DeltaNet head with its q / k channels (conv taps folded in as lag * D + dim, the
  ``lagged`` rule of ``tritonexec.py:201-203``) and its value heads (v channels, z gates, decay
  selector a, write gate beta, output columns), plus the decay row count ``nrows``
  (``tritonexec.py:229-231``);
* the embedding of every chip token, tabulated the way ``FreeRun`` tabulates it
  (``fastexec.py:264-281``: a table row for families of at most 4,096 tokens, ``base + sum of
  payload-bit rows`` for the big ones), restricted to the token-feature dims and ONE, which are the
  only dims an embedding sets (``tritonexec.py:265-270``);
* the output-code dims (``c.out_fam`` / ``c.out_pay``), the snapshot tables (``c.tables``) with
  their value-head positions, and the register bit columns (``c.reg_cols``).

All weights are stored as float32, the precision ``Executor2`` computes in; ``export_graph``
asserts that the conversion from the graph's exact values loses nothing.

``load_graph`` returns a :class:`GraphData` with plain numpy arrays; nothing here imports the
reference unless ``export_graph`` is called.
"""

from __future__ import annotations

import dataclasses
from pathlib import Path

import numpy as np

HD = 128  # key / value head dim (ERV/chipformer/q35/ir.py:43)
REF_COLS = (0, 1)  # ballast columns of a state row (ir.py:41)
A_REF = 2.0 ** 24  # ballast value (ir.py:39)
A_BIT = 2.0 ** 7  # value of a set bit in a state row (ir.py:40)
ONE = 0  # dim of the constant-one feature (ERV/chipformer/dsl/graph.py:29)
FORMAT_VERSION = 1
TEXT_TOKEN = 1 << 24  # a text token in the circuit's stream: TEXT_TOKEN | qid (ERV/chipformer/rv/spec.py:89)
# a text token's bits (ERV/chipformer/rv/core.py:139-165): its text row's 16 bytes (bit 8k + i =
# bit i of byte k), isTCO, isTCC, printable, then the 21 bits of its own output code (family Q,
# payload = its printable index) when printable; TEXT_WORDS uint32 words per token
TEXT_ROW_BITS, TEXT_NBITS, TEXT_WORDS = 128, 152, 5


def _f32(x: float) -> np.float32:
    v = np.float32(x)
    if float(v) != float(x):
        raise ValueError(f"weight {x!r} is not exact in float32")
    return v


@dataclasses.dataclass
class Forms:
    """A list of sparse linear forms in CSR: form i = sum of w[j] * src[idx[j]] for
    j in ptr[i]..ptr[i+1]. ``idx`` is lag * D + dim (lag 0 = the current residual)."""

    ptr: np.ndarray  # int64 [n + 1]
    idx: np.ndarray  # int32 [nnz]
    w: np.ndarray  # float32 [nnz]

    @property
    def n(self) -> int:
        return len(self.ptr) - 1

    def row(self, i: int) -> tuple[np.ndarray, np.ndarray]:
        a, b = self.ptr[i], self.ptr[i + 1]
        return self.idx[a:b], self.w[a:b]

    @staticmethod
    def build(rows: list[dict]) -> "Forms":
        """Forms from {source index: weight} dicts, each form's terms in ascending source order
        (the graph builder's own term order depends on Python's string-hash seed; the sums are
        exact in any order, so a canonical order makes the export reproducible)."""
        ptr = [0]
        idx, w = [], []
        for r in rows:
            for k, v in sorted((int(k), v) for k, v in r.items()):
                if v:
                    idx.append(k)
                    w.append(_f32(v))
            ptr.append(len(idx))
        return Forms(np.asarray(ptr, np.int64), np.asarray(idx, np.int32),
                     np.asarray(w, np.float32))


@dataclasses.dataclass
class GraphData:
    """The executor's view of a compiled graph (see the module doc)."""

    D: int
    levels: np.ndarray  # int32 [L]: the sublayer levels, ascending
    level_kind: np.ndarray  # int8 [L]: 0 FFN, 1 heads
    # FFN nodes (c.nodes order)
    ffn_level: np.ndarray  # int32 [N]
    ffn_out: np.ndarray  # int32 [N]
    ffn_into: np.ndarray  # bool [N]
    ffn_uptr: np.ndarray  # int64 [N + 1] into the unit arrays
    unit_coef: np.ndarray  # float32 [U]
    unit_a: Forms  # U forms
    unit_b: Forms  # U forms
    # heads (c.nodes order)
    head_level: np.ndarray  # int32 [H]
    head_name: np.ndarray  # str [H]
    head_qhot: np.ndarray  # int32 [H]
    head_q: np.ndarray  # int32 [H, HD]: form index into q_forms, -1 = no channel
    head_k: np.ndarray  # int32 [H, HD]
    q_forms: Forms
    k_forms: Forms
    # value heads (per head, vheads() order)
    vh_head: np.ndarray  # int32 [VH]: owning head
    vh_into: np.ndarray  # bool [VH]
    vh_v: np.ndarray  # int32 [VH, HD]: index into v_forms, -1 none
    vh_z: np.ndarray  # int32 [VH, HD]: index into z_forms, -1 none
    v_forms: Forms
    z_forms: Forms
    vh_a: Forms  # VH forms (decay selector)
    vh_beta: Forms  # VH forms (write gate)
    vh_has_beta: np.ndarray  # bool [VH]
    vh_nrows: np.ndarray  # int32 [VH]
    vh_out_ptr: np.ndarray  # int64 [VH + 1]
    out_col: np.ndarray  # int32 [O]
    out_dim: np.ndarray  # int32 [O]
    out_w: np.ndarray  # float32 [O]
    # token embedding (FreeRun's tables, on the feature dims only)
    feat_dims: np.ndarray  # int32 [F]: ONE first, then the token-feature dims ascending
    fam_names: np.ndarray  # str [nf]
    fam_ids: np.ndarray  # int64 [nf]: first token id of the family
    fam_size: np.ndarray  # int64 [nf]
    fam_small: np.ndarray  # bool [nf]
    fam_row0: np.ndarray  # int64 [nf]
    emb_base: np.ndarray  # float32 [nf, F]
    emb_bits: np.ndarray  # float32 [nf, NPAY, F]
    emb_table: np.ndarray  # float32 [R, F]
    fam_dims: np.ndarray  # int32 [NFAM]
    pay_dims: np.ndarray  # int32 [NPAY]
    vocab: int
    # snapshot tables
    table_names: np.ndarray  # str [T]
    table_head: np.ndarray  # int32 [T]: head index
    reg_cols: np.ndarray  # int32 [32, 8]: bit -> source columns (-1 padded)
    # merged graphs (built with the text bridge, ERV/chipformer/rv/core.py:1128-1163): the
    # prediction is read from the signs of the code dims (empty for a standalone graph, which
    # reads fam_dims / pay_dims), the P3 echo family Q names text tokens, and text tokens
    # (TEXT_TOKEN | qid) are embedded as text_base + sum of the rows of their set bits
    code_dims: np.ndarray = dataclasses.field(default_factory=lambda: np.zeros(0, np.int32))
    keep_dims: np.ndarray = dataclasses.field(default_factory=lambda: np.zeros(0, np.int32))
    q_fid: np.ndarray = dataclasses.field(default_factory=lambda: np.full(1, -1, np.int64))  # [1]
    printable: np.ndarray = dataclasses.field(default_factory=lambda: np.zeros(0, np.int32))  # Q payload -> qid
    text_words: np.ndarray = dataclasses.field(default_factory=lambda: np.zeros((0, TEXT_WORDS), np.uint32))
    text_base: np.ndarray = dataclasses.field(default_factory=lambda: np.zeros(0, np.float32))  # [F]
    text_bits: np.ndarray = dataclasses.field(default_factory=lambda: np.zeros((0, 0), np.float32))  # [152, F]

    # ---- derived views -------------------------------------------------------------------
    def head_sublayers(self) -> list[int]:
        return [int(lv) for lv, k in zip(self.levels, self.level_kind) if k == 1]

    def heads_at(self, level: int) -> list[int]:
        return [h for h in range(len(self.head_level)) if self.head_level[h] == level]

    def vheads_of(self, h: int) -> list[int]:
        return [j for j in range(len(self.vh_head)) if self.vh_head[j] == h]

    def vheads_at(self, level: int) -> list[int]:
        """Value heads of a head sublayer in Executor2's order (heads in node order, then each
        head's value heads; tritonexec.py:197-198)."""
        return [j for h in self.heads_at(level) for j in self.vheads_of(h)]

    def table_position(self, name: str) -> tuple[int, int, int]:
        """(sublayer level, first value-head index within that sublayer, value heads) of a
        snapshot table."""
        t = list(self.table_names).index(name)
        h = int(self.table_head[t])
        lv = int(self.head_level[h])
        vhs = self.vheads_at(lv)
        mine = self.vheads_of(h)
        return lv, vhs.index(mine[0]), len(mine)

    def embed(self, toks) -> np.ndarray:
        """[n, D] float32 embeddings through the tabulated FreeRun rule (fastexec.py:305-307)."""
        out = np.zeros((len(toks), self.D), np.float32)
        for i, t in enumerate(toks):
            if int(t) >= TEXT_TOKEN:
                out[i, self.feat_dims] = self.text_embedding(int(t) - TEXT_TOKEN)
                continue
            f, p = self.family_of(int(t))
            if self.fam_small[f]:
                row = self.emb_table[self.fam_row0[f] + p]
            else:
                pay = np.array([(p >> b) & 1 for b in range(self.emb_bits.shape[1])], np.float32)
                row = self.emb_base[f] + np.einsum("i,id->d", pay, self.emb_bits[f])
            out[i, self.feat_dims] = row
        return out

    @property
    def merged(self) -> bool:
        return len(self.code_dims) > 0

    def text_embedding(self, qid: int) -> np.ndarray:
        """The feature row of text token qid: text_base + the rows of its set bits (summed in bit
        order; exact values)."""
        if not self.merged or not 0 <= qid < len(self.text_words):
            raise ValueError(f"text token {qid} is not in this graph's text vocabulary")
        w = self.text_words[qid]
        row = self.text_base.astype(np.float32).copy()
        for j in range(TEXT_NBITS):
            if w[j >> 5] >> (j & 31) & 1:
                row = row + self.text_bits[j]
        return row

    def decode(self, x: np.ndarray) -> int:
        """The token a residual row predicts (FreeRun._step's rule, fastexec.py:298-307, for a
        standalone graph; core.predictions' merged rule, core.py:1287-1304, for a merged one:
        code dims > 0 are the bits, a Q code is the text token of printable payload p). -1: the
        code names no token, or (merged) every code dim is 0 (the circuit does not predict)."""
        nf, npay = int(self.fam_dims.size or 5), int(self.pay_dims.size or 16)
        if self.merged:
            v = x[self.code_dims]
            if not np.any(v != 0):
                return -1
            bits = (v > 0).astype(np.int64)
            nf = len(self.code_dims) - npay
            fid = int(sum(int(b) << i for i, b in enumerate(bits[:nf])))
            p = int(sum(int(b) << i for i, b in enumerate(bits[nf:])))
            if fid == int(self.q_fid[0]):
                return TEXT_TOKEN + int(self.printable[p]) if p < len(self.printable) else -1
        else:
            fid = int(sum(int(np.rint(x[d])) << i for i, d in enumerate(self.fam_dims)))
            p = int(sum(int(np.rint(x[d])) << i for i, d in enumerate(self.pay_dims)))
        if not 0 <= fid < len(self.fam_ids) or p >= int(self.fam_size[fid]):
            return -1
        return int(self.fam_ids[fid]) + p

    def family_of(self, t: int) -> tuple[int, int]:
        for f in range(len(self.fam_ids)):
            if self.fam_ids[f] <= t < self.fam_ids[f] + self.fam_size[f]:
                return f, t - int(self.fam_ids[f])
        raise ValueError(f"token {t} is in no family")


def _forms_to_npz(prefix: str, f: Forms, out: dict) -> None:
    out[prefix + ".ptr"] = f.ptr
    out[prefix + ".idx"] = f.idx
    out[prefix + ".w"] = f.w


def _forms_from_npz(prefix: str, z) -> Forms:
    return Forms(z[prefix + ".ptr"], z[prefix + ".idx"], z[prefix + ".w"])


def save_graph(g: GraphData, path: str | Path) -> None:
    out = {"format_version": np.int32(FORMAT_VERSION), "D": np.int64(g.D),
           "vocab": np.int64(g.vocab)}
    for fld in dataclasses.fields(GraphData):
        v = getattr(g, fld.name)
        if isinstance(v, Forms):
            _forms_to_npz(fld.name, v, out)
        elif fld.name not in ("D", "vocab"):
            out[fld.name] = np.asarray(v)
    np.savez_compressed(path, **out)


def load_graph(path: str | Path) -> GraphData:
    z = np.load(path, allow_pickle=False)
    if int(z["format_version"]) != FORMAT_VERSION:
        raise ValueError(f"{path}: graph format {int(z['format_version'])}, "
                         f"expected {FORMAT_VERSION}")
    kw = {}
    for fld in dataclasses.fields(GraphData):
        if fld.name in ("D", "vocab"):
            kw[fld.name] = int(z[fld.name])
        elif fld.type == "Forms":
            kw[fld.name] = _forms_from_npz(fld.name, z)
        elif fld.name in z.files:
            kw[fld.name] = z[fld.name]
    return GraphData(**kw)


def default_graph_path() -> Path:
    """The standalone RV32IM machine shipped with the package."""
    return Path(__file__).parent / "plans" / "rv32im_graph.npz"


def merged_graph_path() -> Path:
    """The machine with the text bridge (merged readout, text tokens) over a byte-level vocabulary."""
    return Path(__file__).parent / "plans" / "rv32im_merged_graph.npz"


# ---- export from a live chipformer graph (needs the reference importable) -------------------


def export_graph(c) -> GraphData:
    """Lower a ``chipformer.q35.ir.Graph`` (a standalone ``core.build()`` machine) into
    :class:`GraphData`. Follows ``Executor2.__init__`` (tritonexec.py:176-244) for the weights and
    ``FreeRun.__init__`` (fastexec.py:254-283) for the embedding / decode tables, except that the
    P3 echo family ``Q`` is skipped: it has no token family without the text bridge
    (ERV/chipformer/rv/spec.py:58-65; FreeRun raises KeyError on it)."""
    from chipformer.q35.ir import FFN, Head  # noqa: F401  (reference types)
    from chipformer.rv import core as C
    from chipformer.rv import spec as S

    D = len(c.dims)
    levels = sorted({n.level for n in c.nodes})
    kinds = []
    for lv in levels:
        nodes = [n for n in c.nodes if n.level == lv]
        kinds.append(0 if isinstance(nodes[0], FFN) else 1)
        assert all(isinstance(n, FFN) == (kinds[-1] == 0) for n in nodes), lv

    def terms(e) -> dict:
        return {int(d): float(cf) for d, cf in e.terms.items()}

    def lagged(ch) -> dict:  # tritonexec.py:201-203
        return {lag * D + d: float(cf) * tw for lag, tw in enumerate(ch.taps) if tw
                for d, cf in ch.expr.terms.items()}

    # FFN nodes in level order (Executor2 walks levels, then c.nodes order inside a level)
    ffn_nodes = [n for lv in levels for n in c.nodes if n.level == lv and isinstance(n, FFN)]
    uptr, coef, arows, brows = [0], [], [], []
    for n in ffn_nodes:
        for cf, a, b in n.terms:
            coef.append(_f32(float(cf)))
            arows.append(terms(a))
            brows.append(terms(b))
        uptr.append(len(coef))

    heads = [n for lv in levels for n in c.nodes if n.level == lv and isinstance(n, Head)]
    qrows, krows = [], []
    head_q = np.full((len(heads), HD), -1, np.int32)
    head_k = np.full((len(heads), HD), -1, np.int32)
    vh_head, vh_into, vrows, zrows, arows_v, brows_v, has_beta, nrows = ([] for _ in range(8))
    vh_v, vh_z, out_ptr, out_col, out_dim, out_w = [], [], [0], [], [], []
    for h, n in enumerate(heads):
        for s in range(HD):
            if s in n.q:
                head_q[h, s] = len(qrows)
                qrows.append(lagged(n.q[s]))
            if s in n.k:
                head_k[h, s] = len(krows)
                krows.append(lagged(n.k[s]))
        reach = set(n.k) | {r for x in (n.init or []) for r in x}
        for vd in n.vheads():
            vh_head.append(h)
            vh_into.append(bool(vd.into))
            vv = np.full(HD, -1, np.int32)
            zz = np.full(HD, -1, np.int32)
            for col in range(HD):
                if col in vd.v:
                    vv[col] = len(vrows)
                    vrows.append(lagged(vd.v[col]))
                if col in vd.z:
                    zz[col] = len(zrows)
                    zrows.append(terms(vd.z[col]))
            vh_v.append(vv)
            vh_z.append(zz)
            arows_v.append(terms(vd.a))
            if vd.beta is None:
                brows_v.append({})
                has_beta.append(False)
            else:
                brows_v.append(terms(vd.beta))
                has_beta.append(True)
            nrows.append(max(reach) + 1 if vd.a.terms and reach else 0)
            for col, d, w in vd.out:
                out_col.append(int(col))
                out_dim.append(int(d))
                out_w.append(_f32(float(w)))
            out_ptr.append(len(out_col))
    assert max(len(r) for r in arows_v + brows_v) <= 32  # tritonexec.py:232

    # embedding / decode (FreeRun)
    feat_ids = sorted(c.token_fns)
    feat_dims = [ONE] + feat_ids

    def emb(toks):
        out = np.zeros((len(toks), len(feat_dims)), np.float64)
        out[:, 0] = 1.0
        for j, d in enumerate(feat_ids):
            out[:, j + 1] = [float(c.feature_value(d, t)) for t in toks]
        return out

    names = [nm for nm in C.OUT_NAMES if nm in S.CONTROLS or nm in S.FAMILIES]
    assert names == C.OUT_NAMES[:len(names)], "skipped families must be the last ones"
    merged = c.out_fam is None
    nf, nb = len(names), C.NPAY
    base = np.zeros((nf, len(feat_dims)))
    bits = np.zeros((nf, nb, len(feat_dims)))
    ids, sizes = np.zeros(nf, np.int64), np.zeros(nf, np.int64)
    small, row0, table = np.zeros(nf, bool), np.zeros(nf, np.int64), []
    for f, nm in enumerate(names):
        t0 = S.tok(nm) if nm in S.CONTROLS else S.tok(nm, 0)
        size = 1 if nm in S.CONTROLS else S.FAMILIES[nm][1]
        ids[f], sizes[f] = t0, size
        base[f] = emb([t0])[0]
        if size <= 4096:
            small[f], row0[f] = True, len(table)
            table += list(emb(list(range(t0, t0 + size))))
        else:
            for i in range(size.bit_length() - 1):
                bits[f, i] = emb([t0 + (1 << i)])[0] - base[f]
    for arr in (base, bits, np.asarray(table)):
        assert np.all(arr.astype(np.float32).astype(np.float64) == arr)

    def dim_of(e):
        ((d, w),) = e.terms.items()
        assert w == 1
        return int(d)

    extra = {}
    if merged:
        extra = _export_text(c, feat_ids, feat_dims, emb)
    tnames = list(c.tables)
    hidx = {id(n): i for i, n in enumerate(heads)}
    reg_cols = np.full((32, 8), -1, np.int32)
    for i, cols in c.reg_cols.items():
        reg_cols[i, :len(cols)] = cols

    return GraphData(
        D=D, levels=np.asarray(levels, np.int32), level_kind=np.asarray(kinds, np.int8),
        ffn_level=np.asarray([n.level for n in ffn_nodes], np.int32),
        ffn_out=np.asarray([n.out for n in ffn_nodes], np.int32),
        ffn_into=np.asarray([bool(n.into) for n in ffn_nodes]),
        ffn_uptr=np.asarray(uptr, np.int64), unit_coef=np.asarray(coef, np.float32),
        unit_a=Forms.build(arows), unit_b=Forms.build(brows),
        head_level=np.asarray([n.level for n in heads], np.int32),
        head_name=np.asarray([n.name for n in heads]),
        head_qhot=np.asarray([getattr(n, "qhot", 2) for n in heads], np.int32),
        head_q=head_q, head_k=head_k, q_forms=Forms.build(qrows), k_forms=Forms.build(krows),
        vh_head=np.asarray(vh_head, np.int32), vh_into=np.asarray(vh_into),
        vh_v=np.asarray(vh_v, np.int32).reshape(-1, HD),
        vh_z=np.asarray(vh_z, np.int32).reshape(-1, HD),
        v_forms=Forms.build(vrows), z_forms=Forms.build(zrows),
        vh_a=Forms.build(arows_v), vh_beta=Forms.build(brows_v),
        vh_has_beta=np.asarray(has_beta), vh_nrows=np.asarray(nrows, np.int32),
        vh_out_ptr=np.asarray(out_ptr, np.int64), out_col=np.asarray(out_col, np.int32),
        out_dim=np.asarray(out_dim, np.int32), out_w=np.asarray(out_w, np.float32),
        feat_dims=np.asarray(feat_dims, np.int32), fam_names=np.asarray(names),
        fam_ids=ids, fam_size=sizes, fam_small=small, fam_row0=row0,
        emb_base=base.astype(np.float32), emb_bits=bits.astype(np.float32),
        emb_table=np.asarray(table, np.float32).reshape(-1, len(feat_dims)),
        fam_dims=np.asarray([dim_of(e) for e in c.out_fam] if not merged else [], np.int32),
        pay_dims=np.asarray([dim_of(e) for e in c.out_pay] if not merged else [], np.int32),
        vocab=int(S.VOCAB),
        table_names=np.asarray(tnames),
        table_head=np.asarray([hidx[id(c.tables[t])] for t in tnames], np.int32),
        reg_cols=reg_cols,
        **extra,
    )


def _export_text(c, feat_ids: list, feat_dims: list, emb) -> dict:
    """The merged graph's readout and text-token tables: code / keep dims, the Q family's id, the
    printable tokens, and every text token's bits with the rows they add (the text row's byte
    bits, the <tool_call> / </tool_call> flags, its own Q code when printable:
    ERV/chipformer/rv/core.py:139-165).  Checked against the graph's own feature functions for
    every text token of the vocabulary."""
    from chipformer.rv import core as C

    text = c.text
    fcol = {d: j for j, d in enumerate(feat_dims)}
    name = {c.dims[d].name: d for d in feat_ids}

    def dim_of(e):
        ((d, w),) = e.terms.items()
        assert w == 1
        return int(d)

    code = [dim_of(e) for e in c.code]
    F = len(feat_dims)
    rows = np.zeros((TEXT_NBITS, F))
    for k in range(16):
        for i in range(8):
            rows[8 * k + i, fcol[name[f"tb{k}.b{i}"]]] = 1.0
    rows[128, fcol[name["isTCO"]]] = 1.0
    rows[129, fcol[name["isTCC"]]] = 1.0
    for j, d in enumerate(code):
        rows[130, fcol[d]] = -C.CODE_AMP  # printable: every code dim -CODE_AMP ...
        rows[131 + j, fcol[d]] = 2 * C.CODE_AMP  # ... + 2 CODE_AMP where its code bit is 1
    base = emb([TEXT_TOKEN + text.n])[0]  # a text token with no bit set (beyond the vocabulary)
    words = np.zeros((text.n, TEXT_WORDS), np.uint32)
    for q in range(text.n):
        rb = text.row_bytes(q)
        bits = [rb[k] >> i & 1 for k in range(16) for i in range(8)]
        p = text.printable_index(q)
        bits += [int(q == text.TCO), int(q == text.TCC), int(p is not None)]
        bits += C.code_bits("Q", p) if p is not None else [0] * (C.NFAM + C.NPAY)
        for j, b in enumerate(bits):
            if b:
                words[q, j >> 5] |= np.uint32(1 << (j & 31))
    # every text token's features through the bits equal the graph's own
    want = emb([TEXT_TOKEN + q for q in range(text.n)])
    for q in range(text.n):
        got = base.copy()
        for j in range(TEXT_NBITS):
            if words[q, j >> 5] >> (j & 31) & 1:
                got = got + rows[j]
        if not np.array_equal(got, want[q]):
            bad = np.flatnonzero(got != want[q])
            raise AssertionError(f"text token {q}: feature dims {[feat_dims[b] for b in bad[:5]]} differ")
    for a in (base, rows):
        assert np.all(a.astype(np.float32).astype(np.float64) == a)
    return dict(code_dims=np.asarray(code, np.int32), keep_dims=np.asarray(c.keep, np.int32),
                q_fid=np.asarray([C.OUT_NAMES.index("Q")], np.int64),
                printable=np.asarray(text.printable, np.int32), text_words=words,
                text_base=base.astype(np.float32), text_bits=rows.astype(np.float32))
