"""A numpy interpreter of the executor's phase program (test infrastructure): runs a compiled
plan exactly as the CUDA kernel's phases describe it, on the CPU, so the plan compiler can be
checked against the oracle without a GPU."""

import numpy as np

from qwenputer_b200.plan import PH

NONE = 0xFFFFFFFF


class _ByteIndexed:
    """Rows of the word-indexed array addressed by byte offsets."""

    def __init__(self, a):
        self.a = a

    def __getitem__(self, k):
        if isinstance(k, tuple):
            return self.a[(int(k[0]) // 4,) + k[1:]]
        return self.a[int(k) // 4]

    def __setitem__(self, k, v):
        if isinstance(k, tuple):
            self.a[(int(k[0]) // 4,) + k[1:]] = v
        else:
            self.a[int(k) // 4] = v


def _f32(x):
    return np.float32(x)


class PlanInterp:
    def __init__(self, P, B: int):
        self.P, self.B = P, B
        s = P.sec
        self.s = s
        h = P.hdr
        self.rows = h["n_slots"] + h["n_scratch"]
        # machines a CTA runs, and record slots a warp (bundled plans: lines of `ways` quads)
        self.group = h.get("group", 32)
        self.ways = 32 // self.group
        # indexed by shared-memory word offset (byte offset / 4, rows group + 1 words apart); the
        # row after the last is zero
        self.Xw = np.zeros(((self.rows + 1) * (self.group + 1), B), np.float32)
        self.X = _ByteIndexed(self.Xw)
        self.hl_v = s["HL_V"]
        self.S = [np.zeros((B, int(v), 128, 128), np.float32) for v in s["HL_V"]]
        self.H = [np.zeros((3, int(ne), B), np.float32) for ne in s["HL_NE"]]
        self.one = h["one_row"]
        self.ksel, self.qsel = {}, {}
        # value-head outputs go to delta rows (byte offset j * 128), which VHSUM phases add into
        # the residual rows
        self.Dw = np.zeros((128 * 32, B), np.float32)
        self.delta = _ByteIndexed(self.Dw)

    def warp_records(self, c, k):
        """Per warp, its records of a stream phase: lists of (header, body quads) pieces, the
        R_SKIP padding dropped (a record's pieces are consecutive and end with R_LAST).  In a
        bundled plan a piece is a header line and n body lines of `ways` quads: record slot s
        reads quad s of each line; the bundle's padding records (R_NOP) are dropped."""
        from qwenputer_b200.plan import R_LAST, R_NOP, R_SKIP, R_SPLIT

        st = self.s["STREAM"].astype(np.int64)
        wp = self.s["WARP_PTR"].astype(np.int64)
        nw = self.P.hdr["nw"] * self.P.hdr["cluster"]  # the warps of a group's cluster
        R = self.ways
        out = []
        for w in range(nw):
            i, end, start = wp[c + w], wp[c + w + 1], wp[c + w]
            recs, cur = [], [[] for _ in range(R)]
            while i < end:
                hs = st[i:i + R]
                n, fl = int(hs[0][3]) & 0xFFFFFF, int(hs[0][3]) >> 24
                if fl & R_SKIP:
                    i = start + ((i - start) // (32 * R) + 1) * (32 * R)
                    continue
                body = st[i + R:i + R * (1 + n)].reshape(n, R, 4) if n else np.zeros((0, R, 4), np.int64)
                for sl in range(R):
                    fs = int(hs[sl][3]) >> 24
                    assert int(hs[sl][3]) & 0xFFFFFF == n and (fs ^ fl) & 3 == 0, "a bundle's pieces differ"
                    cur[sl].append((hs[sl], body[:, sl]))
                i += R * (1 + n)
                if fl & R_LAST:
                    if fl & R_SPLIT:  # one record over the slots: its pieces hold every slot's terms
                        recs.append([(pc[0], np.concatenate([cur[sl][j][1] for sl in range(R)]))
                                     for j, pc in enumerate(cur[0])])
                    else:
                        for sl in range(R):
                            if not (int(cur[sl][0][0][3]) >> 24) & R_NOP:
                                recs.append(cur[sl])
                    cur = [[] for _ in range(R)]
            assert not any(cur)
            out.append(recs)
        return out

    def entries(self, ent):
        q = ent.reshape(-1, 4)
        acc = np.zeros(self.B, np.float32)
        for off, w in list(zip(q[:, 0], q[:, 1])) + list(zip(q[:, 2], q[:, 3])):
            acc = acc + np.uint32(w).view(np.float32) * self.X[off]
        return acc

    def row(self, r, m=slice(None)):
        return self.X[r, m]

    def step(self, x: np.ndarray) -> np.ndarray:
        """Step mode on x [B, D] (in place)."""
        s = self.s
        for ph in s["STEP_PROG"]:
            k, a, b, c = (int(ph[f]) for f in ("kind", "a", "b", "c"))
            k &= 0xFF
            if k == PH["END"]:
                break
            if k == PH["ZERO"]:
                for i in range(b):
                    self.X[s["ROWS"][a + i]] = 0
            elif k == PH["LOADX"]:
                for r, d in s["PAIRS"][a:a + b]:
                    self.X[r] = x[:, d]
            elif k == PH["WRITEOUT"]:
                for r, d in s["PAIRS"][a:a + b]:
                    x[:, d] = self.X[r]
            elif k == PH["APPLY"]:
                for dst, src in s["PAIRS"][a:a + b]:
                    self.X[dst] = self.X[dst] + self.X[src]
            elif k == PH["STAGE"]:
                H = self.H[c]
                for st in s["STAGES"][a:a + b]:
                    e, xr, ml = int(st["e"]), int(st["x_row"]), int(st["ml"])
                    h = H[:, e].copy()
                    for lag, key in enumerate(("s0", "s1", "s2")):
                        if st[key] != NONE:
                            self.X[st[key]] = h[lag]
                    H[0, e] = self.X[xr]
                    if ml >= 2:
                        H[1, e] = h[0]
                    if ml >= 3:
                        H[2, e] = h[1]
            elif k == PH["FORMS"]:
                f32 = lambda v: np.uint32(v).view(np.float32)
                for recs in self.warp_records(c, k):
                    for pcs in recs:
                        body = np.concatenate([q for _, q in pcs])
                        fa = np.zeros(self.B, np.float32)
                        fb = np.zeros(self.B, np.float32)
                        for e in body:
                            fa = fa + f32(e[1]) * self.X[e[0]]
                            fb = fb + f32(e[3]) * self.X[e[2]]
                        self.X[pcs[0][0][0]] = fa
                        self.X[pcs[0][0][1]] = fb
            elif k == PH["UNITS"]:
                f32 = lambda v: np.uint32(v).view(np.float32)
                for recs in self.warp_records(c, k):
                    for pcs in recs:
                        acc = np.zeros(self.B, np.float32)
                        for h, q in pcs:
                            nc = int(h[1])
                            for u in q[:nc]:
                                acc = acc + f32(u[1]) * np.maximum(self.X[u[0]] + f32(u[2]), 0)
                            for j in range(nc, len(q), 2):
                                u, u2 = q[j], q[j + 1]
                                av = self.X[u[0]] + f32(u[3])
                                acc = acc + (f32(u[2]) * av) * np.maximum(self.X[u[1]] + f32(u2[0]), 0)
                        out = pcs[0][0][0]
                        self.X[out] = self.X[out] + acc
            elif k == PH["KSEL"]:
                f32 = lambda v: np.uint32(v).view(np.float32)

                def word(v, ch):
                    # the kernel's slot word: value bits above bit 7, 127 - channel below (0: none)
                    w = np.maximum(v.view(np.uint32) & np.uint32(0xFFFFFF80), np.uint32(0x80))
                    return np.where(v > 0, w | (np.uint32(127) - ch.astype(np.uint32)), np.uint32(0))

                # the slots start cleared (the previous value-head serving phase clears them)
                self.kword, self.qword = {}, {}
                for recs in self.warp_records(c, k):
                    for pcs in recs:
                        # a key part or a query part of a key head (or a part of one: R_MERGE)
                        x0 = int(pcs[0][0][0])
                        slot, qhot, lo = x0 & 0xFFFF, (x0 >> 16) & 0xFF, x0 >> 24
                        fl = int(pcs[0][0][3]) >> 24
                        query, merge = bool(fl & 8), bool(fl & 0x10)
                        vals = []
                        for h, q in pcs:
                            com, x1 = self.X[h[1]], self.X[h[2]]
                            for qq in q:
                                v = f32(qq[2]) * x1 + (f32(qq[1]) + (f32(qq[3]) * com + self.X[qq[0]]))
                                vals.append(np.maximum(v, 0))
                        vv = np.stack(vals) if vals else np.zeros((1, self.B), np.float32)
                        # the part's own selection (first maxima, exact)
                        sel = []
                        for j in range(1 if not query else qhot):
                            qm, qa = vv.max(0), vv.argmax(0)
                            sel.append(word(qm, qa + lo))
                            vv[qa, np.arange(self.B)] = 0
                        levels = 1 if not query else qhot
                        tab = self.kword if not query else self.qword
                        if not merge:
                            tab[slot] = sel
                        else:  # the merged levels: the largest words of every part, in order
                            prev = tab.get(slot, [np.zeros(self.B, np.uint32)] * levels)
                            allw = np.sort(np.stack(prev + sel), axis=0)[::-1]
                            tab[slot] = list(allw[:levels])
                dec = lambda w: np.where(w != 0, 127 - (w & 0x7F).astype(np.int64), -1)
                self.ksel = {sl: dec(w[0]) for sl, w in self.kword.items()}
                self.qsel = {sl: [dec(x) for x in w] for sl, w in self.qword.items()}
            elif k == PH["MMA"]:
                # tensor-core forms: per form block, D = sum over its tiles of A (bf16 weights,
                # [128 forms x 16 rows]) x the staged source rows (bf16-exact, checked); the sums
                # are exact, so float64 accumulation cast to float32 is the kernel's result
                mp = s["MMA_PHASES"][a]
                n_kb, kr0, n_fb, dst0 = (int(mp[f]) for f in ("n_kb", "kr0", "n_fb", "dst0"))
                src = s["ROWS"][kr0:kr0 + 16 * n_kb]
                xs = np.stack([self.X[int(r)] for r in src]).astype(np.float32)
                assert not (xs.view(np.uint32) & 0xFFFF).any(), "a staged value is not bf16-exact"
                xs = xs.astype(np.float64)
                data = s["TILEDATA"].reshape(-1, 128, 16)
                acc = np.zeros((n_fb, 128, self.B))
                for t in s["MMA_TILES"][int(mp["t0"]):int(mp["t1"])]:
                    A = (data[int(t["data"])].astype(np.uint32) << 16).view(np.float32).astype(np.float64)
                    kb, fb = int(t["kb"]), int(t["fb"])
                    part = A @ xs[16 * kb:16 * kb + 16]
                    acc[fb] = part if int(t["acc"]) == 0 else acc[fb] + part
                for fb in range(n_fb):
                    for i in range(128):
                        dst = int(s["ROWS"][dst0 + fb * 128 + i])
                        if dst != NONE:
                            self.X[dst] = acc[fb, i].astype(np.float32)
            elif k == PH["VHRUN"]:
                pass  # the row work a VH phase lists is done here while it is listed
            elif k == PH["VHSUM"]:
                for jj in range(b):
                    self.X[int(s["VHSUM_ROWS"][a + jj])] += self.delta[jj * 128]
            elif k == PH["VH"]:
                self.Dw[:] = 0
                # direct plans (one CTA a group) add the outputs into the residual rows themselves
                out_rows = self.X if self.P.hdr.get("flags", 0) & 4 else self.delta
                x0 = self.X[self.one]
                for vh in s["VHEADS"][a:b]:
                    hl, j, col, sl = int(vh["hl"]), int(vh["vh"]), int(vh["col"]), int(vh["slot"])
                    for m in range(self.B):
                        Sb = self.S[hl][m, j]
                        if vh["nrows"]:
                            av = self.row(int(vh["a_row"]), m) + vh["ca"] * x0[m]
                            fac = 1.0 if av == 0 else (0.5 if av == 110 else 0.0)
                            if fac != 1.0:
                                Sb[:vh["nrows"]] *= np.float32(fac)
                        bv = (self.row(int(vh["b_row"]), m) + vh["cb"] * x0[m]) + vh["bconst"]
                        kr = self.ksel[sl][m]
                        if kr >= 0 and bv == 1.0:
                            vals = np.zeros(128, np.float32)
                            for cc in range(128):
                                cf = s["VFORM"][col + cc]
                                if cf["live"]:
                                    vals[cc] = max(self.X[int(cf["row"]), m] + cf["c"] * x0[m], 0)
                            Sb[kr] = vals
                        o = np.zeros(128, np.float32)
                        anyr = False
                        for sel in self.qsel[sl]:
                            if sel[m] >= 0:
                                o = o + Sb[sel[m]]
                                anyr = True
                        if not anyr:
                            continue
                        ref = np.float32(o[0] * o[0]) + np.float32(o[1] * o[1])
                        norm = np.sqrt(np.float32(ref / np.float32(128)))
                        for cc in range(128):
                            orow = int(s["OUT_ROW"][col + cc])
                            if orow == NONE:
                                continue
                            if int(vh["nout"]) != 0xFF:
                                orow = int(vh["out4"][orow])  # an index into the head's 4 rows
                            zf = s["ZFORM"][col + cc]
                            z = max(self.X[int(zf["row"]), m] + zf["c"] * x0[m], 0) if zf["live"] else 0
                            out = o[cc] / norm if ref > 0 else np.float32(0)
                            out_rows[orow, m] += np.float32(out * np.float32(z)) * s["OUT_W"][col + cc]
        return x
