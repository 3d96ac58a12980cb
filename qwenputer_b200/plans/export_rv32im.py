"""Writes the reference's RV32IM (+Zba, bignum) compiled stack (``ERV/chipformer/rv/core.py:299
build()``, target Qwen3.5-4B layer shapes ``core.T4B``) in the executor's file format
(``qwenputer_b200/graphfile.py``):

* ``rv32im_graph.npz``         the standalone machine (``core.build()``);
* ``rv32im_merged_graph.npz``  the machine with the text bridge (``core.build(text=...)``: the
  graph a merged Qwen3.5 checkpoint carries), over ``ByteVocab``, a byte-level vocabulary in
  the shape of Qwen's (its tokenizer file is not available here).

Needs the reference tree importable (``ERV`` = ``experimental/riscv``), given as the argument
or as ``QX_REFERENCE_ROOT``::

    python qwenputer_b200/plans/export_rv32im.py /path/to/reference/experimental/riscv
"""

import os
import random
import sys
import time
from pathlib import Path

sys.dont_write_bytecode = True  # the reference tree is read-only

SPECIAL_TOKENS = ["<tool_call>", "</tool_call>", "<tool_response>", "</tool_response>", "<think>",
                  "</think>", "<|im_start|>", "<|im_end|>"]
PRINTED_SPECIALS = ["<tool_response>", "</tool_response>", "<think>", "</think>"]  # putchar(256 + k)
# the pieces Qwen's tool-call syntax is written in (each within a 16-byte text row)
CALL_TOKENS = ["<function=", "calc>", "<parameter=", "expression>", "</parameter>", "</function>"]


class ByteVocab:
    """The text bridge's view of a vocabulary (the interface of ``chipformer.rv.bridge.Text``,
    ERV/chipformer/rv/bridge.py:45-91): token q < 256 is the byte q, then Qwen's special tokens,
    then the tool-call pieces (CALL_TOKENS), then ``n_words`` seeded multi-byte tokens (2 to 8
    printable ASCII bytes).  ``printable[b]`` is the token of byte b (b < 256), then the four
    specials the firmware prints."""

    def __init__(self, n_words: int = 4096, seed: int = 35):
        from chipformer.rv import spec as S

        self._row = S.TEXT_ROW
        rng = random.Random(seed)
        self.bytes = [bytes([b]) for b in range(256)] + [s.encode() for s in SPECIAL_TOKENS + CALL_TOKENS]
        seen = set(self.bytes)
        while len(self.bytes) < 256 + len(SPECIAL_TOKENS) + len(CALL_TOKENS) + n_words:
            w = bytes(rng.randrange(0x21, 0x7F) for _ in range(rng.randint(2, 8)))
            if w not in seen:
                seen.add(w)
                self.bytes.append(w)
        self.n = len(self.bytes)
        ids = {s: 256 + i for i, s in enumerate(SPECIAL_TOKENS + CALL_TOKENS)}
        self.ids = ids
        self.TCO, self.TCC = ids["<tool_call>"], ids["</tool_call>"]
        self.printable = list(range(256)) + [ids[s] for s in PRINTED_SPECIALS]
        self.pindex = {q: p for p, q in enumerate(self.printable)}
        self.NL = self.printable[10]

    def printable_index(self, qid: int):
        return self.pindex.get(qid)

    def row_bytes(self, qid: int) -> bytes:
        b = self.bytes[qid] if 0 <= qid < self.n else b""
        return b[:self._row].ljust(self._row, bytes(1))


def main(ref_root: str) -> None:
    sys.path.insert(0, ref_root)
    sys.path.insert(0, str(Path(__file__).resolve().parents[2]))
    from chipformer.rv import core

    from qwenputer_b200.graphfile import default_graph_path, export_graph, merged_graph_path, save_graph

    for path, text in ((default_graph_path(), None), (merged_graph_path(), ByteVocab())):
        t0 = time.time()
        c = core.build(text=text)
        g = export_graph(c)
        save_graph(g, path)
        print(f"exported {c.stats()} in {time.time() - t0:.1f} s -> {path} ({path.stat().st_size} bytes)")


if __name__ == "__main__":
    root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("QX_REFERENCE_ROOT")
    if not root:
        sys.exit("usage: export_rv32im.py REFERENCE/experimental/riscv (or set QX_REFERENCE_ROOT)")
    main(root)
