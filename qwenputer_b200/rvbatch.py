"""Batched conversations with the machine: the executor's merged graph inside a Qwen3.5 decode loop.

The reference's ``RvBatch`` (``ERV/chipformer/rv/rvbatch.py:55-195``) runs N conversations of
``RvChat`` (``ERV/chipformer/rv/chat.py:323-432``): a batched Qwen step for text, and per row a
batch-1 ``ExecRow`` for the chip bursts, whose tokens Qwen never sees (decoding with transparent
chip tokens; the bridge, ``ERV/chipformer/rv/bridge.py:1-21``).  Here one executor holds every
row's machine (the merged graph, ``graphfile.merged_graph_path()``), so a tool call's whole run —
GO, the records, each putchar's echo, ``</tool_response>`` — is generated on the device for all
rows at once, and the Qwen layers read only text: the prompt, then the echoed tool response.

The Qwen side is stock transformers ``Qwen3_5ForCausalLM`` modules with random weights at
Qwen3.5-4B's shape (hidden 2,560, 32 layers, 16 key / 32 value DeltaNet heads, intermediate
9,216: the reference's ``core.T4B`` and its size notes; the full-attention layout, three linear
layers to one full-attention layer with 16 query / 4 key-value heads of dim 256, is the family's
default in transformers, as the 4B checkpoint's own config is not available), in bf16 or with fp8
e4m3 weights (per-output-channel scales; the activations quantised per token at run time, so the
products run as ``torch._scaled_mm``).  The compiled machine computes in fp32 as everywhere else.

    python -m qwenputer_b200.rvbatch [--batch 64 --prompt 512 --fp8 0|1]

prints one JSON line: every row's tool response checked against A*B, and the time and tokens of
each stage.
"""

from __future__ import annotations

import argparse
import json
import random
import time

import numpy as np

from .calc import calc_program, expected_response
from .graphfile import TEXT_TOKEN, load_graph, merged_graph_path

QWEN35_4B = dict(hidden_size=2560, num_hidden_layers=32, intermediate_size=9216, linear_num_key_heads=16,
                 linear_num_value_heads=32, linear_key_head_dim=128, linear_value_head_dim=128,
                 linear_conv_kernel_dim=4, num_attention_heads=16, num_key_value_heads=4, head_dim=256,
                 hidden_act="silu", rms_norm_eps=1e-6, tie_word_embeddings=True)


def _text_ids(g) -> dict:
    """Token ids of the graph's byte-level vocabulary: bytes, <tool_call>, </tool_call>, the
    tool-call pieces, and the ids a random prompt may use (no special token, no call piece)."""
    words = g.text_words
    row = [bytes(sum(((int(words[q, (8 * k + i) >> 5]) >> ((8 * k + i) & 31)) & 1) << i for i in range(8))
                 for k in range(16)).rstrip(b"\0") for q in range(len(words))]
    by = {b: q for q, b in enumerate(row)}
    tco = next(q for q in range(len(words)) if words[q, 4] & 1)
    tcc = next(q for q in range(len(words)) if words[q, 4] >> 1 & 1)
    pieces = ["<function=", "calc>", "<parameter=", "expression>", "</parameter>", "</function>",
              "</tool_response>"]
    ids = {p: by[p.encode()] for p in pieces}
    free = [q for q, b in enumerate(row) if q not in (tco, tcc) and not b.startswith(b"<") and b]
    return {"tco": tco, "tcc": tcc, "byte": lambda c: by[bytes([c])], "pieces": ids, "free": free, "bytes": row}


def prompts(g, batch: int, length: int, seed: int = 0) -> list[tuple[list[int], int, int]]:
    """Per row: `length` text tokens (seeded random vocabulary ids) ending in Qwen's tool-call
    syntax naming calc with A*B, A and B random 9-18 digit integers (chip stream ids:
    TEXT_TOKEN | qid)."""
    v = _text_ids(g)
    P = v["pieces"]
    rng = random.Random(seed)
    out = []
    for _ in range(batch):
        a, b = (rng.randint(10 ** (d - 1), 10 ** d - 1) for d in (rng.randint(9, 18), rng.randint(9, 18)))
        nl = v["byte"](10)
        call = ([v["tco"], nl, P["<function="], P["calc>"], nl, P["<parameter="], P["expression>"], nl]
                + [v["byte"](c) for c in str(a).encode()] + [v["byte"](ord("*"))]
                + [v["byte"](c) for c in str(b).encode()]
                + [nl, P["</parameter>"], nl, P["</function>"], nl, v["tcc"]])
        pre = [rng.choice(v["free"]) for _ in range(length - len(call))]  # </tool_call> ends every row
        out.append(([TEXT_TOKEN + q for q in pre + call], a, b))
    return out


class Fp8Linear:
    """A Linear with fp8 e4m3 weights and a per-output-channel scale; the input is quantised
    per token to e4m3 at run time and the product runs as torch._scaled_mm (bf16 out)."""

    @staticmethod
    def convert(model) -> int:
        import torch

        n = 0
        for name, mod in list(model.named_modules()):
            for cname, child in list(mod.named_children()):
                if isinstance(child, torch.nn.Linear) and "lm_head" not in cname and \
                        child.in_features % 16 == 0 and child.out_features % 16 == 0:
                    setattr(mod, cname, _Fp8Module(child))
                    n += 1
        return n


def _fp8_module_class():
    import torch

    class Fp8(torch.nn.Module):
        def __init__(self, lin):
            super().__init__()
            w = lin.weight.detach().float()
            s = (w.abs().amax(dim=1, keepdim=True) / 448.0).clamp(min=1e-12)
            self.register_buffer("w", (w / s).to(torch.float8_e4m3fn).contiguous())  # [out, in]
            self.register_buffer("sw", s.reshape(1, -1).float())  # [1, out]
            self.bias = lin.bias

        def forward(self, x):
            shp = x.shape
            x2 = x.reshape(-1, shp[-1])
            sx = (x2.abs().amax(dim=1, keepdim=True).float() / 448.0).clamp(min=1e-12)
            xq = (x2.float() / sx).to(torch.float8_e4m3fn)
            y = torch._scaled_mm(xq, self.w.t(), scale_a=sx, scale_b=self.sw, out_dtype=torch.bfloat16)
            if self.bias is not None:
                y = y + self.bias
            return y.reshape(*shp[:-1], -1)

    return Fp8


_FP8 = None


def _Fp8Module(lin):
    global _FP8
    if _FP8 is None:
        _FP8 = _fp8_module_class()
    return _FP8(lin)


def qwen_text_model(vocab: int, layers: int = 32, fp8: bool = False, seed: int = 0, device="cuda"):
    """Random-init Qwen3.5-4B-shaped text layers (bf16; fp8 e4m3 linear weights with fp8)."""
    import torch
    from transformers import Qwen3_5ForCausalLM, Qwen3_5TextConfig

    cfg = dict(QWEN35_4B, num_hidden_layers=layers, vocab_size=-(-vocab // 64) * 64)
    cfg["layer_types"] = [("full_attention" if i % 4 == 3 else "linear_attention") for i in range(layers)]
    torch.manual_seed(seed)
    with torch.device(device):
        model = Qwen3_5ForCausalLM(Qwen3_5TextConfig(**cfg)).to(torch.bfloat16).eval()
    n = Fp8Linear.convert(model) if fp8 else 0
    return model, n


def park(programs, max_tokens: int = 4096) -> list:
    """Each firmware run from its image to its first park (the exit ecall: HALT), as the bridge
    starts it (ERV/chipformer/rv/bridge.py:106-111): free running on a standalone executor one
    token a launch; a machine's state (x, anchor, n, RAM) is read back from the heads once its
    HALT has been consumed as an input too (a record commits as its tokens are read: the exit's
    n + 1, ref.py:526-529, lands then)."""
    import torch

    from .executor import Executor

    ex = Executor(None, batch=len(programs))
    ex.load_machines(0, programs)
    ex.reset()
    g = ex.g
    go = int(g.fam_ids[list(g.fam_names).index("GO")])
    ex.set_tokens(0, [go] * len(programs))
    one = torch.empty(1, len(programs), dtype=torch.int32, device=ex.dev)
    out: list = [None] * len(programs)
    for _ in range(max_tokens):
        ex.run(1, one)
        halt, count = ex.halt_at.cpu().numpy(), ex.count.cpu().numpy()
        for r in np.flatnonzero((halt >= 0) & (count == halt + 1)):
            if out[r] is None:
                st = ex.readback(int(r))
                out[r] = (list(st.x), int(st.anchor), int(st.n), np.ctypeslib.as_array(st.ram).copy())
        if all(o is not None for o in out):
            return out
    raise RuntimeError("a firmware did not park")


def run(batch: int = 64, length: int = 512, fp8: bool = False, layers: int = 32, seed: int = 0,
        chunk: int = 1024, max_chip: int = 20000) -> dict:
    """One batch of conversations; returns the checks and stage timings."""
    import torch

    from .executor import Executor

    g = load_graph(merged_graph_path())
    dev = torch.device("cuda")
    rows = prompts(g, batch, length, seed)
    v = _text_ids(g)
    tre = TEXT_TOKEN + v["pieces"]["</tool_response>"]
    p = calc_program()
    states = park([p] * batch)
    ex = Executor(g, batch=batch, table_images=1)  # every row runs the one firmware: one table copy
    ex.load_machines(0, [p] * batch, states=states)
    model, n_fp8 = qwen_text_model(len(g.text_words), layers, fp8, seed, dev)
    with torch.no_grad():  # warm-up (library initialisation, first-call kernel set-up), untimed
        w = model(input_ids=torch.zeros(batch, 64, dtype=torch.long, device=dev), use_cache=True)
        model(input_ids=torch.zeros(batch, 1, dtype=torch.long, device=dev), past_key_values=w.past_key_values,
              use_cache=True)
        del w
    torch.cuda.synchronize()
    t = {}
    # 1. the prompt: teacher-forced through the executor (text tokens), prefilled into Qwen
    toks = np.asarray([r[0] for r in rows], np.int64)  # [batch, length]
    t0 = time.perf_counter()
    for j in range(length):
        ex.set_tokens(0, toks[:, j].astype(np.int32))
        ex.step(ex.x)
    torch.cuda.synchronize()
    t["chip_prompt_s"] = time.perf_counter() - t0
    qids = torch.from_numpy(toks - TEXT_TOKEN).to(dev)
    t0 = time.perf_counter()
    with torch.no_grad():
        out = model(input_ids=qids, use_cache=True)
    cache = out.past_key_values
    torch.cuda.synchronize()
    t["qwen_prefill_s"] = time.perf_counter() - t0
    # 2. the tool call's run: the circuit owns the stream from </tool_call>; the device decodes
    #    and embeds every token (chip tokens and echoes) until each row has echoed </tool_response>
    go = [g.decode(x) for x in ex.x.cpu().numpy()]
    ex.set_tokens(0, go)
    gen, done, n_chip = [], np.zeros(batch, bool), 0
    t0 = time.perf_counter()
    buf = torch.empty(chunk, batch, dtype=torch.int32, device=dev)
    while not done.all() and n_chip < max_chip:
        ex.run(chunk, buf)
        part = buf.cpu().numpy()
        gen.append(part)
        n_chip += chunk
        done |= (part == tre).any(axis=0) | (part == -1).any(axis=0)
    torch.cuda.synchronize()
    t["chip_run_s"] = time.perf_counter() - t0
    stream = np.concatenate([np.asarray(go, np.int64)[None]] + [x.astype(np.int64) for x in gen]).T
    # 3. the echoes (text) to Qwen, one position at a time, up to and including </tool_response>
    echoes = []
    for r in range(batch):
        e = []
        for tok in stream[r]:
            if tok >= TEXT_TOKEN:
                e.append(int(tok) - TEXT_TOKEN)
                if int(tok) == tre:
                    break
        echoes.append(e)
    E = max(len(e) for e in echoes)
    t0 = time.perf_counter()
    with torch.no_grad():
        for j in range(E):
            col = torch.tensor([e[j] if j < len(e) else e[-1] for e in echoes], device=dev)[:, None]
            out = model(input_ids=col, past_key_values=cache, use_cache=True)
            cache = out.past_key_values
    torch.cuda.synchronize()
    t["qwen_echo_s"] = time.perf_counter() - t0
    # checks: every row's tool response is A*B's
    ok = 0
    for (_, a, b), e in zip(rows, echoes):
        text = b"".join(v["bytes"][q] for q in e)
        ok += text == expected_response(a, b)[:len(text)] and text.endswith(b"</tool_response>")
    chip_tokens = int(sum(int(np.argmax(stream[r] == tre)) + 1 for r in range(batch)))
    text_tokens = batch * length + sum(len(e) for e in echoes)
    total = sum(t.values())
    return {"workload": "merged machine + Qwen3.5-4B-shaped layers (random init), calc tool calls A*B",
            "batch": batch, "prompt_tokens": length, "qwen_layers": layers,
            "qwen_weights": "fp8 e4m3, per-channel scales (W8A8 torch._scaled_mm)" if fp8 else "bf16",
            "fp8_linears": n_fp8, "rows_correct": ok, "chip_tokens": chip_tokens, "text_tokens": text_tokens,
            "seconds": t, "tokens_per_s": (chip_tokens + text_tokens) / total,
            "chip_tokens_per_s_in_run": chip_tokens / t["chip_run_s"], "device_errors": ex.errors()}


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--batch", type=int, default=64)
    ap.add_argument("--prompt", type=int, default=512)
    ap.add_argument("--fp8", type=int, default=0, choices=[0, 1])
    ap.add_argument("--layers", type=int, default=32)
    ap.add_argument("--seed", type=int, default=0)
    a = ap.parse_args()
    print(json.dumps(run(a.batch, a.prompt, bool(a.fp8), a.layers, a.seed)))


if __name__ == "__main__":
    main()
