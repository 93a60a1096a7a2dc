"""Golden vectors from the reference's own WGSL kernels, run on the CPU.

Usage (in a checkout that has the reference next to it; the vectors are
committed, the reference is not needed afterwards):

    python tests/golden/make_wgsl_golden.py <reference root>

For each kernel of LlamaWgslEngine.runToken (src/lib/llama-wgsl-runtime.ts:
the GGUF Q4_K / Q6_K / Q8_0 / Q5_0 / Q5_1 matvecs and embeddings, the f32
embedding, RMS_NORM, ADD_RMS_NORM, ROPE_STORE (split and interleaved),
QK_NORM_ROPE_STORE (split and interleaved), ATTENTION_SCORE +
ATTENTION_VALUE with and without a sliding window, ADD, ADD_CLAMP,
SILU_MUL, GELU_TANH_MUL, ARGMAX_STAGE1 with a repetition penalty, NaN and
ties, ARGMAX_STAGE2) this script reads the shader text from the reference
source, prepends the constants block the reference's createPipelines
builds for a model (:1695-1712), fills the buffers and uniforms as the
engine's dispatch does, runs it with oracle/wgsl.py and writes the inputs
and outputs to tests/golden/wgsl_golden.npz.  tests/test_wgsl_golden.py
checks the C oracle's restatement of each kernel against them.  The Q5_1
matvec shader is derived the way the reference derives it (:2280-2289): the
`.replace(...)` chain after its definition is read from the source and
applied to the Q5_0 text.  No reference text is stored, only numbers.
"""
from __future__ import annotations

import decimal
import math
import json
import os
import re
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle import wgsl  # noqa: E402

SRC = "src/lib/llama-wgsl-runtime.ts"

# a small model: the constants block and the dispatch shapes follow from it
CFG = {"hidden": 256, "intermediate": 320, "heads": 4, "kv_heads": 2, "head_dim": 64, "rope_theta": 10000.0,
       "norm_eps": 1e-5, "qk_norm_eps": 1e-6, "embedding_scale": 1.0, "max_context": 16}


def js_number(x: float) -> str:
    """Number.prototype.toString for a finite double (ECMAScript
    Number::toString: shortest round-trip digits, fixed notation for
    decimal exponents in (-7, 21])."""
    if x == 0:
        return "0"
    sign = "-" if x < 0 else ""
    d = decimal.Decimal(repr(abs(float(x))))
    t = d.as_tuple()
    digits = "".join(map(str, t.digits)).rstrip("0") or "0"
    k = len(digits)
    n = len(t.digits) + t.exponent           # value = 0.digits x 10^n
    if k <= n <= 21:
        return sign + digits + "0" * (n - k)
    if 0 < n <= 21:
        return sign + digits[:n] + "." + digits[n:]
    if -6 < n <= 0:
        return sign + "0." + "0" * (-n) + digits
    e = n - 1
    return sign + digits[0] + ("." + digits[1:] if k > 1 else "") + "e" + ("+" if e >= 0 else "-") + str(abs(e))


def constants_block(c: dict) -> str:
    """The WGSL constants createPipelines prepends to every shader."""
    lines = [
        f"const HIDDEN: u32 = {c['hidden']}u;",
        f"const EMBEDDING_DIM: u32 = {c['hidden']}u;",
        f"const INTERMEDIATE: u32 = {c['intermediate']}u;",
        f"const HEADS: u32 = {c['heads']}u;",
        f"const KV_HEADS: u32 = {c['kv_heads']}u;",
        f"const HEAD_DIM: u32 = {c['head_dim']}u;",
        f"const ROTARY_HALF: u32 = {c['head_dim'] // 2}u;",
        f"const KV_GROUP: u32 = {c['heads'] // c['kv_heads']}u;",
        f"const KV_DIM: u32 = {c['kv_heads'] * c['head_dim']}u;",
        f"const ROPE_THETA: f32 = {c['rope_theta']:.1f};",
        f"const NORM_EPS: f32 = {js_number(c['norm_eps'])};",
        f"const QK_NORM_EPS: f32 = {js_number(c['qk_norm_eps'])};",
        f"const ATTN_SCALE: f32 = {js_number(1.0 / math.sqrt(c['head_dim']))};",
        f"const EMBEDDING_SCALE: f32 = {js_number(c['embedding_scale'])};",
    ]
    return "\n" + "\n".join(lines) + "\n"


def _js_string(lit: str) -> str:
    return json.loads(lit)


def _read_literal(src: str, i: int):
    """A JS string ("...") or regex (/.../flags) literal at src[i]: (kind,
    text, end)."""
    q = src[i]
    j = i + 1
    while src[j] != q:
        j += 2 if src[j] == "\\" else 1
    if q == '"':
        return "str", json.loads(src[i:j + 1]), j + 1
    k = j + 1
    while src[k].isalpha():
        k += 1
    return "re", src[i + 1:j], k


def derived_shaders(src: str, shaders: dict) -> dict:
    """Shaders the reference builds from another one by a chain of
    String.prototype.replace calls (`const B = A.replace(p, s)...;`)."""
    out = {}
    for m in re.finditer(r"const (\w+_WGSL) = (\w+_WGSL)\b", src):
        name, base = m.groups()
        text, i = shaders[base], m.end()
        while True:
            while src[i].isspace():
                i += 1
            if not src.startswith(".replace(", i):
                break
            i += len(".replace(")
            while src[i].isspace():
                i += 1
            kind, pat, i = _read_literal(src, i)
            while src[i] in " \n,":
                i += 1
            _, rep, i = _read_literal(src, i)
            while src[i] in " \n,":
                i += 1
            assert src[i] == ")", src[i:i + 20]
            i += 1
            text = re.sub(pat, lambda _m: rep, text) if kind == "re" else text.replace(pat, rep, 1)
        out[name] = text
    return out


def main(ref_root: str) -> None:
    ts = open(os.path.join(ref_root, SRC)).read()
    shaders = wgsl.extract_shaders(ts)
    shaders.update(derived_shaders(ts, shaders))
    pre = constants_block(CFG)
    rng = np.random.default_rng(2024)
    gold = {"config": np.frombuffer(json.dumps(CFG).encode(), dtype=np.uint8)}

    def run(name, groups, bufs):
        wgsl.Shader(pre + shaders[name]).run("main", groups, bufs)

    sys.path.insert(0, ROOT)
    import torch
    from chonklm_b200.gguf import GGML_TYPE
    from chonklm_b200.quant import quantize

    qtypes = {"q4_k": (GGML_TYPE.Q4_K, "GGUF_Q4_K", 144, 256), "q6_k": (GGML_TYPE.Q6_K, "GGUF_Q6_K", 210, 256),
              "q8_0": (GGML_TYPE.Q8_0, "GGUF_Q8_0", 34, 32), "q5_0": (GGML_TYPE.Q5_0, "GGUF_Q5_0", 22, 32),
              "q5_1": (GGML_TYPE.Q5_1, "GGUF_Q5_1", 24, 32)}
    # --- matvec and embedding per block type -------------------------------
    for key, (t, prefix, bb, bw) in qtypes.items():
        for k, n in ((512, 5), (96, 3)) if bw == 32 else ((512, 5), (256, 3)):
            w = torch.tensor(rng.standard_normal((n, k)).astype(np.float32) * 0.05)
            data = np.frombuffer(quantize(w, t), dtype=np.uint8).copy()
            pad = (-data.size) % 4
            words = np.concatenate([data, np.zeros(pad, np.uint8)]).view(np.uint32).copy()
            x = rng.standard_normal(k).astype(np.float32)
            y = np.zeros(n, np.float32)
            run(prefix + "_MATVEC_WGSL", (n, 1, 1),
                {"input": x, "data": words, "output": y,
                 "params": {"k": k, "n": n, "block_bytes": bb, "x_groups": n}})
            tag = f"mv_{key}_{k}x{n}"
            gold[tag + ".w"], gold[tag + ".x"], gold[tag + ".y"] = data, x, y
            if (prefix + "_EMBEDDING_WGSL") in shaders and k == 512:
                out = np.zeros(k, np.float32)
                run(prefix + "_EMBEDDING_WGSL", ((k + 127) // 128, 1, 1),
                    {"data": words, "output": out, "params": {"token": n - 1, "k": k, "block_bytes": bb}})
                gold[f"emb_{key}.w"], gold[f"emb_{key}.y"] = data, out
    # f32 embedding table
    table = rng.standard_normal((6, CFG["hidden"])).astype(np.float32)
    out = np.zeros(CFG["hidden"], np.float32)
    run("EMBEDDING_WGSL", ((CFG["hidden"] + 127) // 128, 1, 1),
        {"embedding": table.ravel().copy(), "output": out, "params": {"token": 4, "rows": 6}})
    gold["emb_f32.table"], gold["emb_f32.y"] = table, out

    # --- norms ------------------------------------------------------------------
    H = CFG["hidden"]
    x = rng.standard_normal(H).astype(np.float32)
    w = (1.0 + 0.1 * rng.standard_normal(H)).astype(np.float32)
    out = np.zeros(H, np.float32)
    run("RMS_NORM_WGSL", (1, 1, 1), {"input": x, "weight": w, "output": out, "params": {"n": H}})
    gold["rms.x"], gold["rms.w"], gold["rms.y"] = x, w, out
    a = rng.standard_normal(H).astype(np.float32)
    io = x.copy()
    out = np.zeros(H, np.float32)
    run("ADD_RMS_NORM_WGSL", (1, 1, 1), {"a": a, "io": io, "weight": w, "output": out, "params": {"n": H}})
    gold["addrms.a"], gold["addrms.io_in"], gold["addrms.io"], gold["addrms.y"] = a, x, io, out

    # --- rope + KV store, plain and with the per-head norm -------------------------
    hd, nh, nkv, ctx, pos = CFG["head_dim"], CFG["heads"], CFG["kv_heads"], CFG["max_context"], 9
    rp = {"pos": pos, "max_context": ctx, "heads": nh, "kv_heads": nkv, "rope_theta": int(CFG["rope_theta"])}
    for layout, sfx in (("split", ""), ("interleaved", "_INTERLEAVED")):
        q = rng.standard_normal(nh * hd).astype(np.float32)
        k_ = rng.standard_normal(nkv * hd).astype(np.float32)
        v = rng.standard_normal(nkv * hd).astype(np.float32)
        qq = q.copy()
        kc = np.zeros(nkv * ctx * hd, np.float32)
        vc = np.zeros(nkv * ctx * hd, np.float32)
        run("ROPE_STORE" + sfx + "_WGSL", ((nh * hd // 2 + 127) // 128, 1, 1),
            {"q": qq, "k": k_, "v": v, "key_cache": kc, "value_cache": vc, "params": rp})
        tag = f"rope_{layout}"
        gold[tag + ".q_in"], gold[tag + ".k"], gold[tag + ".v"] = q, k_, v
        gold[tag + ".q"], gold[tag + ".kc"], gold[tag + ".vc"] = qq, kc, vc
        qw = (1.0 + 0.1 * rng.standard_normal(hd)).astype(np.float32)
        kw = (1.0 + 0.1 * rng.standard_normal(hd)).astype(np.float32)
        qo = np.zeros(nh * hd, np.float32)
        kc = np.zeros(nkv * ctx * hd, np.float32)
        vc = np.zeros(nkv * ctx * hd, np.float32)
        run("QK_NORM_ROPE_STORE" + sfx + "_WGSL", (nh, 1, 1),
            {"q": q, "k": k_, "v": v, "q_weight": qw, "k_weight": kw, "q_out": qo, "key_cache": kc,
             "value_cache": vc, "params": rp})
        tag = f"qknorm_{layout}"
        gold[tag + ".q"], gold[tag + ".k"], gold[tag + ".v"], gold[tag + ".qw"], gold[tag + ".kw"] = q, k_, v, qw, kw
        gold[tag + ".q_out"], gold[tag + ".kc"], gold[tag + ".vc"] = qo, kc, vc

    # --- attention: scores then values, without and with a window ---------------
    for window in (0, 4):
        q = rng.standard_normal(nh * hd).astype(np.float32)
        kc = rng.standard_normal(nkv * ctx * hd).astype(np.float32)
        vc = rng.standard_normal(nkv * ctx * hd).astype(np.float32)
        scores = np.zeros(nh * ctx, np.float32)
        ap = {"pos": pos, "max_context": ctx, "heads": nh, "kv_heads": nkv, "window": window}
        run("ATTENTION_SCORE_WGSL", (nh, pos + 1, 1), {"q": q, "key_cache": kc, "scores": scores, "params": ap})
        out = np.zeros(nh * hd, np.float32)
        run("ATTENTION_VALUE_WGSL", (nh, 1, 1), {"scores": scores, "value_cache": vc, "output": out, "params": ap})
        tag = f"attn_w{window}"
        gold[tag + ".q"], gold[tag + ".kc"], gold[tag + ".vc"] = q, kc, vc
        gold[tag + ".scores"], gold[tag + ".out"] = scores, out

    # --- elementwise --------------------------------------------------------------
    I = CFG["intermediate"]
    a = rng.standard_normal(H).astype(np.float32)
    io = (rng.standard_normal(H) * 40000).astype(np.float32)
    io0 = io.copy()
    run("ADD_WGSL", ((H + 127) // 128, 1, 1), {"a": a, "io": io, "params": {"n": H}})
    gold["add.a"], gold["add.io_in"], gold["add.io"] = a, io0, io
    io = io0.copy()
    run("ADD_CLAMP_WGSL", ((H + 127) // 128, 1, 1), {"a": (a * 40000).astype(np.float32), "io": io, "params": {"n": H}})
    gold["addclamp.a"], gold["addclamp.io"] = (a * 40000).astype(np.float32), io
    g = (rng.standard_normal(I) * 3).astype(np.float32)
    u = rng.standard_normal(I).astype(np.float32)
    for name, tag in (("SILU_MUL_WGSL", "silu"), ("GELU_TANH_MUL_WGSL", "gelu")):
        out = np.zeros(I, np.float32)
        run(name, ((I + 127) // 128, 1, 1), {"gate": g, "up": u, "output": out, "params": {"n": I}})
        gold[tag + ".g"], gold[tag + ".u"], gold[tag + ".out"] = g, u, out

    # --- argmax with a repetition penalty, a NaN and ties ---------------------------
    V = 700
    logits = rng.standard_normal(V).astype(np.float32)
    logits[5] = np.nan
    logits[300] = logits[301] = logits[650] = np.float32(4.5)     # a three-way tie for the maximum
    logits[10] = np.float32(5.5)                                   # the largest until penalised (5.5 / 1.3 < 4.5)
    pen = np.array([10, 301, 42], dtype=np.uint32)
    milli = 1300
    groups = (V + 255) // 256
    parts = np.zeros(groups * 2, np.uint32)                        # Candidate {value: f32, index: u32}
    run("ARGMAX_STAGE1_WGSL", (groups, 1, 1),
        {"logits": logits, "partials": parts, "penalty_ids": pen,
         "params": {"vocab": V, "penalty_count": len(pen), "repetition_penalty_milli": milli}})
    result = np.zeros(1, np.uint32)
    run("ARGMAX_STAGE2_WGSL", (1, 1, 1), {"partials": parts.copy(), "result": result, "params": {"groups": groups}})
    gold["argmax.logits"], gold["argmax.pen"] = logits, pen
    gold["argmax.milli"] = np.array([milli], np.uint32)
    gold["argmax.cand_val"], gold["argmax.cand_idx"] = parts[0::2].view(np.float32).copy(), parts[1::2].copy()
    gold["argmax.result"] = result

    path = os.path.join(HERE, "wgsl_golden.npz")
    np.savez_compressed(path, **gold)
    print(f"wrote {path}: {len(gold)} arrays")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit(__doc__)
    main(sys.argv[1])
