"""The C oracle against the reference's own WGSL kernels.

tests/golden/wgsl_golden.npz holds the inputs and outputs of each kernel of
LlamaWgslEngine.runToken as the reference's shader text computes them (run
on the CPU by oracle/wgsl.py; tests/golden/make_wgsl_golden.py made the
file).  Here every kernel's restatement in oracle/oracle.c runs on the same
inputs:

* bit for bit where the kernel's arithmetic is fully specified: the five
  GGUF matvecs (per-thread stride-128 sums and the 128-wide tree, the
  oracle's WGSL mode), the embeddings, ADD / ADD_CLAMP, argmax stages 1 and
  2 with the repetition penalty, a NaN and ties;
* within stated tolerances where the shader goes through a builtin whose
  last bits WGSL leaves to the implementation (inverseSqrt, pow, cos, sin,
  exp, tanh): the interpreter evaluates those correctly rounded, the
  oracle with the C library's single-precision functions.
"""
import json
import os

import numpy as np
import pytest

from chonklm_b200.gguf import GGML_TYPE
from oracle import oracle

with np.load(os.path.join(os.path.dirname(__file__), "golden", "wgsl_golden.npz")) as _f:
    G = {k: np.ascontiguousarray(_f[k]) for k in _f.files}   # loaded once: the oracle gets live pointers
CFG = json.loads(bytes(G["config"]).decode())
L = oracle.lib()

# max |oracle - shader| / max |shader| for kernels through implementation-
# defined builtins (a few single-precision ulps)
TOL_NORM = 2e-6      # inverseSqrt
TOL_ROPE = 4e-6      # pow, cos, sin of angles up to ~9 rad
TOL_EXP = 2e-6       # exp, tanh


def p(a):
    return a.ctypes.data


def bits_equal(a, b):
    return np.array_equal(np.asarray(a, np.float32).view(np.uint32), np.asarray(b, np.float32).view(np.uint32))


def rel(a, b):
    return float(np.abs(np.asarray(a, np.float64) - np.asarray(b, np.float64)).max() / max(np.abs(b).max(), 1e-30))


TYPES = {"q4_k": GGML_TYPE.Q4_K, "q6_k": GGML_TYPE.Q6_K, "q8_0": GGML_TYPE.Q8_0, "q5_0": GGML_TYPE.Q5_0,
         "q5_1": GGML_TYPE.Q5_1}
MV = sorted({k.rsplit(".", 1)[0] for k in G if k.startswith("mv_")})


@pytest.mark.parametrize("tag", MV)
def test_matvec_bit_exact(tag):
    key, shape = tag[3:].rsplit("_", 1)
    k, n = map(int, shape.split("x"))
    y = oracle.matvec(TYPES[key], G[tag + ".w"], k, n, G[tag + ".x"], oracle.MODE_WGSL)
    assert bits_equal(y, G[tag + ".y"]), (y, G[tag + ".y"])


@pytest.mark.parametrize("key", sorted(TYPES))
def test_embedding_bit_exact(key):
    if f"emb_{key}.w" not in G:
        pytest.skip("the reference has no embedding shader for this type")
    k, token = 512, 4
    out = np.zeros(k, np.float32)
    w = np.ascontiguousarray(G[f"emb_{key}.w"])
    L.or_embedding(TYPES[key], p(w), k, token, np.float32(CFG["embedding_scale"]), p(out))
    assert bits_equal(out, G[f"emb_{key}.y"])


def test_f32_embedding_bit_exact():
    table = np.ascontiguousarray(G["emb_f32.table"])
    assert bits_equal(table[4], G["emb_f32.y"])


def test_rms_norms():
    H = CFG["hidden"]
    out = np.zeros(H, np.float32)
    L.or_rms_norm(p(G["rms.x"]), p(G["rms.w"]), p(out), H, np.float32(CFG["norm_eps"]))
    assert rel(out, G["rms.y"]) < TOL_NORM
    io = G["addrms.io_in"].copy()
    out = np.zeros(H, np.float32)
    L.or_add_rms_norm(p(G["addrms.a"]), p(io), p(G["rms.w"]), p(out), H, np.float32(CFG["norm_eps"]))
    assert bits_equal(io, G["addrms.io"])            # the residual sum is exact
    assert rel(out, G["addrms.y"]) < TOL_NORM


@pytest.mark.parametrize("layout", ["split", "interleaved"])
def test_rope_store(layout):
    hd, nh, nkv, ctx, pos = CFG["head_dim"], CFG["heads"], CFG["kv_heads"], CFG["max_context"], 9
    t = f"rope_{layout}"
    q = G[t + ".q_in"].copy()
    kc = np.zeros(nkv * ctx * hd, np.float32)
    vc = np.zeros(nkv * ctx * hd, np.float32)
    L.or_rope_store(p(q), p(G[t + ".k"]), p(G[t + ".v"]), p(kc), p(vc), nh, nkv, hd, ctx, pos,
                    int(CFG["rope_theta"]), 1 if layout == "interleaved" else 0)
    assert rel(q, G[t + ".q"]) < TOL_ROPE
    assert rel(kc, G[t + ".kc"]) < TOL_ROPE
    assert bits_equal(vc, G[t + ".vc"])              # V is stored as is


@pytest.mark.parametrize("layout", ["split", "interleaved"])
def test_qk_norm_rope_store(layout):
    hd, nh, nkv, ctx, pos = CFG["head_dim"], CFG["heads"], CFG["kv_heads"], CFG["max_context"], 9
    t = f"qknorm_{layout}"
    qo = np.zeros(nh * hd, np.float32)
    kc = np.zeros(nkv * ctx * hd, np.float32)
    vc = np.zeros(nkv * ctx * hd, np.float32)
    L.or_qk_norm_rope_store(p(G[t + ".q"]), p(G[t + ".k"]), p(G[t + ".v"]), p(G[t + ".qw"]), p(G[t + ".kw"]),
                            p(qo), p(kc), p(vc), nh, nkv, hd, ctx, pos, int(CFG["rope_theta"]),
                            np.float32(CFG["qk_norm_eps"]), 1 if layout == "interleaved" else 0)
    assert rel(qo, G[t + ".q_out"]) < TOL_ROPE
    assert rel(kc, G[t + ".kc"]) < TOL_ROPE
    assert bits_equal(vc, G[t + ".vc"])


@pytest.mark.parametrize("window", [0, 4])
def test_attention(window):
    hd, nh, nkv, ctx, pos = CFG["head_dim"], CFG["heads"], CFG["kv_heads"], CFG["max_context"], 9
    t = f"attn_w{window}"
    out = np.zeros(nh * hd, np.float32)
    scores = np.zeros(nh * ctx, np.float32)
    L.or_attention(p(G[t + ".q"]), p(G[t + ".kc"]), p(G[t + ".vc"]), p(out), p(scores), nh, nkv, hd, ctx, pos,
                   window, np.float32(1.0 / np.sqrt(hd)), oracle.MODE_WGSL)
    # (the oracle reuses `scores` for the softmax weights exp(s - max); the
    # shader keeps the raw scaled scores there: the outputs are compared)
    assert rel(out, G[t + ".out"]) < TOL_EXP


def test_add_and_clamp_bit_exact():
    io = G["add.io_in"].copy()
    L.or_add(p(G["add.a"]), p(io), io.size, 0)
    assert bits_equal(io, G["add.io"])
    io = G["add.io_in"].copy()
    L.or_add(p(G["addclamp.a"]), p(io), io.size, 1)
    assert bits_equal(io, G["addclamp.io"])
    assert np.abs(io).max() <= 65000.0


@pytest.mark.parametrize("tag,fn", [("silu", "or_silu_mul"), ("gelu", "or_gelu_tanh_mul")])
def test_gated_activations(tag, fn):
    out = np.zeros(G[tag + ".g"].size, np.float32)
    getattr(L, fn)(p(G[tag + ".g"]), p(G[tag + ".u"]), p(out), out.size)
    assert rel(out, G[tag + ".out"]) < TOL_EXP


def test_argmax_stages_exact():
    logits = np.ascontiguousarray(G["argmax.logits"])
    pen = np.ascontiguousarray(G["argmax.pen"])
    groups = (logits.size + 255) // 256
    cv = np.zeros(groups, np.float32)
    ci = np.zeros(groups, np.uint32)
    L.or_argmax_stage1(p(logits), logits.size, p(pen), pen.size, int(G["argmax.milli"][0]), p(cv), p(ci))
    assert bits_equal(cv, G["argmax.cand_val"])
    assert np.array_equal(ci, G["argmax.cand_idx"])
    assert L.or_argmax_stage2(p(cv), p(ci), groups) == int(G["argmax.result"][0])
    # the penalised maximum (id 10) lost; the tie at 4.5 went to the lower id
    # among the unpenalised (300, 650): 300
    assert int(G["argmax.result"][0]) == 300
