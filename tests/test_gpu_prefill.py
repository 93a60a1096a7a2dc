"""Tensor-core prefill (ck_set_prefill_gemm): a prompt's tokens through the
layers together as tcgen05 GEMMs, K/V rows written into the engine's cache.

The reference prefills token by token (generateLlamaWgsl, runToken per
prompt id); the results must equal that sequence of steps within the decode
tolerance: logits after the prompt within 1e-3 of the oracle (max |gpu -
oracle| / max |oracle| over the vocabulary), the following greedy ids
identical wherever the oracle's top two logits are further apart than the
tolerance."""
import numpy as np
import pytest

from conftest import tiny_model
from chonklm_b200.registry import ModelDef
from chonklm_b200.runtime import loadLlamaWgslModel
from oracle import oracle

pytestmark = pytest.mark.gpu

LOGIT_TOL = 1e-3


def _load(path, kv="float16", ctx=256):
    import gguf as ggufpy
    r = ggufpy.GGUFReader(path)
    V = int([t for t in r.tensors if t.name == "token_embd.weight"][0].shape[1])
    d = ModelDef(id="t", label="t", vocab=V, layers=0, kvHeads=0, headDim=0, maxContext=ctx, gguf=path,
                 kvDtype=kv, eosIds=[])
    return loadLlamaWgslModel(d), V


def _rel(a, b):
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


def _clear(lo, tol):
    top2 = np.sort(lo)[-2:]
    return top2[1] - top2[0] > 4 * tol * np.abs(lo).max()


def _continue(eng, orc, nid, oid, steps, tol):
    """Greedy decode after the prompt on both sides, fed the oracle's ids."""
    for i in range(steps):
        gid = eng.run_token(oid, True)
        oid2 = orc.run_token(oid, True)
        lg, lo = eng.logits(), orc.logits()
        assert _rel(lg, lo) < tol, f"decode step {i}: {_rel(lg, lo)}"
        if _clear(lo, tol):
            assert gid == oid2, f"decode step {i}: {gid} != {oid2}"
        oid = oid2


SHAPES = {"hd64": {}, "hd128": {"head_dim": 128}, "g3": {"heads": 6, "kv_heads": 2},
          "i544": {"intermediate": 544}}   # not a multiple of 64: gate / up tiles kept apart


@pytest.mark.parametrize("shape", list(SHAPES))
@pytest.mark.parametrize("kv", ["float16", "float32"])
@pytest.mark.parametrize("arch", ["llama", "qwen3"])
def test_gemm_prefill_matches_oracle(tiny_dir, arch, kv, shape):
    """200-token prompts: the attention spans two 128-position chunks (the
    online softmax rescales across them); head_dim 64 and 128, and 3 query
    heads per kv head (42-token query blocks)."""
    path = tiny_model(tiny_dir, arch, "q4_k_m", **SHAPES[shape])
    loaded, V = _load(path, kv)
    eng = loaded.engine.dev
    eng.set_prefill_gemm(2)
    toks = np.random.default_rng(3).integers(0, V, size=200).tolist()
    nid = eng.prefill(toks, True)
    assert eng.position == len(toks)
    orc = oracle.OracleModel(path, max_context=256)
    for t in toks[:-1]:
        orc.run_token(t, False)
    oid = orc.run_token(toks[-1], True)
    lg, lo = eng.logits(), orc.logits()
    assert _rel(lg, lo) < LOGIT_TOL, _rel(lg, lo)
    if _clear(lo, LOGIT_TOL):
        assert nid == oid
    _continue(eng, orc, nid, oid, 16, LOGIT_TOL)
    loaded.engine.dispose()


@pytest.mark.parametrize("arch", ["llama", "qwen3"])
def test_gemm_prefill_chunks_and_offset(tiny_dir, arch):
    """Two prefill calls (the second starts at position 20) in 48-token
    chunks, so attention reads rows written by earlier calls and chunks."""
    path = tiny_model(tiny_dir, arch, "q4_k_m")
    loaded, V = _load(path)
    eng = loaded.engine.dev
    eng.set_prefill_gemm(2, 48)
    toks = np.random.default_rng(9).integers(0, V, size=170).tolist()
    eng.prefill(toks[:20], False)
    nid = eng.prefill(toks[20:], True)
    assert eng.position == 170
    orc = oracle.OracleModel(path, max_context=256)
    for t in toks[:-1]:
        orc.run_token(t, False)
    oid = orc.run_token(toks[-1], True)
    assert _rel(eng.logits(), orc.logits()) < LOGIT_TOL
    _continue(eng, orc, nid, oid, 8, LOGIT_TOL)
    loaded.engine.dispose()


@pytest.mark.parametrize("arch", ["llama", "qwen3"])
def test_gemm_prefill_matches_token_by_token(tiny_dir, arch):
    """The tensor-core prefill against the engine's own token-by-token
    prefill (min_tokens 0) over the same 120-token prompt."""
    path = tiny_model(tiny_dir, arch, "q4_k_m")
    toks = np.random.default_rng(21).integers(0, 512, size=120).tolist()
    out = []
    for mt in (0, 2):
        loaded, V = _load(path)
        eng = loaded.engine.dev
        eng.set_prefill_gemm(mt)
        out.append((eng.prefill([t % V for t in toks], True), eng.logits()))
        loaded.engine.dispose()
    assert _rel(out[1][1], out[0][1]) < LOGIT_TOL


def test_gemm_prefill_unsupported_graph_keeps_token_path(tiny_dir):
    """Graphs outside the tensor-core prefill's set (gemma3) keep the
    token-by-token prefill, bit for bit."""
    path = tiny_model(tiny_dir, "gemma3", "q4_k_m")
    toks = np.random.default_rng(4).integers(0, 256, size=30).tolist()
    out = []
    for mt in (0, 2):
        loaded, V = _load(path)
        eng = loaded.engine.dev
        eng.set_prefill_gemm(mt)
        out.append((eng.prefill([t % V for t in toks], True), eng.logits()))
        loaded.engine.dispose()
    assert out[0][0] == out[1][0]
    assert np.array_equal(out[0][1].view(np.uint32), out[1][1].view(np.uint32))
