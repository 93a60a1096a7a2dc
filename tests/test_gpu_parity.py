"""GPU parity: the CUDA path (through the C ABI) against the CPU oracle.

Tolerances: dequantized weights bit-exact; logits
within 1e-3 max relative error, measured as max|gpu - oracle| / max|oracle|
over the vocabulary; identical greedy ids over 64 tokens.
"""
import math

import numpy as np
import pytest

from conftest import tiny_model
from chonklm_b200 import _lib
from chonklm_b200.gguf import GGML_TYPE
from chonklm_b200.quant import quantize
from chonklm_b200.registry import ModelDef
from chonklm_b200.runtime import generateLlamaWgsl, loadLlamaWgslModel, resetLlamaWgslConversation
from oracle import oracle

pytestmark = pytest.mark.gpu

LOGIT_TOL = 1e-3        # fp16 KV cache (the product default)
LOGIT_TOL_F32KV = 2e-4  # fp32 KV cache: only the matvec's 16-bit activation grid differs
QTYPES = [GGML_TYPE.Q4_K, GGML_TYPE.Q6_K, GGML_TYPE.Q8_0, GGML_TYPE.Q5_0, GGML_TYPE.Q5_1]


def _blocks(t, k, n, seed, scale=0.02):
    import torch
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(n, k, generator=g) * scale
    return quantize(x, t)


def _random_blocks(t, k, n, seed):
    """Arbitrary bytes with finite fp16 scales (subnormals included)."""
    rng = np.random.default_rng(seed)
    bw = {GGML_TYPE.Q4_K: 256, GGML_TYPE.Q6_K: 256}.get(t, 32)
    bb = {GGML_TYPE.Q4_K: 144, GGML_TYPE.Q6_K: 210, GGML_TYPE.Q8_0: 34, GGML_TYPE.Q5_0: 22, GGML_TYPE.Q5_1: 24}[t]
    nb = n * k // bw
    b = rng.integers(0, 256, size=(nb, bb), dtype=np.uint8)
    exps = rng.integers(0, 31, size=(nb, 2))            # exponent 0..30: subnormal or normal, never inf/nan
    halves = ((rng.integers(0, 2, size=(nb, 2)) << 15) | (exps << 10) | rng.integers(0, 1024, size=(nb, 2)))
    halves = halves.astype(np.uint16)
    if t == GGML_TYPE.Q6_K:
        b[:, 208:210] = halves[:, :1].view(np.uint8).reshape(nb, 2)
    else:
        b[:, 0:2] = halves[:, :1].view(np.uint8).reshape(nb, 2)
        if t in (GGML_TYPE.Q4_K, GGML_TYPE.Q5_1):
            b[:, 2:4] = halves[:, 1:2].view(np.uint8).reshape(nb, 2)
    return b.tobytes()


@pytest.mark.parametrize("t", QTYPES)
@pytest.mark.parametrize("kind", ["quantized", "random", "subnormal"])
def test_dequant_bit_exact(t, kind):
    k, n = (512, 48) if t in (GGML_TYPE.Q4_K, GGML_TYPE.Q6_K) else (576, 40)
    if kind == "quantized":
        data = _blocks(t, k, n, 1)
    elif kind == "subnormal":
        data = _blocks(t, k, n, 2, scale=1e-5)          # fp16 d/dmin below 6.1e-5
    else:
        data = _random_blocks(t, k, n, 3)
    gpu = _lib.dequant(t, data, k, n)
    ref = oracle.dequant(t, np.frombuffer(data, np.uint8), k, n)
    assert np.array_equal(gpu.view(np.uint32), ref.view(np.uint32)), \
        f"{np.count_nonzero(gpu.view(np.uint32) != ref.view(np.uint32))} weights differ"


MV_SHAPES = [(256, 7), (576, 130), (1024, 1000), (1536, 77), (2048, 333), (3072, 1024)]
_KQUANTS = (GGML_TYPE.Q4_K, GGML_TYPE.Q6_K)


@pytest.mark.parametrize("t,k,n", [(t, k, n) for t in QTYPES for k, n in MV_SHAPES
                                   if not (t in _KQUANTS and k % 256)])
def test_matvec(t, k, n):
    data = _blocks(t, k, n, k + n)
    rng = np.random.default_rng(k * n)
    x = rng.standard_normal(k).astype(np.float32)
    y = _lib.matvec(t, data, k, n, x)
    ref = oracle.matvec(t, np.frombuffer(data, np.uint8), k, n, x, oracle.MODE_F64)
    err = np.abs(y - ref).max() / np.abs(ref).max()
    assert err < 1e-4, err


@pytest.mark.parametrize("t", _KQUANTS)
def test_matvec_rejects_partial_super_blocks(t):
    """A K-quant row is whole 256-weight super-blocks (the reference's
    Q4_K / Q6_K shaders index them so): k = 576 is refused with an error,
    not computed."""
    with pytest.raises(_lib.CkError, match="requires 256-element rows"):
        _lib.matvec(t, bytes(130 * 3 * 210), 576, 130, np.ones(576, np.float32))


def _def(path, vocab, kv="float16", ctx=256, eos=()):
    return ModelDef(id="t", label="t", vocab=vocab, layers=0, kvHeads=0, headDim=0, maxContext=ctx,
                    gguf=path, kvDtype=kv, eosIds=list(eos))


def _vocab(path):
    import gguf as ggufpy
    r = ggufpy.GGUFReader(path)
    return int([t for t in r.tensors if t.name == "token_embd.weight"][0].shape[1])


def _rel(a, b):
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


ARCHS = ["llama", "qwen3", "gemma3"]


@pytest.mark.parametrize("mode", [_lib.MODE_STREAM, _lib.MODE_MEGAKERNEL, _lib.MODE_GRAPH])
@pytest.mark.parametrize("kv", ["float16", "float32"])
@pytest.mark.parametrize("quant", ["q4_k_m", "q8_0"])
@pytest.mark.parametrize("arch", ARCHS)
def test_teacher_forced_logits(tiny_dir, arch, quant, kv, mode):
    path = tiny_model(tiny_dir, arch, quant)
    V = _vocab(path)
    loaded = loadLlamaWgslModel(_def(path, V, kv))
    eng = loaded.engine.dev
    eng.set_mode(mode)
    orc = oracle.OracleModel(path, max_context=256)
    rng = np.random.default_rng(7)
    toks = rng.integers(0, V, size=40).tolist()
    tol = LOGIT_TOL if kv == "float16" else LOGIT_TOL_F32KV
    worst = 0.0
    for i, t in enumerate(toks):
        gid = eng.run_token(t, True)
        oid = orc.run_token(t, True)
        lg, lo = eng.logits(), orc.logits()
        r = _rel(lg, lo)
        worst = max(worst, r)
        assert r < tol, f"step {i}: rel err {r}"
        top2 = np.sort(lo)[-2:]
        if top2[1] - top2[0] > 4 * tol * np.abs(lo).max():
            assert gid == oid, f"step {i}: argmax {gid} != {oid}"
    loaded.engine.dispose()


@pytest.mark.parametrize("arch", ARCHS)
def test_greedy_64_identical(tiny_dir, arch):
    path = tiny_model(tiny_dir, arch, "q4_k_m")
    V = _vocab(path)
    loaded = loadLlamaWgslModel(_def(path, V))
    prompt = np.random.default_rng(11).integers(0, V, size=8).tolist()
    res = generateLlamaWgsl(loaded, prompt, {"maxNewTokens": 64})
    orc = oracle.OracleModel(path, max_context=256)
    ref = oracle.generate(orc, prompt, 64)
    assert res["ids"] == ref
    # the host-driven loop (onToken) must give the same ids
    resetLlamaWgslConversation(loaded)
    seen = []
    res2 = generateLlamaWgsl(loaded, prompt, {"maxNewTokens": 64, "onToken": lambda d: seen.append(d["id"])})
    assert res2["ids"] == ref and seen == ref
    loaded.engine.dispose()


@pytest.mark.parametrize("arch", ARCHS)
def test_modes_and_prefill_bitwise(tiny_dir, arch):
    """Size-independent properties: megakernel == per-phase graph (the same
    phase functions), and ck_prefill == token-by-token runs in the megakernel
    and in the streaming step, bit for bit."""
    path = tiny_model(tiny_dir, arch, "q4_k_m")
    V = _vocab(path)
    toks = np.random.default_rng(5).integers(0, V, size=30).tolist()
    groups = [[(_lib.MODE_MEGAKERNEL, False), (_lib.MODE_GRAPH, False), (_lib.MODE_MEGAKERNEL, True)],
              [(_lib.MODE_STREAM, False), (_lib.MODE_STREAM, True)]]
    for group in groups:
        outs = []
        for mode, batched in group:
            loaded = loadLlamaWgslModel(_def(path, V))
            eng = loaded.engine.dev
            eng.set_mode(mode)
            eng.set_prefill_gemm(0)        # every prompt id through the step under test
            if batched:
                nid = eng.prefill(toks, True)
            else:
                for t in toks[:-1]:
                    eng.run_token(t, False)
                nid = eng.run_token(toks[-1], True)
            outs.append((nid, eng.logits()))
            loaded.engine.dispose()
        for nid, lg in outs[1:]:
            assert nid == outs[0][0]
            assert np.array_equal(lg.view(np.uint32), outs[0][1].view(np.uint32))


@pytest.mark.parametrize("arch", ["gemma3", "qwen3"])
def test_enqueued_sampled_steps_match_decode(tiny_dir, arch):
    """ck_enqueue_decode_steps_sampled (the bench's timed steps) samples and
    chains exactly as ck_decode (generateLlamaWgsl's device loop): the same
    draws give the same ids, so the last step's logits are bit-identical."""
    path = tiny_model(tiny_dir, arch, "q4_k_m")
    V = _vocab(path)
    loaded = loadLlamaWgslModel(_def(path, V))
    eng = loaded.engine.dev
    prompt = np.random.default_rng(9).integers(0, V, size=10).tolist()
    s, _ = _lib.make_sampling(1.0, 0.9, 20, 1.0, seed=3, offset=0)
    first = eng.prefill(prompt, True, s)
    ids = eng.decode(first, 17, s)
    lg_decode = eng.logits().copy()
    eng.truncate(len(prompt))       # the first id stays stored at this position
    eng.enqueue_decode_steps(16, s)
    eng.sync()
    assert eng.position == len(prompt) + 16
    assert np.array_equal(eng.logits().view(np.uint32), lg_decode.view(np.uint32))
    assert len(set(ids)) > 1        # the draws did vary
    loaded.engine.dispose()


@pytest.mark.parametrize("arch", ["gemma3", "qwen3"])
def test_sampling_matches_reference_sampler(tiny_dir, arch):
    """Given the device's own candidate list and the same Philox draw, the
    device sampler picks what sampleFromCandidateBuffer picks."""
    path = tiny_model(tiny_dir, arch, "q4_k_m")
    V = _vocab(path)
    loaded = loadLlamaWgslModel(_def(path, V))
    eng = loaded.engine.dev
    rng = np.random.default_rng(3)
    hist = []
    for i, t in enumerate(rng.integers(0, V, size=24).tolist()):
        hist.append(t)
        T, p, k, rp = [(1.0, 0.95, 3, 1.0), (0.7, 1.0, 0, 1.3), (1.3, 0.5, 0, 1.0)][i % 3]
        s, _ = _lib.make_sampling(T, p, k, rp, seed=1234, offset=i)
        got = eng.run_token(t, True, s)
        cv, ci = eng.candidates()
        want = oracle.sample_from_candidates(cv, ci, T, p, k, rp, hist, oracle.philox_uniform(1234, i))
        assert got == want, f"step {i}"
    loaded.engine.dispose()


def test_sampled_generation_matches_oracle(tiny_dir):
    path = tiny_model(tiny_dir, "gemma3", "q4_k_m")
    V = _vocab(path)
    loaded = loadLlamaWgslModel(_def(path, V))
    prompt = np.random.default_rng(9).integers(0, V, size=6).tolist()
    opts = {"maxNewTokens": 40, "temperature": 1.0, "topK": 64, "topP": 0.95, "seed": 7}
    res = generateLlamaWgsl(loaded, prompt, opts)
    orc = oracle.OracleModel(path, max_context=256)
    ref = oracle.generate(orc, prompt, 40, temperature=1.0, top_k=64, top_p=0.95, seed=7)
    assert res["ids"] == ref
    loaded.engine.dispose()


@pytest.mark.parametrize("arch", ["llama", "qwen3"])
def test_repetition_penalty_greedy(tiny_dir, arch):
    path = tiny_model(tiny_dir, arch, "q4_k_m")
    V = _vocab(path)
    loaded = loadLlamaWgslModel(_def(path, V))
    prompt = np.random.default_rng(13).integers(0, V, size=8).tolist()
    res = generateLlamaWgsl(loaded, prompt, {"maxNewTokens": 32, "repetitionPenalty": 1.3})
    orc = oracle.OracleModel(path, max_context=256)
    ref = oracle.generate(orc, prompt, 32, repetition_penalty=1.3)
    assert res["ids"] == ref
    loaded.engine.dispose()


def test_prefix_reuse_eos_and_errors(tiny_dir):
    path = tiny_model(tiny_dir, "qwen3", "q4_k_m")
    V = _vocab(path)
    orc = oracle.OracleModel(path, max_context=256)
    prompt = np.random.default_rng(17).integers(0, V, size=8).tolist()
    ref = oracle.generate(orc, prompt, 12)
    # EOS: stop on the 5th generated id
    loaded = loadLlamaWgslModel(_def(path, V, eos=[ref[4]]))
    res = generateLlamaWgsl(loaded, prompt, {"maxNewTokens": 12})
    assert res["ids"] == ref[:ref.index(ref[4]) + 1]
    assert loaded.cachedNextId is None
    assert loaded.engine.position == len(prompt) + len(res["ids"]) - 1
    # prefix reuse: extending the cached ids does not reset the engine
    resetLlamaWgslConversation(loaded)
    loaded2 = loadLlamaWgslModel(_def(path, V))
    r1 = generateLlamaWgsl(loaded2, prompt, {"maxNewTokens": 6})
    ext = prompt + r1["ids"] + [3, 4]
    r2 = generateLlamaWgsl(loaded2, ext, {"maxNewTokens": 6})
    # oracle: same engine-call sequence (the last generated id of call 1 is
    # never fed, as in generateLlamaWgsl)
    orc.reset()
    for t in prompt[:-1]:
        orc.run_token(t, False)
    nid = orc.run_token(prompt[-1], True)
    for _ in range(5):
        nid = orc.run_token(nid, True)
    orc.run_token(3, False)
    nid = orc.run_token(4, True)
    want = [nid]
    for _ in range(5):
        nid = orc.run_token(nid, True)
        want.append(nid)
    assert r2["ids"] == want
    eng = loaded2.engine.dev
    with pytest.raises(_lib.CkError):
        eng.run_token(V + 5, True)
    eng.prefill([1] * (256 - eng.position), False)
    with pytest.raises(_lib.ContextExhausted):
        eng.run_token(1, True)
    eng.reset()
    assert eng.position == 0
    loaded.engine.dispose()
    loaded2.engine.dispose()


@pytest.mark.parametrize("mode", [_lib.MODE_MEGAKERNEL, _lib.MODE_GRAPH, _lib.MODE_STREAM])
@pytest.mark.parametrize("arch", ["gemma3", "qwen3"])
def test_exact_sampler_matches_oracle(tiny_dir, arch, mode):
    """ck_set_sampler(h, 1): the sampled id equals the oracle's exact sampler
    (top-K of the whole vocabulary by radix select, then
    sampleFromCandidateBuffer) on the device's own logits with the same
    Philox draw, in every execution mode."""
    path = tiny_model(tiny_dir, arch, "q4_k_m")
    V = _vocab(path)
    loaded = loadLlamaWgslModel(_def(path, V))
    eng = loaded.engine.dev
    eng.set_mode(mode)
    eng.set_sampler(True)
    rng = np.random.default_rng(31)
    hist = []
    settings = [(1.0, 0.95, 64, 1.0), (0.7, 1.0, 0, 1.3), (1.3, 0.5, 5, 1.0), (1.0, 1.0, 1, 1.0), (2.0, 0.9, 1023, 1.2)]
    for i, t in enumerate(rng.integers(0, V, size=25).tolist()):
        hist.append(t)
        T, p, k, rp = settings[i % len(settings)]
        s, _ = _lib.make_sampling(T, p, k, rp, seed=77, offset=i)
        got = eng.run_token(t, True, s)
        want = oracle.sample_exact(eng.logits(), T, p, k, rp, hist, oracle.philox_uniform(77, i), hist)
        assert got == want, f"step {i}: {got} != {want}"
    loaded.engine.dispose()


def test_exact_sampled_generation(tiny_dir):
    """generateLlamaWgsl with {"sampler": "exact"}: every sampled id is the
    exact sampler's choice on that step's logits (checked by replaying the
    ids one step at a time), and the default sampler is untouched."""
    path = tiny_model(tiny_dir, "gemma3", "q4_k_m")
    V = _vocab(path)
    loaded = loadLlamaWgslModel(_def(path, V))
    prompt = np.random.default_rng(33).integers(0, V, size=6).tolist()
    opts = {"maxNewTokens": 24, "temperature": 1.0, "topK": 64, "topP": 0.95, "seed": 5, "sampler": "exact"}
    res = generateLlamaWgsl(loaded, prompt, opts)
    eng = loaded.engine.dev
    eng.reset()
    eng.set_sampler(True)
    for t in prompt[:-1]:
        eng.run_token(t, False)
    tok = prompt[-1]
    for i, want_id in enumerate(res["ids"]):
        s, _ = _lib.make_sampling(1.0, 0.95, 64, 1.0, seed=5, offset=i)
        got = eng.run_token(tok, True, s)
        assert got == want_id
        assert got == oracle.sample_exact(eng.logits(), 1.0, 0.95, 64, 1.0, [], oracle.philox_uniform(5, i))
        tok = got
    # the reference sampler is back for calls that do not ask for it
    res2 = generateLlamaWgsl(loaded, prompt, {k: v for k, v in opts.items() if k != "sampler"})
    orc = oracle.OracleModel(path, max_context=256)
    assert res2["ids"] == oracle.generate(orc, prompt, 24, temperature=1.0, top_k=64, top_p=0.95, seed=5)
    loaded.engine.dispose()
