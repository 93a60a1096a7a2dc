"""The oracle pinned: dequant bit-exact against gguf-py's decode of the same
blocks (committed fixtures), Philox known-answer vectors, argmax/sampling
rules of the reference, and a regression guard on the tiny models."""
import math
import os

import numpy as np
import pytest

from conftest import tiny_model
from chonklm_b200.gguf import GGML_TYPE
from oracle import oracle

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")
TYPES = {"Q4_K": GGML_TYPE.Q4_K, "Q6_K": GGML_TYPE.Q6_K, "Q8_0": GGML_TYPE.Q8_0, "Q5_0": GGML_TYPE.Q5_0,
         "Q5_1": GGML_TYPE.Q5_1}


@pytest.mark.parametrize("name", list(TYPES))
def test_dequant_matches_gguf_py_fixtures(name):
    z = np.load(os.path.join(GOLDEN, "dequant_golden.npz"))
    raw, deq, k = z[f"{name}_raw"], z[f"{name}_deq"], int(z[f"{name}_k"][0])
    n = deq.size // k
    got = oracle.dequant(TYPES[name], raw, k, n).reshape(-1)
    assert np.array_equal(got.view(np.uint32), deq.view(np.uint32))


@pytest.mark.parametrize("name", list(TYPES))
def test_dequant_matches_gguf_py_live(name):
    """Same check on fresh random bytes with finite fp16 scales."""
    import gguf
    from gguf import quants
    bb = {"Q4_K": 144, "Q6_K": 210, "Q8_0": 34, "Q5_0": 22, "Q5_1": 24}[name]
    k = 256 if name in ("Q4_K", "Q6_K") else 32
    rng = np.random.default_rng(42)
    blocks = rng.integers(0, 256, size=(64, bb), dtype=np.uint8)
    halves = ((rng.integers(0, 2, 128) << 15) | (rng.integers(0, 31, 128) << 10) | rng.integers(0, 1024, 128))
    halves = halves.astype(np.uint16).reshape(64, 2)
    if name == "Q6_K":
        blocks[:, 208:210] = halves[:, :1].view(np.uint8)
    else:
        blocks[:, 0:4] = halves.view(np.uint8)
    ref = quants.dequantize(blocks, getattr(gguf.GGMLQuantizationType, name)).astype(np.float32).reshape(-1)
    got = oracle.dequant(TYPES[name], blocks.reshape(-1), k, 64).reshape(-1)
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))


def test_q4k_known_answer():
    """A hand-decoded Q4_K block: d=1, dmin=0.5, scale/min of sub-block 5
    come from the high-bit packing (scale_min_k4, j >= 4)."""
    z = np.load(os.path.join(GOLDEN, "dequant_golden.npz"))
    raw = z["Q4_K_raw"].reshape(-1, 144)[8]      # first KAT block (after 6 + 2 seeded)
    deq = oracle.dequant(GGML_TYPE.Q4_K, raw, 256, 1)[0]
    sc = [(9 * j) % 64 for j in range(8)]
    mn = [(13 * j + 1) % 64 for j in range(8)]
    for w in (0, 37, 64 + 33, 5 * 32 + 7, 255):
        g, lane, high = w // 64, w % 32, (w % 64) >= 32
        byte = (lane % 16) | (((lane * 3) % 16) << 4)
        q = (byte >> 4) if high else (byte & 15)
        j = 2 * g + (1 if high else 0)
        want = np.float32(1.0) * np.float32(sc[j]) * np.float32(q) - np.float32(0.5) * np.float32(mn[j])
        assert deq[w] == want, (w, deq[w], want)


def test_matvec_wgsl_order_vs_f64():
    z = np.load(os.path.join(GOLDEN, "dequant_golden.npz"))
    raw = z["Q4_K_raw"][:144 * 6]
    x = np.random.default_rng(0).standard_normal(256).astype(np.float32)
    y32 = oracle.matvec(GGML_TYPE.Q4_K, raw, 256, 6, x, oracle.MODE_WGSL)
    y64 = oracle.matvec(GGML_TYPE.Q4_K, raw, 256, 6, x, oracle.MODE_F64)
    w = oracle.dequant(GGML_TYPE.Q4_K, raw, 256, 6).astype(np.float64)
    assert np.allclose(y64, w @ x.astype(np.float64), rtol=1e-6, atol=1e-9)
    assert np.abs(y32 - y64).max() <= 1e-5 * np.abs(y64).max()


@pytest.mark.parametrize("name", list(TYPES))
def test_matvec_wgsl_mode_bit_exact_restatement(name):
    """The oracle's fp32 matvec (rows dequantized once, then summed) equals,
    bit for bit, the GGUF_*_MATVEC_WGSL reduction written out here in numpy
    over the per-weight dequantizer: 128 strided per-thread sums in column
    order, then the stride-64..1 tree (llama-wgsl-runtime.ts:2247-2277)."""
    t = TYPES[name]
    k = 1024 if name in ("Q4_K", "Q6_K") else 576
    n = 48
    rng = np.random.default_rng(5)
    data = _quantized_blocks(t, k, n, rng)
    x = rng.standard_normal(k).astype(np.float32)
    w = oracle.dequant(t, data, k, n)
    prod = (x[None, :] * w).astype(np.float32)
    acc = np.zeros((n, 128), dtype=np.float32)
    pad = np.zeros((n, -k % 128), dtype=np.float32)
    cols = np.concatenate([prod, pad], axis=1).reshape(n, -1, 128)
    for j in range(cols.shape[1]):
        acc = (acc + cols[:, j, :]).astype(np.float32)
    stride = 64
    while stride >= 1:
        acc[:, :stride] = (acc[:, :stride] + acc[:, stride:2 * stride]).astype(np.float32)
        stride //= 2
    got = oracle.matvec(t, data, k, n, x, oracle.MODE_WGSL)
    assert np.array_equal(got.view(np.uint32), acc[:, 0].view(np.uint32))


def _quantized_blocks(t, k, n, rng):
    import torch
    from chonklm_b200.quant import quantize
    w = torch.from_numpy(rng.standard_normal((n, k)).astype(np.float32) * 0.02)
    return np.frombuffer(quantize(w, t), dtype=np.uint8)


def test_philox_known_answers():
    """Random123 known-answer vectors for philox4x32-10."""
    assert oracle.philox4x32([0, 0, 0, 0], [0, 0]) == [0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8]
    assert oracle.philox4x32([0xFFFFFFFF] * 4, [0xFFFFFFFF] * 2) == [0x408F276D, 0x41C83B0E, 0xA20BC7C6, 0x6D5451FD]
    assert oracle.philox4x32([0x243F6A88, 0x85A308D3, 0x13198A2E, 0x03707344], [0xA4093822, 0x299F31D0]) == \
        [0xD16CFE09, 0x94FDCCEB, 0x5001E420, 0x24126EA1]
    u = [oracle.philox_uniform(7, i) for i in range(1000)]
    assert 0 <= min(u) and max(u) < 1 and abs(np.mean(u) - 0.5) < 0.03


def test_argmax_rules():
    """NaN never wins, ties go to the lower index, penalty divides positive
    and multiplies negative logits (ARGMAX_STAGE1/2)."""
    lg = np.full(600, -1.0, np.float32)
    lg[10] = np.nan
    lg[300] = 2.0
    lg[301] = 2.0
    lg[5] = 2.0
    cv, ci, best = oracle.argmax_candidates(lg)
    assert best == 5 and ci[0] == 5 and ci[1] == 300 and len(cv) == 3
    allnan = np.full(256, np.nan, np.float32)
    cv, ci, best = oracle.argmax_candidates(allnan)
    assert ci[0] == 0 and math.isnan(cv[0])
    lg = np.zeros(300, np.float32)
    lg[7], lg[8] = 1.2, 1.0
    cv, ci, best = oracle.argmax_candidates(lg, penalty_ids=[7], penalty=1.3)
    assert best == 8                       # 1.2 / 1.3 < 1.0
    lg[7] = -0.1
    lg[8] = -0.12
    lg[:] = np.minimum(lg, -0.05)
    cv, ci, best = oracle.argmax_candidates(lg, penalty_ids=[9], penalty=2.0)
    assert ci[0] != 9


def test_sampler_semantics():
    cv = np.array([1.0, 3.0, 2.0, np.inf, 3.0], np.float32)
    ci = np.array([10, 20, 30, 40, 0xFFFFFFFF], np.uint32)
    # temperature 0 -> highest (first of ties), non-finite / sentinel dropped
    assert oracle.sample_from_candidates(cv, ci, 0.0) == 20
    # top-k 1 always returns the best
    for u in (0.0, 0.5, 0.999):
        assert oracle.sample_from_candidates(cv, ci, 1.0, 1.0, 1, 1.0, (), u) == 20
    # u = 0 picks the first; u -> 1 picks the last kept
    assert oracle.sample_from_candidates(cv, ci, 1.0, 1.0, 0, 1.0, (), 0.0) == 20
    assert oracle.sample_from_candidates(cv, ci, 1.0, 1.0, 0, 1.0, (), 0.999999) == 10
    # top-p cuts after the first candidate whose cdf reaches p
    assert oracle.sample_from_candidates(cv, ci, 1.0, 0.5, 0, 1.0, (), 0.999999) == 20
    # repetition penalty on seen ids re-ranks
    assert oracle.sample_from_candidates(cv, ci, 0.0, 1.0, 0, 2.0, [20]) == 30
    assert oracle.needs_sampling_readback(0.0, 1.0, 0) is False
    assert oracle.needs_sampling_readback(0.0, 0.9, 0) is True
    assert oracle.needs_sampling_readback(0.0, 1.0, 3) is True


def test_tiny_model_regression(tiny_dir):
    z = np.load(os.path.join(GOLDEN, "tiny_logits.npz"))
    for arch in ("llama", "qwen3", "gemma3"):
        m = oracle.OracleModel(tiny_model(tiny_dir, arch), max_context=64)
        for i, t in enumerate(z[f"{arch}_tokens"].tolist()):
            assert m.run_token(t, True) == z[f"{arch}_ids"][i]
            np.testing.assert_array_equal(m.logits(), z[f"{arch}_logits"][i])
        m.close()


def test_oracle_wgsl_vs_f64_model(tiny_dir):
    """The fp32 WGSL-order restatement and the fp64 mode agree to ~1e-6."""
    for arch in ("llama", "qwen3", "gemma3"):
        a = oracle.OracleModel(tiny_model(tiny_dir, arch), max_context=64)
        b = oracle.OracleModel(tiny_model(tiny_dir, arch), max_context=64, mode=oracle.MODE_F64)
        for t in [5, 6, 7, 8, 9, 10]:
            a.run_token(t, True)
            b.run_token(t, True)
        la, lb = a.logits(), b.logits()
        assert np.abs(la - lb).max() / np.abs(lb).max() < 1e-5


def test_context_exhausted(tiny_dir):
    m = oracle.OracleModel(tiny_model(tiny_dir, "llama"), max_context=4)
    for t in range(4):
        m.run_token(t, False)
    with pytest.raises(RuntimeError, match="context exhausted"):
        m.run_token(1, True)
