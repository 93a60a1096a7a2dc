"""Batched decode (continuous batching, ck_batch_*): every sequence of a batch
must get the ids the oracle's greedy generateLlamaWgsl gives it alone.
Sequences of different prompt lengths join at different steps, stop on EOS
or on max_new, and free their slots for later ones."""
import numpy as np
import pytest

from conftest import tiny_model
from oracle import oracle

pytestmark = pytest.mark.gpu


def _engine(path):
    from chonklm_b200.gguf import ByteSource, fetch_gguf_header
    from chonklm_b200.registry import ModelDef
    from chonklm_b200.runtime import loadLlamaWgslModel
    g = fetch_gguf_header(ByteSource(path))
    V = g.tensor_map["token_embd.weight"].shape[1]
    loaded = loadLlamaWgslModel(ModelDef(id="t", label="t", vocab=V, maxContext=256, gguf=path, eosIds=[]))
    return loaded, V


def _run(batch, pending, max_steps=2000):
    """Add pending (prompt, max_new, eos) as slots free up; step to the end."""
    ids = {}
    queue = list(enumerate(pending))
    live = {}
    steps = 0
    while queue or live:
        while queue:
            j, (prompt, max_new, eos) = queue[0]
            try:
                live[batch.add(prompt, max_new, eos)] = j
            except Exception as e:  # every slot taken: try after the next step
                if "slots" not in str(e):
                    raise
                break
            queue.pop(0)
        batch.step()
        steps += 1
        assert steps < max_steps
        for sid in list(live):
            got, done = batch.collect(sid)
            if done:
                ids[live.pop(sid)] = got
    return [ids[j] for j in range(len(pending))]


MATMUL_TOL = 2e-5   # relative: x and w each split into two fp16 parts (~22 bits), fp32 accumulation


@pytest.mark.parametrize("t,k,n,T", [(12, 1024, 300, 1), (14, 512, 129, 37), (8, 576, 260, 130), (6, 576, 200, 16),
                                     (7, 64, 130, 5), (12, 256, 6272, 3), (14, 256, 20000, 200),
                                     (8, 576, 300, 600), (12, 1024, 260, 520), (14, 256, 20000, 600)])
def test_tensor_core_matmul(t, k, n, T):
    """The batched path's tcgen05 GEMM (prologue split of x + dequant split of
    W, three MMAs per step) against fp64 over the oracle's dequantized
    weights: single token, partial and multiple 128-token tiles, partial
    128-row tiles, every block type, K split over clusters, and two token
    tiles per CTA (>= 4 token tiles, the last CTA holding only one)."""
    import torch
    from chonklm_b200 import _lib
    from chonklm_b200.quant import quantize
    g = torch.Generator().manual_seed(t * 1000 + k + T)
    data = quantize(torch.randn(n, k, generator=g) * 0.02, t)
    x = (np.random.default_rng(T).standard_normal((T, k)) * 3).astype(np.float32)
    y = _lib.matmul(t, data, k, n, x)
    w = oracle.dequant(t, np.frombuffer(data, dtype=np.uint8), k, n).astype(np.float64)
    ref = x.astype(np.float64) @ w.T
    err = np.abs(y - ref).max() / np.abs(ref).max()
    assert err < MATMUL_TOL, err


@pytest.mark.parametrize("arch,kw", [("llama", {}), ("qwen3", {}), ("llama", {"intermediate": 544}),
                                     ("llama", {"heads": 6, "kv_heads": 2}), ("qwen3", {"head_dim": 128}),
                                     ("llama", {"heads": 8, "kv_heads": 2})])
def test_batch_matches_oracle_greedy(tiny_dir, arch, kw):
    """intermediate 544 (not a multiple of 64) keeps gate and up as separate
    tiles with the SiLU prologue; the others fuse SiLU into the GEMM.  The
    attention shapes cover the grouped-heads kernel (2 or 3 query heads per
    kv head at head_dim 64) and the per-head-group kernel (head_dim 128, or 4
    query heads per kv head)."""
    from chonklm_b200 import _lib
    path = tiny_model(tiny_dir, arch, "q4_k_m", **kw)
    loaded, V = _engine(path)
    rng = np.random.default_rng(5)
    pending = []
    for j in range(7):
        n = int(rng.integers(1, 20))
        pending.append((rng.integers(0, V, size=n).tolist(), int(rng.integers(1, 40)), ()))
    batch = _lib.Batch(loaded.engine.dev, max_seqs=4)   # fewer slots than sequences: slots are reused
    got = _run(batch, pending)
    orc = oracle.OracleModel(path, max_context=256)
    for (prompt, max_new, _), ids in zip(pending, got):
        orc.reset()
        assert ids == oracle.generate(orc, prompt, max_new), (prompt, max_new)
    steps, fed, gen = batch.stats()
    assert gen == sum(len(x) for x in got)
    assert fed == sum(len(p) + len(x) - 1 for (p, _, _), x in zip(pending, got))
    batch.close()
    loaded.engine.dispose()


@pytest.mark.parametrize("arch,kw", [("llama", {}), ("llama", {"heads": 6, "kv_heads": 2}),
                                     ("qwen3", {"head_dim": 128})])
def test_batch_long_sequences(tiny_dir, arch, kw):
    """Sequences past 128 positions (prompt + generated up to 240): the
    attention kernels' multi-round position loop (128 positions per round in
    the grouped-heads kernel) and the merge across rounds, against the
    oracle's greedy ids."""
    from chonklm_b200 import _lib
    path = tiny_model(tiny_dir, arch, "q4_k_m", **kw)
    loaded, V = _engine(path)
    rng = np.random.default_rng(11)
    pending = [(rng.integers(0, V, size=n).tolist(), m, ()) for n, m in ((150, 90), (129, 40), (200, 40), (60, 120))]
    batch = _lib.Batch(loaded.engine.dev, max_seqs=3)
    got = _run(batch, pending)
    orc = oracle.OracleModel(path, max_context=256)
    for (prompt, max_new, _), ids in zip(pending, got):
        orc.reset()
        assert ids == oracle.generate(orc, prompt, max_new), (len(prompt), max_new)
    batch.close()
    loaded.engine.dispose()


def test_batch_eos_and_limits(tiny_dir):
    from chonklm_b200 import _lib
    path = tiny_model(tiny_dir, "llama", "q4_k_m")
    loaded, V = _engine(path)
    orc = oracle.OracleModel(path, max_context=256)
    prompt = [5, 17, 29, 41]
    ref = oracle.generate(orc, prompt, 30)
    eos = ref[6]
    stop = ref.index(eos) + 1
    batch = _lib.Batch(loaded.engine.dev, max_seqs=2)
    got = _run(batch, [(prompt, 30, (eos,)), (prompt, 3, ())])
    assert got[0] == ref[:stop] and got[1] == ref[:3]
    # a full batch refuses more sequences; bad token ids are rejected on the host
    a = batch.add(prompt, 5)
    b = batch.add(prompt, 5)
    with pytest.raises(_lib.CkError, match="slots"):
        batch.add(prompt, 5)
    with pytest.raises(_lib.CkError, match="outside embedding table"):
        _lib.Batch(loaded.engine.dev, max_seqs=1).add([V + 3], 4)
    batch.close()
    # a KV pool too small for a sequence is reported, not overrun
    small = _lib.Batch(loaded.engine.dev, max_seqs=2, kv_blocks=1)
    with pytest.raises(_lib.CkError, match="KV pool"):
        small.add(prompt, 30)
    small.close()
    loaded.engine.dispose()
