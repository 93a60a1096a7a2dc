"""Host side: GGUF container, shard manifests and the manifest rules of
buildGgufLlamaManifest."""
import json
import math
import os
import struct

import numpy as np
import pytest

from conftest import tiny_model
from chonklm_b200.gguf import (GGML_TYPE, ByteSource, fetch_gguf_header, ggml_tensor_byte_length, parse_gguf,
                               shard_gguf, write_gguf)
from chonklm_b200.manifest import build_gguf_llama_manifest
from chonklm_b200.registry import MODELS, ModelDef, getModel
from chonklm_b200.synth import SPECS, tensor_plan, tiny_spec


def _def(path, vocab=1000, ctx=256, layers=2):
    return ModelDef(id="t", label="t", vocab=vocab, layers=layers, kvHeads=0, headDim=0, maxContext=ctx, gguf=path)


def test_byte_lengths():
    assert ggml_tensor_byte_length(GGML_TYPE.Q4_K, 512) == 288
    assert ggml_tensor_byte_length(GGML_TYPE.Q6_K, 256) == 210
    assert ggml_tensor_byte_length(GGML_TYPE.Q8_0, 64) == 68
    assert ggml_tensor_byte_length(GGML_TYPE.Q5_0, 32) == 22
    with pytest.raises(ValueError, match="256-element blocks"):
        ggml_tensor_byte_length(GGML_TYPE.Q4_K, 576)
    with pytest.raises(ValueError, match="unsupported"):
        ggml_tensor_byte_length(2, 32)


def test_roundtrip_and_gguf_py_reads_our_files(tiny_dir):
    import gguf as ggufpy
    for arch in ("llama", "qwen3", "gemma3"):
        p = tiny_model(tiny_dir, arch)
        g = fetch_gguf_header(ByteSource(p))
        r = ggufpy.GGUFReader(p)
        assert g.data_offset % 32 == 0
        assert {t.name for t in r.tensors} == set(g.tensor_map)
        for t in r.tensors:
            mine = g.tensor_map[t.name]
            assert list(t.shape) == mine.shape and int(t.tensor_type) == mine.type
            assert t.data_offset == g.data_offset + mine.offset
        assert r.fields["general.architecture"].parts[-1].tobytes().decode() == arch


def test_parse_errors(tmp_path):
    with pytest.raises(ValueError, match="invalid GGUF magic"):
        parse_gguf(b"XXXX" + bytes(60))
    p = tmp_path / "trunc.gguf"
    write_gguf(str(p), {"general.architecture": "llama"}, [("a", [32, 2], GGML_TYPE.Q8_0, bytes(68))])
    data = p.read_bytes()
    with pytest.raises(Exception):
        parse_gguf(data[:40])
    with pytest.raises(ValueError, match="expected"):
        write_gguf(str(p), {}, [("a", [32, 2], GGML_TYPE.Q8_0, bytes(60))])


def test_shard_manifest_range_reads(tiny_dir, tmp_path):
    p = tiny_model(tiny_dir, "qwen3")
    d = str(tmp_path / "q4_k_m")
    m = shard_gguf(p, d, shard_size=100_000)
    assert m["shardCount"] > 2 and sum(s["size"] for s in m["shards"]) == os.path.getsize(p)
    a, b = ByteSource(p), ByteSource(d)
    assert b.sharded and b.total_size == a.total_size
    rng = np.random.default_rng(0)
    for _ in range(20):
        off = int(rng.integers(0, a.total_size - 1))
        n = int(rng.integers(0, min(300_000, a.total_size - off)))
        assert a.read(off, n) == b.read(off, n)
    with pytest.raises(ValueError, match="out of bounds"):
        b.read(a.total_size - 10, 20)
    g1, g2 = fetch_gguf_header(a), fetch_gguf_header(b)
    assert g1.data_offset == g2.data_offset and list(g1.tensor_map) == list(g2.tensor_map)


def test_manifest_llama_qwen3(tiny_dir):
    for arch, layout in (("llama", "interleaved"), ("qwen3", "split")):
        p = tiny_model(tiny_dir, arch)
        g = fetch_gguf_header(ByteSource(p))
        man = build_gguf_llama_manifest(_def(p, ctx=100), g)
        m = man.model
        s = tiny_spec(arch)
        assert (m.hidden, m.heads, m.kvHeads, m.headDim, m.layers) == (s.hidden, s.heads, s.kv_heads, s.head_dim,
                                                                       s.layers)
        assert m.ropeLayout == layout and m.architecture == "llama"
        assert m.qkNorm == (arch == "qwen3")
        assert m.maxContext == 100 and m.embeddingScale == 1.0 and m.activation == "silu"
        assert m.layerRopeTheta == [s.rope_theta] * s.layers and m.layerAttentionWindow == [0] * s.layers
        assert abs(m.normEps - s.norm_eps) < 1e-12 * 1e6
        # tied head: lm_head alias resolves to the embedding
        assert man.resolve("lm_head.MatMul.weight") == "token_embd.weight"
        assert man.resolve("model.layers.1.post_attention_layernorm.weight") == "blk.1.ffn_norm.weight"
        assert man.spec("model.layers.0.attn.q_proj.MatMul.weight").shape == [s.heads * s.head_dim, s.hidden]


def test_manifest_gemma3(tiny_dir):
    p = tiny_model(tiny_dir, "gemma3")
    g = fetch_gguf_header(ByteSource(p))
    man = build_gguf_llama_manifest(_def(p, layers=6), g)
    m = man.model
    assert m.architecture == "gemma3" and m.ropeLayout == "split" and m.activation == "gelu-tanh"
    assert m.embeddingScale == pytest.approx(math.sqrt(320))
    assert m.layerRopeTheta == [10000] * 5 + [1000000]
    assert m.layerAttentionWindow == [16] * 5 + [0]
    assert man.resolve("model.layers.2.post_attention_layernorm.weight") == "blk.2.post_attention_norm.weight"
    assert man.resolve("model.layers.2.pre_feedforward_layernorm.weight") == "blk.2.ffn_norm.weight"
    assert man.resolve("model.layers.2.post_feedforward_layernorm.weight") == "blk.2.post_ffw_norm.weight"


def test_manifest_rejects(tmp_path):
    p = tmp_path / "x.gguf"
    write_gguf(str(p), {"general.architecture": "gpt2"}, [])
    with pytest.raises(ValueError, match="does not support architecture gpt2"):
        build_gguf_llama_manifest(_def(str(p)), fetch_gguf_header(ByteSource(str(p))))
    write_gguf(str(p), {"general.architecture": "openelm"}, [])
    with pytest.raises(ValueError, match="openelm"):
        build_gguf_llama_manifest(_def(str(p)), fetch_gguf_header(ByteSource(str(p))))
    write_gguf(str(p), {"general.architecture": "llama"}, [])
    with pytest.raises(ValueError, match="block_count"):
        build_gguf_llama_manifest(_def(str(p)), fetch_gguf_header(ByteSource(str(p))))


def test_q4_k_m_plan_fallbacks():
    """K-quants need rows of 256: SmolLM2 (576) and Gemma (640) fall back to
    Q5_0/Q8_0 except where the row is the intermediate size."""
    plan = {n: t for n, _, _, t in tensor_plan(SPECS["smollm2-135m"])}
    assert plan["blk.0.attn_q.weight"] == GGML_TYPE.Q5_0
    assert plan["blk.0.attn_v.weight"] == GGML_TYPE.Q8_0
    assert plan["blk.1.attn_v.weight"] == GGML_TYPE.Q5_0
    assert plan["blk.0.ffn_down.weight"] == GGML_TYPE.Q6_K
    assert plan["blk.1.ffn_down.weight"] == GGML_TYPE.Q4_K
    assert plan["token_embd.weight"] == GGML_TYPE.Q8_0
    q = {n: t for n, _, _, t in tensor_plan(SPECS["qwen3-0.6b"])}
    assert q["token_embd.weight"] == GGML_TYPE.Q6_K and q["blk.3.ffn_up.weight"] == GGML_TYPE.Q4_K
    q8 = {n: t for n, _, _, t in tensor_plan(SPECS["qwen3-0.6b-q8"])}
    assert set(t for n, t in q8.items() if not n.endswith("norm.weight")) == {GGML_TYPE.Q8_0}


def test_registry():
    assert getModel("qwen3-0.6b-q4-k-m-synthetic").maxContext == 2048
    assert all(m.runtime == "llama-webgpu" for m in MODELS)
    with pytest.raises(KeyError):
        getModel("nope")
