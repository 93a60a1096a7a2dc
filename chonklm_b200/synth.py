"""Seeded synthetic GGUF decoder models with the shapes of the benchmark configs.

Weights are N(0, std) (std 0.02 by default) drawn from numpy's PCG64 with a
fixed seed, quantized into ggml block layouts by `chonklm_b200.quant`, and
written as GGUF v3 with the tensor names and metadata keys the reference's
manifest builder reads (llama-wgsl-runtime.ts:326-425):
  general.architecture, {arch}.block_count / embedding_length /
  feed_forward_length / attention.head_count / head_count_kv / key_length /
  context_length / rope.freq_base / attention.layer_norm_rms_epsilon,
  gemma3.attention.sliding_window; tensors token_embd, output_norm,
  blk.N.{attn_norm, attn_q, attn_k, attn_v, attn_output, ffn_norm, ffn_gate,
  ffn_up, ffn_down} (+ attn_q_norm/attn_k_norm, + gemma3 post norms).

Q4_K_M mixture (mirrors llama.cpp's recipe closely enough for byte counts):
attn_v and ffn_down are Q6_K on even layers and Q4_K on odd layers, every other
linear is Q4_K, the tied token_embd is Q6_K; a K-quant whose row length is not
a multiple of 256 falls back to Q5_0 (for Q4_K) or Q8_0 (for Q6_K).
"""
from __future__ import annotations

import os
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Tuple

import numpy as np
import torch

from .gguf import GGML_TYPE, VT_ARR, VT_BOOL, VT_F32, VT_I32, VT_STR, VT_U32, write_gguf
from .quant import quantize


@dataclass
class SynthSpec:
    arch: str                  # "llama" | "qwen3" | "gemma3"
    hidden: int
    layers: int
    heads: int
    kv_heads: int
    head_dim: int
    intermediate: int
    vocab: int
    context_length: int
    rope_theta: float = 10000.0
    norm_eps: float = 1e-5
    sliding_window: int = 0
    quant: str = "q4_k_m"      # "q4_k_m" | "q8_0" | "f32" | explicit via overrides
    qk_norm: bool = False
    std: float = 0.02
    norm_init: str = "ones"    # "ones" | "random" (1 + 0.1 N) -- random catches index bugs
    tied: bool = True
    overrides: Dict[str, int] = field(default_factory=dict)  # tensor-name -> ggml type
    tokenizer: bool = False    # write a SentencePiece vocabulary (tokenizer.synthetic_vocab)


SPECS: Dict[str, SynthSpec] = {
    # SmolLM2-135M-shaped llama decoder
    "smollm2-135m": SynthSpec("llama", 576, 30, 9, 3, 64, 1536, 49152, 2048, rope_theta=100000.0, norm_eps=1e-5),
    # Qwen3-0.6B-shaped
    "qwen3-0.6b": SynthSpec("qwen3", 1024, 28, 16, 8, 128, 3072, 151936, 40960, rope_theta=1000000.0,
                            norm_eps=1e-6, qk_norm=True),
    # same, all linears Q8_0
    "qwen3-0.6b-q8": SynthSpec("qwen3", 1024, 28, 16, 8, 128, 3072, 151936, 40960, rope_theta=1000000.0,
                               norm_eps=1e-6, qk_norm=True, quant="q8_0"),
    # Gemma-3-270M-shaped
    "gemma3-270m": SynthSpec("gemma3", 640, 18, 4, 1, 256, 2048, 262144, 32768, rope_theta=1000000.0,
                             norm_eps=1e-6, sliding_window=512, qk_norm=True),
}


def _kquant_fallback(t: int, k: int) -> int:
    if k % 256 == 0:
        return t
    return {GGML_TYPE.Q4_K: GGML_TYPE.Q5_0, GGML_TYPE.Q6_K: GGML_TYPE.Q8_0,
            GGML_TYPE.Q5_K: GGML_TYPE.Q5_1}.get(t, t)


def tensor_plan(spec: SynthSpec) -> List[Tuple[str, int, int, int]]:
    """List of (name, rows n, row length k, ggml type)."""
    h, hd = spec.hidden, spec.head_dim
    qd, kvd, inter = spec.heads * hd, spec.kv_heads * hd, spec.intermediate

    def lin(name: str, layer: int, kind: str, k: int) -> int:
        if name in spec.overrides:
            return spec.overrides[name]
        if spec.quant == "q8_0":
            return GGML_TYPE.Q8_0
        if spec.quant == "f32":
            return GGML_TYPE.F32
        if spec.quant == "q4_k_m":
            t = GGML_TYPE.Q6_K if (kind in ("attn_v", "ffn_down") and layer % 2 == 0) else GGML_TYPE.Q4_K
            return _kquant_fallback(t, k)
        raise ValueError(spec.quant)

    plan: List[Tuple[str, int, int, int]] = []
    emb_t = spec.overrides.get("token_embd.weight")
    if emb_t is None:
        emb_t = {"q8_0": GGML_TYPE.Q8_0, "f32": GGML_TYPE.F32}.get(spec.quant, None)
        if emb_t is None:
            emb_t = _kquant_fallback(GGML_TYPE.Q6_K, h)
    plan.append(("token_embd.weight", spec.vocab, h, emb_t))
    if not spec.tied:
        plan.append(("output.weight", spec.vocab, h, spec.overrides.get("output.weight", emb_t)))
    plan.append(("output_norm.weight", 1, h, GGML_TYPE.F32))
    for i in range(spec.layers):
        p = f"blk.{i}."
        plan.append((p + "attn_norm.weight", 1, h, GGML_TYPE.F32))
        plan.append((p + "attn_q.weight", qd, h, lin(p + "attn_q.weight", i, "attn_q", h)))
        plan.append((p + "attn_k.weight", kvd, h, lin(p + "attn_k.weight", i, "attn_k", h)))
        plan.append((p + "attn_v.weight", kvd, h, lin(p + "attn_v.weight", i, "attn_v", h)))
        if spec.qk_norm:
            plan.append((p + "attn_q_norm.weight", 1, hd, GGML_TYPE.F32))
            plan.append((p + "attn_k_norm.weight", 1, hd, GGML_TYPE.F32))
        plan.append((p + "attn_output.weight", h, qd, lin(p + "attn_output.weight", i, "attn_output", qd)))
        if spec.arch == "gemma3":
            plan.append((p + "post_attention_norm.weight", 1, h, GGML_TYPE.F32))
        plan.append((p + "ffn_norm.weight", 1, h, GGML_TYPE.F32))
        plan.append((p + "ffn_gate.weight", inter, h, lin(p + "ffn_gate.weight", i, "ffn_gate", h)))
        plan.append((p + "ffn_up.weight", inter, h, lin(p + "ffn_up.weight", i, "ffn_up", h)))
        plan.append((p + "ffn_down.weight", h, inter, lin(p + "ffn_down.weight", i, "ffn_down", inter)))
        if spec.arch == "gemma3":
            plan.append((p + "post_ffw_norm.weight", 1, h, GGML_TYPE.F32))
    return plan


def _metadata(spec: SynthSpec, name: str, seed: int) -> Dict[str, object]:
    a = spec.arch
    kv: Dict[str, object] = {
        "general.architecture": a,
        "general.name": name,
        "general.alignment": (32, VT_U32),
        f"{a}.block_count": (spec.layers, VT_U32),
        f"{a}.context_length": (spec.context_length, VT_U32),
        f"{a}.embedding_length": (spec.hidden, VT_U32),
        f"{a}.feed_forward_length": (spec.intermediate, VT_U32),
        f"{a}.attention.head_count": (spec.heads, VT_U32),
        f"{a}.attention.head_count_kv": (spec.kv_heads, VT_U32),
        f"{a}.attention.key_length": (spec.head_dim, VT_U32),
        f"{a}.attention.value_length": (spec.head_dim, VT_U32),
        f"{a}.rope.freq_base": (float(spec.rope_theta), VT_F32),
        f"{a}.attention.layer_norm_rms_epsilon": (float(spec.norm_eps), VT_F32),
        "chonk.synthetic.seed": (seed, VT_U32),
        "chonk.synthetic.std": (float(spec.std), VT_F32),
    }
    if a == "gemma3":
        kv["gemma3.attention.sliding_window"] = (spec.sliding_window, VT_U32)
    if spec.tokenizer:
        from .tokenizer import synthetic_vocab
        toks, scores, types = synthetic_vocab(spec.vocab)
        kv["tokenizer.ggml.model"] = ("llama", VT_STR)
        kv["tokenizer.ggml.tokens"] = toks
        kv["tokenizer.ggml.scores"] = ([float(x) for x in scores], VT_ARR, VT_F32)
        kv["tokenizer.ggml.token_type"] = ([int(x) for x in types], VT_ARR, VT_I32)
        kv["tokenizer.ggml.bos_token_id"] = (toks.index("<bos>"), VT_U32)
        kv["tokenizer.ggml.eos_token_id"] = (toks.index("<eos>"), VT_U32)
        kv["tokenizer.ggml.unknown_token_id"] = (toks.index("<unk>"), VT_U32)
        kv["tokenizer.ggml.padding_token_id"] = (toks.index("<pad>"), VT_U32)
        kv["tokenizer.ggml.add_bos_token"] = (True, VT_BOOL)
        kv["tokenizer.ggml.add_space_prefix"] = (False, VT_BOOL)
    return kv


def write_synthetic_gguf(spec: SynthSpec, path: str, seed: int = 0, name: str = "synthetic",
                         device: Optional[str] = None) -> str:
    """Generate and write the model; returns `path`.

    Weights come from numpy PCG64(seed), tensor by tensor in plan order, so
    the bytes are identical on every machine; `device` only chooses where the
    (deterministic, elementwise) quantization arithmetic runs.
    """
    if device is None:
        device = "cuda" if torch.cuda.is_available() else "cpu"
    rng = np.random.Generator(np.random.PCG64(seed))
    tensors = []
    for tname, n, k, t in tensor_plan(spec):
        if tname.endswith("norm.weight"):
            if spec.norm_init == "random":
                w = (1.0 + 0.1 * rng.standard_normal(k, dtype=np.float32)).astype(np.float32)
            else:
                w = np.ones(k, dtype=np.float32)
            tensors.append((tname, [k], GGML_TYPE.F32, w.tobytes()))
            continue
        parts = []
        rows_per = max(1, (1 << 24) // k)
        for r0 in range(0, n, rows_per):
            r = min(rows_per, n - r0)
            x = rng.standard_normal((r, k), dtype=np.float32) * np.float32(spec.std)
            parts.append(quantize(torch.from_numpy(x).to(device), t))
        tensors.append((tname, [k, n], t, b"".join(parts)))
    os.makedirs(os.path.dirname(os.path.abspath(path)), exist_ok=True)
    write_gguf(path, _metadata(spec, name, seed), tensors)
    return path


def tiny_spec(arch: str, quant: str = "q4_k_m", **kw) -> SynthSpec:
    """Small models for fast CPU/GPU parity tests; shapes keep every kernel
    path exercised (K-quant rows of 256/512, 32-block fallbacks, GQA)."""
    if arch == "llama":
        s = SynthSpec("llama", 256, 2, 4, 2, 64, 512, 1000, 256, rope_theta=10000.0, norm_eps=1e-5,
                      quant=quant, norm_init="random")
    elif arch == "qwen3":
        s = SynthSpec("qwen3", 256, 2, 4, 2, 64, 768, 1000, 256, rope_theta=1000000.0, norm_eps=1e-6,
                      qk_norm=True, quant=quant, norm_init="random")
    elif arch == "gemma3":
        s = SynthSpec("gemma3", 320, 6, 2, 1, 128, 512, 1300, 256, rope_theta=1000000.0, norm_eps=1e-6,
                      qk_norm=True, sliding_window=16, quant=quant, norm_init="random")
    else:
        raise ValueError(arch)
    for k, v in kw.items():
        setattr(s, k, v)
    return s
