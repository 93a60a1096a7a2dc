"""GGUF -> model manifest: the host-side twin of the reference's
`buildGgufLlamaManifest` (llama-wgsl-runtime.ts:326-425) and
`tensorSpecFromGguf` (:431-441).

Rules restated here:
  * architecture must be llama / qwen3 / gemma3 (:331-333).  openelm's packed
    QKV projection is not part of this build and is rejected explicitly;
  * HF-style aliases -> GGUF names, incl. the tied LM head resolving to
    token_embd.weight when output.weight is absent (:342-369);
  * hyper-parameters from `{arch}.*` keys with the same fallbacks (:371-424):
    key_length defaults to hidden/heads, context_length to the ModelDef's,
    rope.freq_base to 10000, layer_norm_rms_epsilon to 1e-5;
  * qkNorm iff blk.0.attn_q_norm and blk.0.attn_k_norm both exist (:399);
  * ropeLayout "interleaved" for arch llama, "split" otherwise (:402);
  * gemma3: embedding scale sqrt(hidden) (:405), local theta 10000 and global
    theta from gemma3.rope.freq_base on layers i % 6 == 5, sliding window on
    the other layers (:384-385, :410-415).
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Dict, List, Optional

from .gguf import GGML_TYPE, GgufFile, GgufValue, metadata_number
from .registry import ModelDef


@dataclass
class TensorSpec:
    name: str
    ggml_type: int
    shape: List[int]          # reversed ggml shape: [rows, cols] (:433)
    offset: int               # absolute byte offset in the GGUF (:436)
    length: int


@dataclass
class LlamaModel:
    id: str
    hidden: int
    intermediate: int
    vocab: int
    layers: int
    heads: int
    kvHeads: int
    headDim: int
    maxContext: int
    ropeTheta: float
    normEps: float
    qkNorm: bool
    qkNormEps: float
    architecture: str         # "llama" | "gemma3"
    ropeLayout: str           # "interleaved" | "split"
    embeddingScale: float
    layerRopeTheta: List[float]
    layerAttentionWindow: List[int]
    activation: str           # "silu" | "gelu-tanh"


@dataclass
class LlamaManifest:
    model: LlamaModel
    aliases: Dict[str, str]
    tensors: Dict[str, TensorSpec]

    def resolve(self, name: str) -> str:
        return self.aliases.get(name, name)

    def has(self, name: str) -> bool:
        return self.resolve(name) in self.tensors

    def spec(self, name: str) -> TensorSpec:
        r = self.resolve(name)
        if r not in self.tensors:
            raise KeyError(f"Llama WGSL manifest missing tensor {name}")
        return self.tensors[r]


def gguf_number(g: GgufFile, key: str, fallback: Optional[float] = None) -> float:
    """llama-wgsl-runtime.ts:469-475"""
    v = g.kv.get(key)
    num = metadata_number(v.value) if v is not None else None
    if num is not None:
        return num
    if fallback is not None:
        return fallback
    raise ValueError(f"GGUF metadata {key} is missing or not numeric")


def gguf_string(g: GgufFile, key: str) -> str:
    v = g.kv.get(key)
    if v is not None and isinstance(v.value, str):
        return v.value
    raise ValueError(f"GGUF metadata {key} is missing or not a string")


SUPPORTED_TYPES = (GGML_TYPE.F32, GGML_TYPE.F16, GGML_TYPE.Q5_0, GGML_TYPE.Q5_1, GGML_TYPE.Q8_0,
                   GGML_TYPE.Q4_K, GGML_TYPE.Q5_K, GGML_TYPE.Q6_K)


def build_gguf_llama_manifest(model: ModelDef, g: GgufFile) -> LlamaManifest:
    arch = gguf_string(g, "general.architecture")
    if arch == "openelm":
        raise ValueError("Llama GGUF runtime: architecture openelm (packed QKV) is not supported by this build")
    if arch not in ("qwen3", "llama", "gemma3"):
        raise ValueError(f"Llama GGUF WGSL does not support architecture {arch}")
    is_gemma3 = arch == "gemma3"
    tensors: Dict[str, TensorSpec] = {}
    for t in g.tensors:
        if t.type not in SUPPORTED_TYPES:
            raise ValueError(f"unsupported GGUF tensor type {t.type}")
        tensors[t.name] = TensorSpec(t.name, t.type, list(reversed(t.shape)), g.data_offset + t.offset, t.n_bytes)

    aliases: Dict[str, str] = {
        "model.embed_tokens.weight": "token_embd.weight",
        f"model.layers.{model.layers}.final_norm_layernorm.weight": "output_norm.weight",
        "lm_head.MatMul.weight": "output.weight" if "output.weight" in g.tensor_map else "token_embd.weight",
    }
    for i in range(model.layers):
        p = f"model.layers.{i}."
        b = f"blk.{i}."
        aliases[p + "input_layernorm.weight"] = b + "attn_norm.weight"
        aliases[p + "post_attention_layernorm.weight"] = b + ("post_attention_norm.weight" if is_gemma3
                                                                 else "ffn_norm.weight")
        if is_gemma3:
            aliases[p + "pre_feedforward_layernorm.weight"] = b + "ffn_norm.weight"
            aliases[p + "post_feedforward_layernorm.weight"] = b + "post_ffw_norm.weight"
        aliases[p + "attn.q_norm.layernorm.weight"] = b + "attn_q_norm.weight"
        aliases[p + "attn.k_norm.layernorm.weight"] = b + "attn_k_norm.weight"
        aliases[p + "attn.q_proj.MatMul.weight"] = b + "attn_q.weight"
        aliases[p + "attn.k_proj.MatMul.weight"] = b + "attn_k.weight"
        aliases[p + "attn.v_proj.MatMul.weight"] = b + "attn_v.weight"
        aliases[p + "attn.o_proj.MatMul.weight"] = b + "attn_output.weight"
        aliases[p + "mlp.gate_proj.MatMul.weight"] = b + "ffn_gate.weight"
        aliases[p + "mlp.up_proj.MatMul.weight"] = b + "ffn_up.weight"
        aliases[p + "mlp.down_proj.MatMul.weight"] = b + "ffn_down.weight"

    layers = int(gguf_number(g, f"{arch}.block_count"))
    hidden = int(gguf_number(g, f"{arch}.embedding_length"))
    heads = int(gguf_number(g, f"{arch}.attention.head_count"))
    kv_heads = int(gguf_number(g, f"{arch}.attention.head_count_kv"))
    intermediate = int(gguf_number(g, f"{arch}.feed_forward_length"))
    head_dim = int(gguf_number(g, f"{arch}.attention.key_length", hidden // heads))
    sliding = int(gguf_number(g, "gemma3.attention.sliding_window", 0)) if is_gemma3 else 0
    global_theta = gguf_number(g, "gemma3.rope.freq_base", 1000000) if is_gemma3 else 0
    local_theta = 10000
    eps = gguf_number(g, f"{arch}.attention.layer_norm_rms_epsilon", 1e-5)
    rope_theta = local_theta if is_gemma3 else gguf_number(g, f"{arch}.rope.freq_base", 10000)
    if is_gemma3:
        layer_theta = [global_theta if i % 6 == 5 else local_theta for i in range(layers)]
        layer_window = [0 if i % 6 == 5 else sliding for i in range(layers)]
    else:
        layer_theta = [rope_theta] * layers
        layer_window = [0] * layers
    m = LlamaModel(
        id=model.id,
        hidden=hidden,
        intermediate=intermediate,
        vocab=model.vocab,
        layers=layers,
        heads=heads,
        kvHeads=kv_heads,
        headDim=head_dim,
        maxContext=int(min(model.maxContext, gguf_number(g, f"{arch}.context_length", model.maxContext))),
        ropeTheta=rope_theta,
        normEps=eps,
        qkNorm=("blk.0.attn_q_norm.weight" in g.tensor_map and "blk.0.attn_k_norm.weight" in g.tensor_map),
        qkNormEps=eps,
        architecture="gemma3" if is_gemma3 else "llama",
        ropeLayout="interleaved" if arch == "llama" else "split",
        embeddingScale=math.sqrt(hidden) if is_gemma3 else 1.0,
        layerRopeTheta=layer_theta,
        layerAttentionWindow=layer_window,
        activation="gelu-tanh" if is_gemma3 else "silu",
    )
    return LlamaManifest(m, aliases, tensors)
