"""Model registry: the `ModelDef` record the runtime loads from.

Mirrors `src/lib/registry.ts` (`ModelDef` :14-46, `getModel` :640) for the
fields the llama-webgpu runtime reads: `runtime`, `vocab`, `layers`, `kvHeads`,
`headDim`, `maxContext`, `eosIds`, `base`/`gguf` (model file location),
`defaultRepetitionPenalty`.  `kvDtype` selects the device KV-cache element
type; the reference only knows "float32" (:26), this build adds "float16".

The entries below are the synthetic stand-ins for the registry's SmolLM2-135M,
Qwen3-0.6B and Gemma-3-270M GGUF models (registry.ts:117-136, :179-226,
:445-484): same shapes and context limits, weights generated from a seed by
`chonklm_b200.synth` because no real model files exist on these machines.
"""
from __future__ import annotations

import dataclasses
from dataclasses import dataclass, field
from typing import List, Optional


@dataclass
class ModelDef:
    id: str
    label: str
    kind: str = "llama"
    runtime: str = "llama-webgpu"
    pitch: str = ""
    chat: bool = False
    eosIds: List[int] = field(default_factory=list)
    vocab: int = 0
    layers: int = 0
    kvHeads: int = 0
    headDim: int = 0
    kvDtype: str = "float16"
    maxContext: int = 0
    base: str = ""
    gguf: str = ""
    tokenizer: Optional[str] = None
    defaultRepetitionPenalty: Optional[float] = None
    defaultTemperature: Optional[float] = None
    defaultTopP: Optional[float] = None
    defaultTopK: Optional[int] = None

    def replace(self, **kw) -> "ModelDef":
        return dataclasses.replace(self, **kw)


MODELS: List[ModelDef] = [
    ModelDef(id="smollm2-135m-q4-k-m-synthetic", label="SmolLM2-135M-shaped (Q4_K_M, synthetic)",
             eosIds=[2], vocab=49152, layers=30, kvHeads=3, headDim=64, maxContext=512,
             base="", gguf="smollm2-135m-q4_k_m.gguf"),
    ModelDef(id="qwen3-0.6b-q4-k-m-synthetic", label="Qwen3-0.6B-shaped (Q4_K_M, synthetic)",
             eosIds=[151645, 151643], vocab=151936, layers=28, kvHeads=8, headDim=128, maxContext=2048,
             base="", gguf="qwen3-0.6b-q4_k_m.gguf"),
    ModelDef(id="qwen3-0.6b-q8-synthetic", label="Qwen3-0.6B-shaped (Q8_0, synthetic)",
             eosIds=[151645, 151643], vocab=151936, layers=28, kvHeads=8, headDim=128, maxContext=2048,
             base="", gguf="qwen3-0.6b-q8_0.gguf"),
    ModelDef(id="gemma-3-270m-q4-k-m-synthetic", label="Gemma-3-270M-shaped (Q4_K_M, synthetic)",
             eosIds=[1, 106], vocab=262144, layers=18, kvHeads=1, headDim=256, maxContext=512,
             base="", gguf="gemma-3-270m-q4_k_m.gguf"),
]


def getModel(model_id: str) -> ModelDef:
    """registry.ts:640-644."""
    for m in MODELS:
        if m.id == model_id:
            return m
    raise KeyError(f"unknown model id: {model_id}")
