"""Host runtime: the module API of ChonkLM's llama-webgpu runtime on the B200
engine.

Same entry points, argument meaning and error behaviour as
src/lib/llama-wgsl-runtime.ts:
  loadLlamaWgslModel(model, onProgress?, onStep?)            :184-240
  generateLlamaWgsl(loaded, promptIds, opts)                 :242-314
  disposeLlamaWgsl(loaded)                                   :316-318
  resetLlamaWgslConversation(loaded)                         :320-324
and the engine surface they use (runToken / reset / position / dispose,
:1011-1150) as `LlamaEngine`.

Differences, all deliberate: weights come from a local GGUF file or shard
directory instead of HTTP + Cache API; the KV cache may be fp16 (the
ModelDef's kvDtype, default "float16"); sampling draws come from a Philox
stream (`seed` option) instead of Math.random; there is no tokenizer on this
path, so `text` stays "" unless the loaded model is given a `decode` callable.
"""
from __future__ import annotations

import math
import os
import time
from dataclasses import dataclass, field
from typing import Any, Callable, Dict, List, Optional, Sequence

import numpy as np

from . import _lib
from .gguf import ByteSource, GGML_TYPE, fetch_gguf_header
from .manifest import LlamaManifest, build_gguf_llama_manifest
from .registry import ModelDef


def needsSamplingReadback(sampling: Optional[Dict[str, Any]]) -> bool:
    """sampling.ts:9-16"""
    if not sampling:
        return False
    t = sampling.get("temperature") or 0
    p = sampling.get("topP")
    k = sampling.get("topK")
    kk = max(0, int(math.floor(k))) if isinstance(k, (int, float)) and math.isfinite(k) else 0
    return t > 0 or (1 if p is None else p) < 1 or kk > 0


def _model_path(model: ModelDef) -> str:
    p = model.gguf
    if os.path.isabs(p) or not model.base:
        return p
    return os.path.join(model.base, p)


def _engine_cfg(m, context_length: int, kv_dtype: str) -> "_lib.ck_model_cfg":
    c = _lib.ck_model_cfg()
    c.hidden, c.intermediate, c.vocab, c.layers = m.hidden, m.intermediate, m.vocab, m.layers
    c.heads, c.kv_heads, c.head_dim = m.heads, m.kvHeads, m.headDim
    c.context_length = context_length
    c.norm_eps = float(np.float32(m.normEps))
    c.qk_norm_eps = float(np.float32(m.qkNormEps))
    c.embedding_scale = float(np.float32(m.embeddingScale))
    c.arch = _lib.CK_ARCH_GEMMA3 if m.architecture == "gemma3" else _lib.CK_ARCH_LLAMA
    c.rope_interleaved = 1 if m.ropeLayout == "interleaved" else 0
    c.qk_norm = 1 if m.qkNorm else 0
    c.kv_dtype = _lib.CK_KV_F32 if kv_dtype == "float32" else _lib.CK_KV_F16
    if m.layers > _lib.CK_MAX_LAYERS:
        raise ValueError(f"{m.layers} layers exceeds {_lib.CK_MAX_LAYERS}")
    for i in range(m.layers):
        c.layer_rope_theta[i] = int(math.floor(m.layerRopeTheta[i] + 0.5))   # Math.round (:1477)
        c.layer_window[i] = int(m.layerAttentionWindow[i])
    return c


class LlamaEngine:
    """Engine surface of LlamaWgslEngine on the B200 (runToken :1025-1150,
    reset :1011, position :1021, dispose :1152)."""

    def __init__(self, engine: "_lib.Engine", manifest: LlamaManifest, context_length: int):
        self.dev = engine
        self.m = manifest.model
        self.contextLength = context_length

    def runToken(self, tokenId: int, needLogits: bool, opts: Optional[Dict[str, Any]] = None) -> int:
        opts = opts or {}
        pen = opts.get("penalizedTokenIds")
        s, keep = _lib.make_sampling(opts.get("temperature", 0), opts.get("topP", 1), opts.get("topK", 0),
                                     opts.get("repetitionPenalty", 1), opts.get("seed", 0),
                                     opts.get("philoxOffset", 0), pen)
        return self.dev.run_token(tokenId, needLogits, s)

    def reset(self) -> None:
        self.dev.reset()

    @property
    def position(self) -> int:
        return self.dev.position

    def dispose(self) -> None:
        self.dev.close()


@dataclass
class LoadedLlamaWgslModel:
    """llama-wgsl-runtime.ts:174-182"""
    runtime: str
    def_: ModelDef
    tokenizer: Any
    engine: LlamaEngine
    ep: str = "cuda"
    cachedTokenIds: List[int] = field(default_factory=list)
    cachedNextId: Optional[int] = None
    manifest: Optional[LlamaManifest] = None

    @property
    def def_model(self) -> ModelDef:
        return self.def_


def loadLlamaWgslModel(model: ModelDef, onProgress: Optional[Callable] = None, onStep: Optional[Callable] = None,
                       device: int = 0) -> LoadedLlamaWgslModel:
    """llama-wgsl-runtime.ts:184-240: parse the GGUF header, build the
    manifest, upload every tensor the step reads, finalize the engine."""
    if model.runtime != "llama-webgpu":
        raise ValueError(f"loadLlamaWgslModel: {model.id} is not configured for the Llama WGSL runtime")
    if onStep:
        onStep({"step": "runtime", "detail": "opening B200 engine"})
    src = ByteSource(_model_path(model))
    gguf = fetch_gguf_header(src)
    manifest = build_gguf_llama_manifest(model, gguf)
    context_length = min(model.maxContext, manifest.model.maxContext)
    eng = _lib.Engine(_engine_cfg(manifest.model, context_length, model.kvDtype), device)
    try:
        names = [t.name for t in gguf.tensors]
        total = sum(manifest.tensors[n].length for n in names)
        done = 0
        for i, name in enumerate(names):
            spec = manifest.tensors[name]
            data = src.read(spec.offset, spec.length)
            eng.upload(name, spec.ggml_type, list(reversed(spec.shape)), data)
            done += spec.length
            if onProgress:
                onProgress({"url": src.name, "loaded": done, "total": total, "fromNetwork": False})
            if onStep and name.startswith("blk.") and name.endswith("ffn_down.weight"):
                layer = int(name.split(".")[1])
                onStep({"step": "weights", "detail": f"uploaded layer {layer + 1} / {manifest.model.layers} to GPU",
                        "progress": {"current": layer + 1, "total": manifest.model.layers}})
        eng.finalize()
    except Exception:
        eng.close()
        raise
    if onStep:
        onStep({"step": "ready", "detail": "Llama B200 runtime ready"})
    return LoadedLlamaWgslModel("llama-webgpu", model, None, LlamaEngine(eng, manifest, context_length),
                                manifest=manifest)


def commonPrefixLength(a: Sequence[int], b: Sequence[int]) -> int:
    """llama-wgsl-runtime.ts:1812-1817"""
    n = min(len(a), len(b))
    i = 0
    while i < n and a[i] == b[i]:
        i += 1
    return i


def generateLlamaWgsl(loaded: LoadedLlamaWgslModel, promptIds: Sequence[int],
                      opts: Optional[Dict[str, Any]] = None) -> Dict[str, Any]:
    """llama-wgsl-runtime.ts:242-314, step for step.

    With neither onToken nor shouldStop the decode loop runs on the device
    (ck_decode) without a host round trip per token; otherwise each token
    comes back to the host as in the reference loop.  Both give the same ids.
    """
    opts = opts or {}
    d = loaded.def_
    prompt = [int(t) for t in promptIds]
    mx = min(opts.get("maxNewTokens", 128) if opts.get("maxNewTokens") is not None else 128,
             d.maxContext - len(prompt))
    eos = set(d.eosIds)
    rp = opts.get("repetitionPenalty")
    if rp is None:
        rp = d.defaultRepetitionPenalty if d.defaultRepetitionPenalty is not None else 1
    sampling = {"temperature": opts.get("temperature", 0) or 0,
                "topP": 1 if opts.get("topP") is None else opts.get("topP"),
                "topK": opts.get("topK", 0) or 0,
                "repetitionPenalty": rp}
    seed = int(opts.get("seed", 0))
    # candidate list of the sampler (an extension of the reference's options):
    # "chunk" (default) = the reference's per-256 chunk maxima, "exact" = the
    # top-K of the whole vocabulary (ck_set_sampler)
    loaded.engine.dev.set_sampler(opts.get("sampler", "chunk") == "exact")
    on_token = opts.get("onToken")
    should_stop = opts.get("shouldStop")
    decode_text = getattr(loaded.tokenizer, "decode", None)
    eng = loaded.engine.dev
    sampled = needsSamplingReadback(sampling)
    draws = 0

    def mk(offset: int):
        s, _ = _lib.make_sampling(sampling["temperature"], sampling["topP"], sampling["topK"],
                                  sampling["repetitionPenalty"], seed, offset)
        return s

    t0 = time.perf_counter()
    prefix_len = commonPrefixLength(loaded.cachedTokenIds, prompt)
    if prefix_len != len(loaded.cachedTokenIds):
        loaded.engine.reset()
        loaded.cachedTokenIds = []
        loaded.cachedNextId = None
        prefix_len = 0

    next_id = 0
    suffix = prompt[prefix_len:]
    if len(suffix) == 0 and loaded.cachedNextId is not None:
        next_id = loaded.cachedNextId
    elif suffix:
        next_id = eng.prefill(suffix, True, mk(draws))
        if sampled:
            draws += 1

    generated: List[int] = []
    cumulative = ""
    if mx > 0 and not on_token and not should_stop:
        ids = eng.decode(next_id, mx, mk(draws), sorted(eos))
        generated = ids
        next_id = ids[-1] if ids else next_id
        if decode_text:
            cumulative = decode_text(generated)
    else:
        for step in range(mx):
            if should_stop and should_stop():
                break
            generated.append(next_id)
            if decode_text:
                full = decode_text(generated)
                piece = full[len(cumulative):]
                cumulative = full
            else:
                piece = ""
            if on_token:
                on_token({"id": next_id, "text": piece, "cumulative": cumulative})
            if next_id in eos:
                break
            if step + 1 >= mx:
                break
            next_id = eng.run_token(next_id, True, mk(draws))
            if sampled:
                draws += 1

    loaded.cachedTokenIds = prompt + generated
    last = generated[-1] if generated else -1
    loaded.cachedNextId = None if last in eos else next_id
    elapsed = time.perf_counter() - t0
    return {"text": cumulative, "ids": generated, "tokensPerSec": len(generated) / max(elapsed, 1e-3)}


def disposeLlamaWgsl(loaded: LoadedLlamaWgslModel) -> None:
    """llama-wgsl-runtime.ts:316-318"""
    loaded.engine.dispose()


def resetLlamaWgslConversation(loaded: LoadedLlamaWgslModel) -> None:
    """llama-wgsl-runtime.ts:320-324"""
    loaded.engine.reset()
    loaded.cachedTokenIds = []
    loaded.cachedNextId = None
