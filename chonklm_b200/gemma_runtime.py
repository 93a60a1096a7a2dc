"""Text-level Gemma runtime: the gemma-webgpu interface on the B200 engine.

Same entry points, argument meaning and error behaviour as
src/lib/gemma-runtime.ts:
  loadGemmaModel(model, onProgress?, onStep?)          :22-52
  generateGemma(loaded, history, opts)                 :77-107
  disposeGemma(loaded)                                 :109-111
  resetGemmaConversation(loaded)                       :113-116
and the engine surface they use from `gemma-webgpu` (`createGemmaEngine`,
`addUserMessage`, `generate`, `resetConversation`, `dispose`) as
`GemmaEngine`.

That engine is a third-party package (`gemma-webgpu@0.1.0`) whose source is
not in the reference tree, so its arithmetic is not pinned; here the model
runs on this repository's engine (the gemma3 graph of the llama runtime,
covered by its parity tests), the vocabulary comes from the GGUF file
(`tokenizer.SpmTokenizer`) and conversations use Gemma's turn format:

    <bos><start_of_turn>user\\n{text}<end_of_turn>\\n<start_of_turn>model\\n

A reply ends at <end_of_turn> or <eos> (neither is part of the text).  The
conversation stays in the KV cache between turns: each generate() prefills
only what was added since the last one.  Sampling options follow
generateGemma (maxTokens, temperature, topP, repPenalty; topK 64 and top-p
0.95 at temperature 1 unless given, Gemma's published defaults), drawing
from the engine's Philox stream (`seed`) instead of Math.random.
"""
from __future__ import annotations

import time
from dataclasses import dataclass
from typing import Any, Callable, Dict, Iterator, List, Optional

from . import _lib
from .gguf import ByteSource, fetch_gguf_header
from .registry import ModelDef
from .runtime import LoadedLlamaWgslModel, _model_path, loadLlamaWgslModel, needsSamplingReadback
from .tokenizer import SpmTokenizer, complete_utf8


class GemmaEngine:
    """The `GemmaEngine` surface generateGemma drives (gemma-runtime.ts:84-101)."""

    def __init__(self, loaded: LoadedLlamaWgslModel, tok: SpmTokenizer, seed: int = 0):
        self._loaded = loaded
        self.tokenizer = tok
        self._seed = seed
        self._draws = 0
        self._pending: List[int] = []     # ids added since the last generate()
        self._unfed: Optional[int] = None  # the last reply's final id (never run through the model)
        self._started = False
        self.history_ids: List[int] = []   # every id of the conversation, in order
        self._stop = {i for i in (tok.eos_id, tok.special.get("<end_of_turn>")) if i is not None}

    @property
    def position(self) -> int:
        return self._loaded.engine.position

    def addUserMessage(self, text: str) -> None:
        tk = self.tokenizer
        ids: List[int] = []
        if self._unfed is not None:            # close the previous model turn
            ids.append(self._unfed)
            if self._unfed not in self._stop:  # the reply was cut short: end its turn
                ids += tk.encode("<end_of_turn>")
            self._unfed = None
            ids += tk.encode("\n")
        elif not self._started and tk.bos_id is not None:
            ids.append(tk.bos_id)
        self._started = True
        ids += tk.encode("<start_of_turn>user\n" + text + "<end_of_turn>\n<start_of_turn>model\n")
        self._pending += ids

    def generate(self, maxTokens: Optional[int] = None, temperature: Optional[float] = None,
                 topP: Optional[float] = None, topK: Optional[int] = None,
                 repPenalty: Optional[float] = None) -> Iterator[str]:
        """Yield the reply as text pieces, one per generated id (a piece may be
        empty while a multi-byte character is incomplete)."""
        if not self._pending:
            raise RuntimeError("GemmaEngine.generate: no user message since the last reply")
        eng = self._loaded.engine.dev
        ctx = self._loaded.engine.contextLength
        t = 1.0 if temperature is None else float(temperature)
        samp = {"temperature": t,
                "topP": (0.95 if t > 0 else 1.0) if topP is None else float(topP),
                "topK": (64 if t > 0 else 0) if topK is None else int(topK),
                "repetitionPenalty": 1.0 if repPenalty is None else float(repPenalty)}
        sampled = needsSamplingReadback(samp)

        def mk():
            s, _ = _lib.make_sampling(samp["temperature"], samp["topP"], samp["topK"], samp["repetitionPenalty"],
                                      self._seed, self._draws)
            return s

        prompt, self._pending = self._pending, []
        room = ctx - eng.position - len(prompt)
        if room <= 0:
            raise _lib.ContextExhausted(f"Gemma conversation exceeds the context of {ctx} tokens")
        mx = room if maxTokens is None else min(int(maxTokens), room)
        self.history_ids += prompt
        nid = eng.prefill(prompt, True, mk())
        if sampled:
            self._draws += 1
        reply: List[int] = []
        self.last_reply_ids = reply
        text = ""
        try:
            for step in range(mx):
                reply.append(nid)
                self.history_ids.append(nid)
                if nid in self._stop:
                    break
                full = complete_utf8(self.tokenizer.decode_bytes(reply))
                piece, text = full[len(text):], full
                yield piece
                if step + 1 >= mx:
                    break
                nid = eng.run_token(nid, True, mk())
                if sampled:
                    self._draws += 1
        finally:
            # also when the caller stops early: the reply's last id has not
            # been run through the model yet
            self._unfed = reply[-1] if reply else None

    def resetConversation(self) -> None:
        self._loaded.engine.reset()
        self._pending, self._unfed, self._started, self._draws = [], None, False, 0
        self.history_ids = []

    def dispose(self) -> None:
        self._loaded.engine.dispose()


def createGemmaEngine(opts: Dict[str, Any], device: int = 0) -> GemmaEngine:
    """gemma-webgpu's createGemmaEngine({model, contextLength, onProgress})."""
    model = opts["model"]
    if isinstance(model, ModelDef):
        mdef = model
    else:
        mdef = ModelDef(id=str(model), label=str(model), gguf=str(model))
    src = ByteSource(_model_path(mdef))
    tok = SpmTokenizer.from_gguf(fetch_gguf_header(src).kv)
    ctx = int(opts.get("contextLength") or mdef.maxContext or 512)
    on_progress = opts.get("onProgress")

    def progress(p):
        if on_progress:
            on_progress({"status": "loading weights", "loaded": p["loaded"], "total": p["total"]})

    llama_def = mdef.replace(runtime="llama-webgpu", maxContext=ctx, vocab=mdef.vocab or len(tok.tokens))
    loaded = loadLlamaWgslModel(llama_def, progress, None, device)
    return GemmaEngine(loaded, tok, int(opts.get("seed", 0)))


@dataclass
class LoadedGemmaModel:
    """gemma-runtime.ts:9-20"""
    runtime: str
    def_: ModelDef
    engine: GemmaEngine
    ep: str = "cuda"
    turnsReplayed: int = 0


def loadGemmaModel(model: ModelDef, onProgress: Optional[Callable] = None, onStep: Optional[Callable] = None,
                   device: int = 0) -> LoadedGemmaModel:
    """gemma-runtime.ts:22-52"""
    if not model.gguf:
        raise ValueError(f"gemma-webgpu model {model.id} missing 'gguf' URL")
    if onStep:
        onStep({"step": "runtime", "detail": "creating Gemma B200 engine"})

    def prog(p):
        if onStep:
            onStep({"step": "weights", "detail": p["status"]})
        if onProgress:
            onProgress({"url": model.gguf, "loaded": p["loaded"], "total": p["total"] if p["total"] > 0 else None,
                        "fromNetwork": False, "status": p["status"]})

    engine = createGemmaEngine({"model": model, "contextLength": model.maxContext, "onProgress": prog}, device)
    if onStep:
        onStep({"step": "ready", "detail": "Gemma B200 engine ready"})
    return LoadedGemmaModel("gemma-webgpu", model, engine)


def generateGemma(loaded: LoadedGemmaModel, history: List[Dict[str, str]],
                  opts: Optional[Dict[str, Any]] = None) -> Dict[str, Any]:
    """gemma-runtime.ts:77-107: replay the user turns the engine has not seen,
    then stream the reply."""
    opts = opts or {}
    for msg in history[loaded.turnsReplayed:]:
        if msg.get("role") == "user":
            loaded.engine.addUserMessage(msg["content"])
    loaded.turnsReplayed = len(history)
    t0 = time.perf_counter()
    cumulative = ""
    count = 0
    on_token = opts.get("onToken")
    should_stop = opts.get("shouldStop")
    for piece in loaded.engine.generate(maxTokens=opts.get("maxNewTokens"), temperature=opts.get("temperature"),
                                        topP=opts.get("topP"), repPenalty=opts.get("repetitionPenalty")):
        if should_stop and should_stop():
            break
        cumulative += piece
        count += 1
        if on_token:
            on_token({"text": piece, "cumulative": cumulative})
    elapsed = time.perf_counter() - t0
    return {"text": cumulative, "tokensPerSec": count / max(elapsed, 1e-3), "generatedTokens": count}


def disposeGemma(loaded: LoadedGemmaModel) -> None:
    """gemma-runtime.ts:109-111"""
    loaded.engine.dispose()


def resetGemmaConversation(loaded: LoadedGemmaModel) -> None:
    """gemma-runtime.ts:113-116"""
    loaded.engine.resetConversation()
    loaded.turnsReplayed = 0
