"""Text-level Gemma runtime (gemma-runtime.ts interface) on the GPU engine:
the ids behind generateGemma's text equal the oracle's greedy ids over the
same token sequence, turn after turn (the conversation stays in the KV
cache), and sampled replies equal generateLlamaWgsl's on the same ids."""
import numpy as np
import pytest

from conftest import tiny_model
from chonklm_b200.gemma_runtime import disposeGemma, generateGemma, loadGemmaModel, resetGemmaConversation
from chonklm_b200.registry import ModelDef
from oracle import oracle

pytestmark = pytest.mark.gpu


def _def(path):
    return ModelDef(id="g", label="g", runtime="gemma-webgpu", maxContext=256, gguf=path, eosIds=[1, 5])


def _oracle_greedy(orc, history, n, stop):
    """Run history through the oracle; greedy ids after it, up to a stop id."""
    orc.reset()
    for t in history[:-1]:
        orc.run_token(t, False)
    nid = orc.run_token(history[-1], True)
    out = []
    for _ in range(n):
        out.append(nid)
        if nid in stop:
            break
        nid = orc.run_token(nid, True)
    return out


def test_generate_gemma_greedy_two_turns(tiny_dir):
    path = tiny_model(tiny_dir, "gemma3", "q4_k_m", tokenizer=True)
    loaded = loadGemmaModel(_def(path))
    eng = loaded.engine
    tk = eng.tokenizer
    orc = oracle.OracleModel(path, max_context=256)
    history = [{"role": "user", "content": "hello world, the model answers"}]
    seen = []
    r1 = generateGemma(loaded, history, {"maxNewTokens": 24, "temperature": 0,
                                         "onToken": lambda d: seen.append(d["text"])})
    ids1 = list(eng.last_reply_ids)
    want1 = _oracle_greedy(orc, eng.history_ids[:len(eng.history_ids) - len(ids1)], 24, eng._stop)
    assert ids1 == want1
    text_ids = [i for i in ids1 if i not in eng._stop]
    assert r1["text"] == tk.decode(text_ids) == "".join(seen)
    assert r1["generatedTokens"] == len(text_ids)
    # second turn: only the new ids are prefilled; the oracle replays everything
    history += [{"role": "assistant", "content": r1["text"]}, {"role": "user", "content": "and again?"}]
    pos_before = eng.position
    r2 = generateGemma(loaded, history, {"maxNewTokens": 16, "temperature": 0})
    ids2 = list(eng.last_reply_ids)
    prompt2 = eng.history_ids[:len(eng.history_ids) - len(ids2)]
    assert pos_before < len(prompt2)   # the first turn's rows were reused, not recomputed
    assert ids2 == _oracle_greedy(orc, prompt2, 16, eng._stop)
    assert r2["text"] == tk.decode([i for i in ids2 if i not in eng._stop])
    resetGemmaConversation(loaded)
    assert eng.position == 0 and loaded.turnsReplayed == 0
    disposeGemma(loaded)


def test_generate_gemma_sampled_matches_llama_runtime(tiny_dir):
    """temperature 1 / top-k 64 / top-p 0.95 (Gemma's defaults) through the
    text API and through generateLlamaWgsl on the same prompt ids and seed."""
    from chonklm_b200.runtime import generateLlamaWgsl, loadLlamaWgslModel
    path = tiny_model(tiny_dir, "gemma3", "q4_k_m", tokenizer=True)
    loaded = loadGemmaModel(_def(path))
    r = generateGemma(loaded, [{"role": "user", "content": "please answer the question"}],
                      {"maxNewTokens": 20, "temperature": 1.0})
    ids = list(loaded.engine.last_reply_ids)
    prompt = loaded.engine.history_ids[:len(loaded.engine.history_ids) - len(ids)]
    disposeGemma(loaded)
    ll = loadLlamaWgslModel(ModelDef(id="l", label="l", vocab=1300, maxContext=256, gguf=path, eosIds=[1, 5]))
    ref = generateLlamaWgsl(ll, prompt, {"maxNewTokens": 20, "temperature": 1.0, "topP": 0.95, "topK": 64,
                                         "seed": 0})
    ll.engine.dispose()
    assert ids == ref["ids"]
    assert len(r["text"]) > 0
