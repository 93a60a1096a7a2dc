"""SentencePiece tokenizer over GGUF metadata (chonklm_b200.tokenizer) and the
host-side turn bookkeeping of the Gemma text runtime: CPU only."""
import numpy as np
import pytest

from chonklm_b200.gguf import ByteSource, fetch_gguf_header
from chonklm_b200.tokenizer import (SPACE, T_BYTE, T_CONTROL, T_NORMAL, T_UNKNOWN, SpmTokenizer, complete_utf8,
                                    synthetic_vocab)


def _mini():
    # hand-built vocabulary: the merge order is fixed by the scores
    pieces = [("<unk>", T_UNKNOWN, 0.0), ("<s>", T_CONTROL, 0.0), ("</s>", T_CONTROL, 0.0),
              (SPACE, T_NORMAL, -1.0), ("h", T_NORMAL, -2.0), ("e", T_NORMAL, -2.0), ("l", T_NORMAL, -2.0),
              ("o", T_NORMAL, -2.0), ("w", T_NORMAL, -2.0), ("r", T_NORMAL, -2.0), ("d", T_NORMAL, -2.0),
              (SPACE + "h", T_NORMAL, -0.5), (SPACE + "he", T_NORMAL, -0.4), ("ll", T_NORMAL, -0.3),
              ("llo", T_NORMAL, -0.35), (SPACE + "hello", T_NORMAL, -0.1), ("lo", T_NORMAL, -0.2),
              ("or", T_NORMAL, -0.6), ("ld", T_NORMAL, -0.7)]
    pieces += [(f"<0x{b:02X}>", T_BYTE, 0.0) for b in range(256)]
    toks = [p[0] for p in pieces]
    return SpmTokenizer(toks, [p[2] for p in pieces], [p[1] for p in pieces], bos_id=1, eos_id=2, unk_id=0,
                        add_space_prefix=True), toks


def test_merges_follow_scores():
    tk, toks = _mini()
    # ▁ h e l l o: "lo" (-0.2) first, then the new pair "l"+"lo" = "llo"
    # (-0.35) beats "▁h" (-0.5); then "▁h", "▁he" (-0.4) and "▁he"+"llo"
    got = [toks[i] for i in tk.encode("hello")]
    assert got == [SPACE + "hello"]
    # ▁ h e l: "▁h", then "▁he"; "▁hel" is not a piece
    assert [toks[i] for i in tk.encode("hel")] == [SPACE + "he", "l"]
    got = [toks[i] for i in tk.encode("world")]
    # ▁ w o r l d: "or"(-0.6), then "ld"(-0.7): ▁ w or ld
    assert got == [SPACE, "w", "or", "ld"]
    # characters with no piece fall back to their UTF-8 bytes
    ids = tk.encode("hé")
    assert [toks[i] for i in ids] == [SPACE + "h", "<0xC3>", "<0xA9>"]
    assert tk.decode(ids) == " hé"


@pytest.mark.parametrize("vocab", [1300, 5000])
def test_round_trip_random_text(vocab):
    toks, scores, types = synthetic_vocab(vocab)
    tk = SpmTokenizer(toks, scores, types, bos_id=2, eos_id=1, unk_id=3)
    rng = np.random.default_rng(vocab)
    alphabet = list("the and hello world model  user token 0123456789,.!?\n\t") + \
        ["é", "ü", "☕", "日", "本", "\U0001F600", "Ж"]
    for _ in range(200):
        s = "".join(rng.choice(alphabet, size=int(rng.integers(0, 40))))
        ids = tk.encode(s, special=False)
        assert tk.decode(ids) == s, (s, ids)
        assert all(0 <= i < vocab for i in ids)


def test_special_tokens_and_turn_template():
    toks, scores, types = synthetic_vocab(1300)
    tk = SpmTokenizer(toks, scores, types, bos_id=2, eos_id=1, unk_id=3)
    ids = tk.encode("<start_of_turn>user\nhello<end_of_turn>\n")
    assert ids[0] == toks.index("<start_of_turn>") and ids[-2] == toks.index("<end_of_turn>")
    assert tk.decode(ids) == "user\nhello\n"                     # control tokens dropped
    assert tk.decode(ids, skip_special=False) == "<start_of_turn>user\nhello<end_of_turn>\n"
    # longer words become single pieces
    assert len(tk.encode("hello world")) <= 3


def test_complete_utf8_holds_back_partial_characters():
    b = "a☕".encode("utf-8")
    assert complete_utf8(b[:1]) == "a"
    assert complete_utf8(b[:2]) == "a"
    assert complete_utf8(b[:3]) == "a"
    assert complete_utf8(b) == "a☕"


def test_gguf_tokenizer_metadata_round_trip(tiny_dir):
    from conftest import tiny_model
    path = tiny_model(tiny_dir, "gemma3", "q4_k_m", tokenizer=True)
    g = fetch_gguf_header(ByteSource(path))
    tk = SpmTokenizer.from_gguf(g.kv)
    toks, scores, types = synthetic_vocab(1300)
    assert tk.tokens == toks and tk.types == types
    assert np.allclose(tk.scores, np.float32(scores))
    assert tk.bos_id == toks.index("<bos>") and tk.eos_id == toks.index("<eos>")
    assert not tk.add_space_prefix


def test_gemma_turn_bookkeeping():
    """Prompt ids of the first and a following turn (no GPU: the engine is
    only used by generate)."""
    from chonklm_b200.gemma_runtime import GemmaEngine
    toks, scores, types = synthetic_vocab(1300)
    tk = SpmTokenizer(toks, scores, types, bos_id=2, eos_id=1, unk_id=3)
    e = GemmaEngine(loaded=None, tok=tk)
    e.addUserMessage("hello")
    first = list(e._pending)
    assert first[0] == tk.bos_id
    assert first[1:] == tk.encode("<start_of_turn>user\nhello<end_of_turn>\n<start_of_turn>model\n")
    e._pending = []
    e._unfed = tk.special["<end_of_turn>"]          # a reply that ended normally
    e.addUserMessage("again")
    assert e._pending == [tk.special["<end_of_turn>"]] + tk.encode("\n") + \
        tk.encode("<start_of_turn>user\nagain<end_of_turn>\n<start_of_turn>model\n")
    e._pending = []
    e._unfed = 500                                   # a reply cut at maxTokens
    e.addUserMessage("x")
    assert e._pending[:2] == [500, tk.special["<end_of_turn>"]]
