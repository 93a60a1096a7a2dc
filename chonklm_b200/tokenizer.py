"""SentencePiece-style tokenizer read from a GGUF file's `tokenizer.ggml.*`
metadata (the vocabulary a Gemma GGUF carries).

The reference's gemma-webgpu runtime (`src/lib/gemma-runtime.ts:22-111`)
hands text to the third-party `gemma-webgpu@0.1.0` engine, which tokenizes
from the model file itself; that package is not in the reference tree, so
this is a restatement of the published SentencePiece BPE procedure over the
GGUF vocabulary, not of its code:

* encode: spaces become U+2581 ("▁") (plus one in front when
  `tokenizer.ggml.add_space_prefix` is set); control / user-defined token
  strings are matched first (longest match) and kept whole; each remaining
  run starts as single characters and adjacent symbols are merged
  repeatedly, always the pair whose merged piece is in the vocabulary with
  the highest score (leftmost on ties); a final symbol not in the vocabulary
  falls back to its UTF-8 bytes as <0xXX> tokens (else the unknown id).
* decode: byte tokens give their byte, "▁" gives a space, control tokens are
  dropped unless asked for; the bytes are decoded as UTF-8.

Only the SentencePiece model (`tokenizer.ggml.model == "llama"`, used by
Gemma and Llama-2 GGUFs) is handled.
"""
from __future__ import annotations

import heapq
from typing import Dict, Iterable, List, Optional, Sequence, Tuple

SPACE = "▁"
# tokenizer.ggml.token_type values
T_NORMAL, T_UNKNOWN, T_CONTROL, T_USER, T_UNUSED, T_BYTE = 1, 2, 3, 4, 5, 6


class SpmTokenizer:
    def __init__(self, tokens: Sequence[str], scores: Sequence[float], types: Sequence[int], *,
                 bos_id: Optional[int] = None, eos_id: Optional[int] = None, unk_id: Optional[int] = None,
                 add_space_prefix: bool = False, add_bos: bool = True):
        if not (len(tokens) == len(scores) == len(types)):
            raise ValueError("tokenizer: tokens, scores and token types differ in length")
        self.tokens = list(tokens)
        self.scores = [float(s) for s in scores]
        self.types = [int(t) for t in types]
        self.bos_id, self.eos_id, self.unk_id = bos_id, eos_id, unk_id
        self.add_space_prefix = add_space_prefix
        self.add_bos = add_bos
        self.piece_id: Dict[str, int] = {}
        self.byte_id: Dict[int, int] = {}
        self.special: Dict[str, int] = {}
        for i, (t, ty) in enumerate(zip(self.tokens, self.types)):
            if ty == T_BYTE and len(t) == 6 and t.startswith("<0x") and t.endswith(">"):
                self.byte_id[int(t[3:5], 16)] = i
            elif ty in (T_CONTROL, T_USER):
                self.special.setdefault(t, i)
            elif ty in (T_NORMAL, T_UNKNOWN):
                self.piece_id.setdefault(t, i)
        self._special_by_len = sorted(self.special, key=len, reverse=True)

    # ---- construction from GGUF metadata ---------------------------------------
    @classmethod
    def from_gguf(cls, kv) -> "SpmTokenizer":
        def val(key, default=None):
            v = kv.get(key)
            if v is None:
                return default
            v = getattr(v, "value", v)
            if isinstance(v, list):
                return [getattr(x, "value", x) for x in v]
            return v
        model = val("tokenizer.ggml.model")
        if model != "llama":
            raise ValueError(f"tokenizer model {model!r} is not supported (SentencePiece 'llama' only)")
        tokens = val("tokenizer.ggml.tokens")
        if not tokens:
            raise ValueError("GGUF has no tokenizer.ggml.tokens")
        scores = val("tokenizer.ggml.scores") or [0.0] * len(tokens)
        types = val("tokenizer.ggml.token_type") or [T_NORMAL] * len(tokens)
        return cls(tokens, scores, types, bos_id=val("tokenizer.ggml.bos_token_id"),
                   eos_id=val("tokenizer.ggml.eos_token_id"), unk_id=val("tokenizer.ggml.unknown_token_id"),
                   add_space_prefix=bool(val("tokenizer.ggml.add_space_prefix", False)),
                   add_bos=bool(val("tokenizer.ggml.add_bos_token", True)))

    def token_id(self, piece: str) -> int:
        if piece in self.special:
            return self.special[piece]
        if piece in self.piece_id:
            return self.piece_id[piece]
        raise KeyError(piece)

    # ---- encode --------------------------------------------------------------------
    def _split_special(self, text: str) -> List[Tuple[bool, str]]:
        out: List[Tuple[bool, str]] = []
        i, start = 0, 0
        while i < len(text):
            hit = None
            if self._special_by_len:
                for s in self._special_by_len:
                    if text.startswith(s, i):
                        hit = s
                        break
            if hit:
                if start < i:
                    out.append((False, text[start:i]))
                out.append((True, hit))
                i += len(hit)
                start = i
            else:
                i += 1
        if start < len(text):
            out.append((False, text[start:]))
        return out

    def _bpe(self, text: str) -> List[int]:
        syms = list(text)
        if not syms:
            return []
        # doubly linked symbols; a heap of candidate merges (-score, left index, left, right)
        prev = list(range(-1, len(syms) - 1))
        nxt = list(range(1, len(syms) + 1))
        nxt[-1] = -1
        alive = [True] * len(syms)
        heap: List[Tuple[float, int, str, str]] = []

        def push(a: int):
            b = nxt[a]
            if a < 0 or b < 0:
                return
            m = syms[a] + syms[b]
            j = self.piece_id.get(m)
            if j is not None:
                heapq.heappush(heap, (-self.scores[j], a, syms[a], syms[b]))

        for a in range(len(syms) - 1):
            push(a)
        while heap:
            _, a, sa, sb = heapq.heappop(heap)
            b = nxt[a] if alive[a] else -1
            if b < 0 or not alive[b] or syms[a] != sa or syms[b] != sb:
                continue   # stale: one side changed since this pair was queued
            syms[a] = sa + sb
            alive[b] = False
            nxt[a] = nxt[b]
            if nxt[b] >= 0:
                prev[nxt[b]] = a
            if prev[a] >= 0:
                push(prev[a])
            push(a)
        ids: List[int] = []
        a = 0
        while a >= 0:
            s = syms[a]
            j = self.piece_id.get(s)
            if j is not None:
                ids.append(j)
            else:
                for byte in s.encode("utf-8"):
                    if byte in self.byte_id:
                        ids.append(self.byte_id[byte])
                    elif self.unk_id is not None:
                        ids.append(self.unk_id)
                    else:
                        raise ValueError(f"tokenizer: no piece, byte token or unknown id for {s!r}")
            a = nxt[a]
        return ids

    def encode(self, text: str, add_bos: bool = False, special: bool = True) -> List[int]:
        ids: List[int] = []
        if add_bos and self.bos_id is not None:
            ids.append(self.bos_id)
        parts = self._split_special(text) if special else [(False, text)]
        first = True
        for is_special, s in parts:
            if is_special:
                ids.append(self.special[s])
            else:
                t = s.replace(" ", SPACE)
                if first and self.add_space_prefix:
                    t = SPACE + t
                ids.extend(self._bpe(t))
            first = False
        return ids

    # ---- decode --------------------------------------------------------------------
    def decode_bytes(self, ids: Iterable[int], skip_special: bool = True) -> bytes:
        out = bytearray()
        for i in ids:
            i = int(i)
            if i < 0 or i >= len(self.tokens):
                continue
            ty = self.types[i]
            if ty == T_BYTE and len(self.tokens[i]) == 6:
                out.append(int(self.tokens[i][3:5], 16))
            elif ty in (T_CONTROL, T_UNUSED) or (ty == T_UNKNOWN and skip_special):
                if not skip_special:
                    out += self.tokens[i].encode("utf-8")
            else:
                out += self.tokens[i].replace(SPACE, " ").encode("utf-8")
        return bytes(out)

    def decode(self, ids: Iterable[int], skip_special: bool = True) -> str:
        return self.decode_bytes(ids, skip_special).decode("utf-8", errors="replace")


def complete_utf8(b: bytes) -> str:
    """The longest prefix of `b` that does not end inside a UTF-8 sequence,
    decoded (for streaming text one token at a time)."""
    n = len(b)
    for back in range(1, min(4, n) + 1):
        c = b[n - back]
        if c & 0xC0 == 0x80:
            continue            # continuation byte: keep looking for the lead byte
        need = 1 if c < 0x80 else 2 if c >> 5 == 0x6 else 3 if c >> 4 == 0xE else 4 if c >> 3 == 0x1E else 1
        if back < need:
            n -= back           # the last sequence is incomplete
        break
    return b[:n].decode("utf-8", errors="replace")


def synthetic_vocab(vocab: int) -> Tuple[List[str], List[float], List[int]]:
    """A deterministic SentencePiece vocabulary of `vocab` entries for the
    synthetic models: control tokens (<pad> <eos> <bos> <unk>
    <start_of_turn> <end_of_turn>), the 256 byte tokens, "▁" and printable
    ASCII characters, word pieces built from a fixed word list (every prefix,
    with and without "▁"; longer pieces score higher), then unused fillers."""
    specials = [("<pad>", T_CONTROL), ("<eos>", T_CONTROL), ("<bos>", T_CONTROL), ("<unk>", T_UNKNOWN),
                ("<start_of_turn>", T_CONTROL), ("<end_of_turn>", T_CONTROL)]
    toks = [s for s, _ in specials]
    types = [t for _, t in specials]
    scores = [0.0] * len(toks)
    for b in range(256):
        toks.append(f"<0x{b:02X}>")
        types.append(T_BYTE)
        scores.append(0.0)
    seen = set(toks)

    def add(piece: str, score: float):
        if piece not in seen and len(toks) < vocab:
            seen.add(piece)
            toks.append(piece)
            types.append(T_NORMAL)
            scores.append(score)

    add(SPACE, -1.0)
    for c in range(0x21, 0x7F):
        add(chr(c), -2.0)
    words = ("the and of to in is that for it with as was on be at by this had not are but from or have an they "
             "which one you were her all she there would their we him been has when who will more no if out so "
             "said what up its about into than them can only other new some could time these two may then do "
             "first any my now such like our over man me even most made after also did many before must through "
             "back years where much your way well down should because each just those people how too little state "
             "good very make world still own see men work long get here between both life being under never day "
             "same another know while last might us great old year off come since against go came right used take "
             "three hello model user token chonk gemma answer question please thank").split()
    for w in words:
        for n in range(2, len(w) + 1):
            add(SPACE + w[:n - 1], -3.0 + 0.1 * n)
            add(w[:n], -3.5 + 0.1 * n)
        add(SPACE + w, -2.0 + 0.1 * len(w))
    i = 0
    while len(toks) < vocab:
        toks.append(f"<unused{i}>")
        types.append(T_UNUSED)
        scores.append(0.0)
        i += 1
    if len(toks) > vocab:
        raise ValueError(f"synthetic vocabulary needs at least {len(toks)} entries, got {vocab}")
    return toks, scores, types
