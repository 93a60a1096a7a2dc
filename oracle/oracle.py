"""CPU ORACLE wrapper — test infrastructure only.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may use
this module, and only as the checker / the timed CPU baseline; the product
path (chonklm_b200) never imports it.

* builds oracle.c (plain C, -ffp-contract=off) into oracle/_build/liboracle.so
* reads a GGUF with gguf-py's GGUFReader (llama.cpp's own reader, an
  independent parser from the product's) and restates the manifest rules of
  buildGgufLlamaManifest (llama-wgsl-runtime.ts:326-425) to configure the
  C engine;
* restates sampleFromCandidateBuffer (sampling.ts:23-76) with the uniform draw
  taken from a Philox4x32-10 stream instead of Math.random (:70);
* restates generateLlamaWgsl (llama-wgsl-runtime.ts:242-314) minus text decode.

Parity status: dequant pinned against gguf-py 0.19.0; every runToken kernel
pinned against the reference's own WGSL text run by oracle/wgsl.py
(tests/test_wgsl_golden.py); the graph order and the sampler are restated
from the TypeScript (no JavaScript runtime here).
"""
from __future__ import annotations

import ctypes
import math
import os
import subprocess
import threading
from typing import Dict, List, Optional, Sequence

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
BUILD = os.path.join(HERE, "_build")
LIB_PATH = os.path.join(BUILD, "liboracle.so")
_lock = threading.Lock()
_lib = None

MODE_WGSL = 0
MODE_F64 = 1


def build(force: bool = False) -> str:
    src = os.path.join(HERE, "oracle.c")
    if not force and os.path.exists(LIB_PATH) and os.path.getmtime(LIB_PATH) >= os.path.getmtime(src):
        return LIB_PATH
    os.makedirs(BUILD, exist_ok=True)
    tmp = LIB_PATH + f".tmp{os.getpid()}"
    cmd = ["gcc", "-O2", "-fPIC", "-shared", "-std=c11", "-ffp-contract=off", "-fno-fast-math", "-fopenmp",
           "-o", tmp, src, "-lm"]
    subprocess.check_call(cmd)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


def lib():
    global _lib
    with _lock:
        if _lib is None:
            L = ctypes.CDLL(build())
            P = ctypes.c_void_p
            I = ctypes.c_int
            F = ctypes.c_float
            U = ctypes.c_uint32
            L.or_dequant.argtypes = [I, P, I, I, P]
            L.or_matvec.argtypes = [I, P, I, I, P, P, I]
            L.or_embedding.argtypes = [I, P, I, U, F, P]
            L.or_row_bytes.argtypes = [I, I]
            L.or_row_bytes.restype = ctypes.c_size_t
            L.or_create.argtypes = [P]
            L.or_create.restype = P
            L.or_set_embedding.argtypes = [P, I, P]
            L.or_set_lm_head.argtypes = [P, I, P]
            L.or_set_final_norm.argtypes = [P, P]
            L.or_set_layer_weight.argtypes = [P, I, I, I, I, I, P]
            L.or_set_layer_norm.argtypes = [P, I, I, P]
            L.or_set_layer_rope.argtypes = [P, I, I, I]
            L.or_reset.argtypes = [P]
            L.or_position.argtypes = [P]
            L.or_set_position.argtypes = [P, I]
            L.or_run_token.argtypes = [P, U, I, P, I, U]
            L.or_run_token.restype = ctypes.c_int64
            for fn in ("or_logits", "or_hidden", "or_cand_val", "or_cand_idx"):
                getattr(L, fn).argtypes = [P]
                getattr(L, fn).restype = P
            L.or_kcache.argtypes = [P, I]
            L.or_kcache.restype = P
            L.or_vcache.argtypes = [P, I]
            L.or_vcache.restype = P
            L.or_destroy.argtypes = [P]
            L.or_rms_norm.argtypes = [P, P, P, I, F]
            L.or_add_rms_norm.argtypes = [P, P, P, P, I, F]
            L.or_rope_store.argtypes = [P, P, P, P, P, I, I, I, I, I, U, I]
            L.or_qk_norm_rope_store.argtypes = [P, P, P, P, P, P, P, P, I, I, I, I, I, U, F, I]
            L.or_attention.argtypes = [P, P, P, P, P, I, I, I, I, I, I, F, I]
            L.or_silu_mul.argtypes = [P, P, P, I]
            L.or_gelu_tanh_mul.argtypes = [P, P, P, I]
            L.or_add.argtypes = [P, P, I, I]
            L.or_argmax_stage1.argtypes = [P, I, P, I, U, P, P]
            L.or_argmax_stage2.argtypes = [P, P, I]
            L.or_argmax_stage2.restype = U
            _lib = L
    return _lib


def _ptr(a: np.ndarray) -> int:
    return a.ctypes.data


def row_bytes(ggml_type: int, k: int) -> int:
    return int(lib().or_row_bytes(ggml_type, k))


def dequant(ggml_type: int, data: np.ndarray, k: int, n: int) -> np.ndarray:
    data = np.ascontiguousarray(data, dtype=np.uint8)
    assert data.size >= row_bytes(ggml_type, k) * n
    out = np.empty((n, k), dtype=np.float32)
    lib().or_dequant(ggml_type, _ptr(data), k, n, _ptr(out))
    return out


def matvec(ggml_type: int, data: np.ndarray, k: int, n: int, x: np.ndarray, mode: int = MODE_WGSL) -> np.ndarray:
    data = np.ascontiguousarray(data, dtype=np.uint8)
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty(n, dtype=np.float32)
    lib().or_matvec(ggml_type, _ptr(data), k, n, _ptr(x), _ptr(y), mode)
    return y


def argmax_candidates(logits: np.ndarray, penalty_ids: Sequence[int] = (), penalty: float = 1.0):
    """ARGMAX_STAGE1 + STAGE2 with the host-side penalty plumbing of
    LlamaWgslEngine.argmax (llama-wgsl-runtime.ts:1647-1677)."""
    logits = np.ascontiguousarray(logits, dtype=np.float32)
    vocab = logits.size
    groups = (vocab + 255) // 256
    apply = penalty > 1 and len(penalty_ids) > 0
    ids = np.asarray(list(penalty_ids), dtype=np.uint32) if apply else np.zeros(1, dtype=np.uint32)
    cv = np.empty(groups, dtype=np.float32)
    ci = np.empty(groups, dtype=np.uint32)
    lib().or_argmax_stage1(_ptr(logits), vocab, _ptr(ids), len(penalty_ids) if apply else 0,
                           int(math.floor(penalty * 1000 + 0.5)), _ptr(cv), _ptr(ci))
    best = int(lib().or_argmax_stage2(_ptr(cv), _ptr(ci), groups))
    return cv, ci, best


# --- Philox4x32-10 (Salmon et al., SC'11) -------------------------------------
_M0, _M1 = 0xD2511F53, 0xCD9E8D57
_W0, _W1 = 0x9E3779B9, 0xBB67AE85


def philox4x32(counter: Sequence[int], key: Sequence[int], rounds: int = 10) -> List[int]:
    c0, c1, c2, c3 = [int(v) & 0xFFFFFFFF for v in counter]
    k0, k1 = [int(v) & 0xFFFFFFFF for v in key]
    for _ in range(rounds):
        p0 = _M0 * c0
        p1 = _M1 * c2
        hi0, lo0 = p0 >> 32, p0 & 0xFFFFFFFF
        hi1, lo1 = p1 >> 32, p1 & 0xFFFFFFFF
        c0, c1, c2, c3 = (hi1 ^ c1 ^ k0) & 0xFFFFFFFF, lo1, (hi0 ^ c3 ^ k1) & 0xFFFFFFFF, lo0
        k0 = (k0 + _W0) & 0xFFFFFFFF
        k1 = (k1 + _W1) & 0xFFFFFFFF
    return [c0, c1, c2, c3]


def philox_uniform(seed: int, offset: int) -> float:
    """Uniform double in [0, 1) for draw number `offset` of stream `seed`:
    53 bits from the first two Philox words (key = seed, counter = offset)."""
    c = philox4x32([offset & 0xFFFFFFFF, (offset >> 32) & 0xFFFFFFFF, 0, 0],
                   [seed & 0xFFFFFFFF, (seed >> 32) & 0xFFFFFFFF])
    return ((c[0] >> 5) * 67108864.0 + (c[1] >> 6)) / 9007199254740992.0


def sample_from_candidates(cand_val: np.ndarray, cand_idx: np.ndarray, temperature: float = 0.0,
                           top_p: float = 1.0, top_k: int = 0, repetition_penalty: float = 1.0,
                           seen_ids: Sequence[int] = (), uniform: Optional[float] = None) -> int:
    """sampleFromCandidateBuffer (sampling.ts:23-76); `uniform` replaces Math.random()."""
    seen = set(int(i) for i in seen_ids)
    rp = max(repetition_penalty if repetition_penalty is not None else 1.0, 1e-6)
    cands = []
    for v, i in zip(cand_val.tolist(), cand_idx.tolist()):
        v = float(np.float32(v))
        if not math.isfinite(v) or i == 0xFFFFFFFF:
            continue
        if rp != 1 and i in seen:
            v = v / rp if v > 0 else v * rp
        cands.append((v, int(i)))
    cands.sort(key=lambda c: -c[0])                     # stable, like Array.prototype.sort
    k = max(0, int(math.floor(top_k))) if top_k is not None and math.isfinite(top_k) else 0
    limited = cands[:min(k, len(cands))] if k > 0 else cands
    if (temperature or 0) <= 0:
        return limited[0][1] if limited else (cands[0][1] if cands else 0)
    tp = min(max(top_p if top_p is not None else 1.0, 0.0), 1.0)
    max_val = limited[0][0] if limited else 0.0
    probs = [math.exp((v - max_val) / temperature) for v, _ in limited]
    total = 0.0
    for p in probs:
        total += p
    cutoff = len(limited)
    if tp < 1 and total > 0:
        cdf = 0.0
        for i, p in enumerate(probs):
            cdf += p / total
            if cdf >= tp:
                cutoff = i + 1
                break
    sample_total = 0.0
    for i in range(cutoff):
        sample_total += probs[i]
    r = (uniform if uniform is not None else np.random.random()) * sample_total
    for i in range(cutoff):
        r -= probs[i]
        if r <= 0:
            return limited[i][1]
    return limited[max(0, cutoff - 1)][1] if limited else 0


def sampler_probabilities(cand_val: np.ndarray, cand_idx: np.ndarray, temperature: float, top_p: float = 1.0,
                          top_k: int = 0) -> Dict[int, float]:
    """The probability sampleFromCandidateBuffer (sampling.ts:23-76) gives
    each id: the candidates it keeps after top-k and the top-p cutoff, with
    weight exp((v - max) / T) over their sum (no repetition penalty)."""
    cands = [(float(np.float32(v)), int(i)) for v, i in zip(cand_val.tolist(), cand_idx.tolist())
             if math.isfinite(float(v)) and i != 0xFFFFFFFF]
    cands.sort(key=lambda c: -c[0])
    k = max(0, int(math.floor(top_k))) if top_k else 0
    limited = cands[:min(k, len(cands))] if k > 0 else cands
    if not limited:
        return {}
    if temperature <= 0:
        return {limited[0][1]: 1.0}
    probs = [math.exp((v - limited[0][0]) / temperature) for v, _ in limited]
    total = sum(probs)
    cutoff = len(limited)
    tp = min(max(top_p, 0.0), 1.0)
    if tp < 1 and total > 0:
        cdf = 0.0
        for i, p in enumerate(probs):
            cdf += p / total
            if cdf >= tp:
                cutoff = i + 1
                break
    st = sum(probs[:cutoff])
    out: Dict[int, float] = {}
    for i in range(cutoff):
        out[limited[i][1]] = out.get(limited[i][1], 0.0) + probs[i] / st
    return out


def exact_candidates(logits: np.ndarray, top_k: int = 0, penalty_ids: Sequence[int] = (),
                     penalty: float = 1.0):
    """Candidate list of the engine's exact sampler (ck_set_sampler(h, 1)):
    the K largest stage-1 values over the whole vocabulary -- the logits with
    ARGMAX_STAGE1_WGSL's milli-fixed-point penalty on penalized ids
    (llama-wgsl-runtime.ts:1661, :3665-3690) -- K = top_k when 1..1023, else
    1024, ties to the lower id, NaN never before a number; returned in id
    order, as the reference's candidate buffer is ordered."""
    v = np.asarray(logits, dtype=np.float32).copy()
    if penalty > 1.0 and len(penalty_ids):
        pen = np.float32(math.floor(penalty * 1000.0 + 0.5) / 1000.0)
        ids = np.unique(np.asarray([i for i in penalty_ids if 0 <= i < v.size], dtype=np.int64))
        pv = v[ids]
        v[ids] = np.where(pv > 0, pv / pen, pv * pen).astype(np.float32)
    K = top_k if 0 < top_k < 1024 else 1024
    K = min(K, v.size)
    # order-preserving key: NaN lowest; sort by (key desc, id asc)
    bits = v.view(np.uint32).astype(np.uint64)
    key = np.where(bits & 0x80000000, (~bits) & 0xFFFFFFFF, bits | 0x80000000)
    key = np.where(np.isnan(v), 0, key)
    order = np.lexsort((np.arange(v.size), -key.astype(np.int64)))[:K]
    order.sort()
    return v[order], order.astype(np.uint32)


def sample_exact(logits: np.ndarray, temperature: float = 0.0, top_p: float = 1.0, top_k: int = 0,
                 repetition_penalty: float = 1.0, seen_ids: Sequence[int] = (), uniform: Optional[float] = None,
                 penalty_ids: Sequence[int] = ()) -> int:
    """The exact sampler: sampleFromCandidateBuffer (sampling.ts:23-76) on
    exact_candidates instead of the chunk maxima."""
    cv, ci = exact_candidates(logits, top_k, penalty_ids, repetition_penalty)
    return sample_from_candidates(cv, ci, temperature, top_p, top_k, repetition_penalty, seen_ids, uniform)


def needs_sampling_readback(temperature: float = 0.0, top_p: float = 1.0, top_k: int = 0) -> bool:
    """needsSamplingReadback (sampling.ts:9-16)."""
    k = max(0, int(math.floor(top_k))) if top_k is not None and math.isfinite(top_k) else 0
    return (temperature or 0) > 0 or (top_p if top_p is not None else 1) < 1 or k > 0


# --- model -------------------------------------------------------------------
class _Cfg(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int) for n in ("hidden", "intermediate", "vocab", "layers", "heads", "kv_heads",
                                            "head_dim", "context_length")] + \
               [(n, ctypes.c_float) for n in ("norm_eps", "qk_norm_eps", "embedding_scale", "attn_scale")] + \
               [(n, ctypes.c_int) for n in ("is_gemma3", "interleaved_rope", "qk_norm", "mode")]


def _kv_num(reader, key, fallback=None):
    f = reader.fields.get(key)
    if f is None:
        if fallback is None:
            raise KeyError(key)
        return fallback
    return f.parts[f.data[0]].tolist()[0]


def _kv_str(reader, key):
    f = reader.fields[key]
    return bytes(f.parts[f.data[0]]).decode("utf-8")


class OracleModel:
    """The C restatement of LlamaWgslEngine, configured from a GGUF file."""

    def __init__(self, path: str, vocab: Optional[int] = None, max_context: Optional[int] = None,
                 mode: int = MODE_WGSL, n_layers: Optional[int] = None):
        import gguf as ggufpy  # llama.cpp's reader (gguf-py), independent of chonklm_b200.gguf
        r = ggufpy.GGUFReader(path)
        self.reader = r
        arch = _kv_str(r, "general.architecture")
        if arch not in ("llama", "qwen3", "gemma3"):
            raise ValueError(f"oracle: unsupported architecture {arch}")
        self.arch = arch
        g = arch == "gemma3"
        t = {x.name: x for x in r.tensors}
        self.tensors = t
        hidden = int(_kv_num(r, f"{arch}.embedding_length"))
        heads = int(_kv_num(r, f"{arch}.attention.head_count"))
        layers = int(_kv_num(r, f"{arch}.block_count"))
        emb = t["token_embd.weight"]
        V = int(emb.shape[1]) if vocab is None else vocab
        ctx = int(_kv_num(r, f"{arch}.context_length", 1 << 30))
        if max_context is not None:
            ctx = min(ctx, max_context)
        eps = float(np.float32(_kv_num(r, f"{arch}.attention.layer_norm_rms_epsilon", 1e-5)))
        hd = int(_kv_num(r, f"{arch}.attention.key_length", hidden // heads))
        c = _Cfg()
        c.hidden = hidden
        c.intermediate = int(_kv_num(r, f"{arch}.feed_forward_length"))
        c.vocab = V
        c.layers = layers if n_layers is None else n_layers
        c.heads = heads
        c.kv_heads = int(_kv_num(r, f"{arch}.attention.head_count_kv"))
        c.head_dim = hd
        c.context_length = ctx
        c.norm_eps = eps
        c.qk_norm_eps = eps
        c.embedding_scale = float(np.float32(math.sqrt(hidden))) if g else 1.0
        c.attn_scale = float(np.float32(1.0 / math.sqrt(hd)))
        c.is_gemma3 = 1 if g else 0
        c.interleaved_rope = 1 if arch == "llama" else 0
        c.qk_norm = 1 if ("blk.0.attn_q_norm.weight" in t and "blk.0.attn_k_norm.weight" in t) else 0
        c.mode = mode
        self.cfg = c
        L = lib()
        self._h = L.or_create(ctypes.byref(c))
        self._keep: List[np.ndarray] = []

        def raw(name):
            a = np.ascontiguousarray(np.asarray(t[name].data).view(np.uint8).reshape(-1))
            self._keep.append(a)
            return a

        def f32(name):
            x = t[name]
            a = np.asarray(x.data)
            a = a.astype(np.float32).reshape(-1) if a.dtype != np.float32 else np.ascontiguousarray(a.reshape(-1))
            self._keep.append(a)
            return a

        L.or_set_embedding(self._h, int(emb.tensor_type), _ptr(raw("token_embd.weight")))
        head = "output.weight" if "output.weight" in t else "token_embd.weight"
        L.or_set_lm_head(self._h, int(t[head].tensor_type), _ptr(raw(head)))
        L.or_set_final_norm(self._h, _ptr(f32("output_norm.weight")))
        gtheta = _kv_num(r, "gemma3.rope.freq_base", 1000000) if g else 0
        window = int(_kv_num(r, "gemma3.attention.sliding_window", 0)) if g else 0
        base_theta = _kv_num(r, f"{arch}.rope.freq_base", 10000)
        slots = ["attn_q", "attn_k", "attn_v", "attn_output", "ffn_gate", "ffn_up", "ffn_down"]
        for i in range(c.layers):
            p = f"blk.{i}."
            for s, nm in enumerate(slots):
                x = t[p + nm + ".weight"]
                k, n = int(x.shape[0]), int(x.shape[1])
                L.or_set_layer_weight(self._h, i, s, int(x.tensor_type), k, n, _ptr(raw(p + nm + ".weight")))
            norms = ["attn_norm", "post_attention_norm" if g else "ffn_norm"]
            norms += ["ffn_norm", "post_ffw_norm"] if g else [None, None]
            norms += ["attn_q_norm", "attn_k_norm"]
            for s, nm in enumerate(norms):
                if nm is not None and p + nm + ".weight" in t:
                    L.or_set_layer_norm(self._h, i, s, _ptr(f32(p + nm + ".weight")))
            if g:
                th = gtheta if i % 6 == 5 else 10000
                win = 0 if i % 6 == 5 else window
            else:
                th, win = base_theta, 0
            L.or_set_layer_rope(self._h, i, int(math.floor(th + 0.5)), win)

    # engine surface (runToken / reset / position), llama-wgsl-runtime.ts:1011-1150
    def run_token(self, token: int, need_logits: bool = True, penalty_ids: Sequence[int] = (),
                  penalty: float = 1.0) -> int:
        apply = penalty > 1 and len(penalty_ids) > 0
        ids = list(penalty_ids)[-self.cfg.context_length:] if apply else []
        arr = np.asarray(ids if ids else [0], dtype=np.uint32)
        r = lib().or_run_token(self._h, int(token), 1 if need_logits else 0, _ptr(arr), len(ids),
                               int(math.floor(penalty * 1000 + 0.5)))
        if r < 0:
            raise RuntimeError(f"Llama WGSL context exhausted at {self.cfg.context_length} tokens")
        return int(r)

    def logits(self) -> np.ndarray:
        p = lib().or_logits(self._h)
        return np.ctypeslib.as_array(ctypes.cast(p, ctypes.POINTER(ctypes.c_float)), (self.cfg.vocab,)).copy()

    def hidden(self) -> np.ndarray:
        p = lib().or_hidden(self._h)
        return np.ctypeslib.as_array(ctypes.cast(p, ctypes.POINTER(ctypes.c_float)), (self.cfg.hidden,)).copy()

    def candidates(self):
        gs = (self.cfg.vocab + 255) // 256
        L = lib()
        v = np.ctypeslib.as_array(ctypes.cast(L.or_cand_val(self._h), ctypes.POINTER(ctypes.c_float)), (gs,)).copy()
        i = np.ctypeslib.as_array(ctypes.cast(L.or_cand_idx(self._h), ctypes.POINTER(ctypes.c_uint32)), (gs,)).copy()
        return v, i

    def kv_cache(self, layer: int):
        n = self.cfg.kv_heads * self.cfg.context_length * self.cfg.head_dim
        L = lib()
        k = np.ctypeslib.as_array(ctypes.cast(L.or_kcache(self._h, layer), ctypes.POINTER(ctypes.c_float)), (n,))
        v = np.ctypeslib.as_array(ctypes.cast(L.or_vcache(self._h, layer), ctypes.POINTER(ctypes.c_float)), (n,))
        shape = (self.cfg.kv_heads, self.cfg.context_length, self.cfg.head_dim)
        return k.reshape(shape).copy(), v.reshape(shape).copy()

    def reset(self) -> None:
        lib().or_reset(self._h)

    @property
    def position(self) -> int:
        return int(lib().or_position(self._h))

    def set_position(self, pos: int) -> None:
        lib().or_set_position(self._h, pos)

    def close(self) -> None:
        if getattr(self, "_h", None):
            lib().or_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def generate(model: OracleModel, prompt_ids: Sequence[int], max_new_tokens: int = 128, eos_ids=(),
             temperature: float = 0.0, top_p: float = 1.0, top_k: int = 0, repetition_penalty: float = 1.0,
             seed: int = 0, max_context: Optional[int] = None) -> List[int]:
    """generateLlamaWgsl (llama-wgsl-runtime.ts:242-314) from a reset engine;
    sampling draws use philox_uniform(seed, i) for the i-th sampled token."""
    ctx = model.cfg.context_length if max_context is None else max_context
    mx = min(max_new_tokens, ctx - len(prompt_ids))
    eos = set(eos_ids)
    sampling = needs_sampling_readback(temperature, top_p, top_k)
    draws = [0]

    def step(tok: int, penal: List[int]) -> int:
        best = model.run_token(tok, True, penal, repetition_penalty)
        if not sampling:
            return best
        cv, ci = model.candidates()
        u = philox_uniform(seed, draws[0])
        draws[0] += 1
        return sample_from_candidates(cv, ci, temperature, top_p, top_k, repetition_penalty, penal, u)

    model.reset()
    next_id = 0
    prompt = list(prompt_ids)
    for i, tok in enumerate(prompt):
        if i == len(prompt) - 1:
            next_id = step(tok, prompt[:i + 1])
        else:
            model.run_token(tok, False)
    generated: List[int] = []
    for s in range(mx):
        generated.append(next_id)
        if next_id in eos or s + 1 >= mx:
            break
        next_id = step(next_id, prompt + generated)
    return generated
