"""ctypes binding of libchonk_b200.so (the C ABI in include/chonk_b200.h).

There is no CPU fallback: if the library cannot be loaded, or the CUDA call
fails, every entry point raises.  The library is built in-tree by
`chonklm_b200.build` (nvcc, sm_100a).
"""
from __future__ import annotations

import ctypes
import os
import threading
from typing import List, Optional, Sequence, Tuple

import numpy as np

from . import build as _build

CK_OK = 0
CK_EINVAL = -1
CK_ECUDA = -2
CK_ESTATE = -3
CK_ECONTEXT = -4
CK_EDEVICE = -5
CK_ENOMEM = -6

CK_ARCH_LLAMA = 0
CK_ARCH_GEMMA3 = 1
CK_KV_F16 = 0
CK_KV_F32 = 1
CK_MAX_LAYERS = 128

MODE_MEGAKERNEL = 0
MODE_GRAPH = 1
MODE_STREAM = 2


class CkError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"{msg} (ck code {code})")
        self.code = code


class ContextExhausted(CkError):
    pass


class ck_model_cfg(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int32) for n in ("hidden", "intermediate", "vocab", "layers", "heads", "kv_heads",
                                              "head_dim", "context_length")] + \
               [("norm_eps", ctypes.c_float), ("qk_norm_eps", ctypes.c_float), ("embedding_scale", ctypes.c_float)] + \
               [(n, ctypes.c_int32) for n in ("arch", "rope_interleaved", "qk_norm", "kv_dtype")] + \
               [("layer_rope_theta", ctypes.c_uint32 * CK_MAX_LAYERS),
                ("layer_window", ctypes.c_uint32 * CK_MAX_LAYERS)]


class ck_sampling(ctypes.Structure):
    _fields_ = [("temperature", ctypes.c_double), ("top_p", ctypes.c_double), ("top_k", ctypes.c_int32),
                ("repetition_penalty", ctypes.c_double), ("penalized_ids", ctypes.POINTER(ctypes.c_uint32)),
                ("n_penalized", ctypes.c_int32), ("philox_seed", ctypes.c_uint64),
                ("philox_offset", ctypes.c_uint64)]


_lock = threading.Lock()
_lib = None


def lib():
    """Load (building first if sources changed) libchonk_b200.so."""
    global _lib
    with _lock:
        if _lib is None:
            path = _build.LIB
            if _build.needs_build():
                try:
                    path = _build.build()
                except Exception as e:  # no nvcc / compile error: fail loudly
                    if not os.path.exists(path):
                        raise RuntimeError(f"libchonk_b200.so is missing and could not be built: {e}") from e
            L = ctypes.CDLL(path)
            P, I, U, S, D = ctypes.c_void_p, ctypes.c_int, ctypes.c_uint32, ctypes.c_size_t, ctypes.c_double
            pp = ctypes.POINTER
            L.ck_create.argtypes = [pp(ck_model_cfg), I, pp(P)]
            L.ck_upload_tensor.argtypes = [P, ctypes.c_char_p, I, pp(ctypes.c_int64), I, P, S]
            L.ck_finalize.argtypes = [P]
            L.ck_destroy.argtypes = [P]
            L.ck_run_token.argtypes = [P, U, I, pp(ck_sampling), pp(U)]
            L.ck_prefill.argtypes = [P, pp(U), I, I, pp(ck_sampling), pp(U)]
            L.ck_decode.argtypes = [P, U, I, pp(ck_sampling), pp(U), I, pp(U), pp(I)]
            L.ck_get_logits.argtypes = [P, P, S]
            L.ck_get_candidates.argtypes = [P, P, P, S]
            L.ck_reset.argtypes = [P]
            L.ck_position.argtypes = [P, pp(I)]
            L.ck_truncate.argtypes = [P, I]
            L.ck_last_error.argtypes = [P]
            L.ck_last_error.restype = ctypes.c_char_p
            L.ck_global_error.argtypes = []
            L.ck_global_error.restype = ctypes.c_char_p
            L.ck_set_stream.argtypes = [P, P]
            L.ck_set_mode.argtypes = [P, I]
            L.ck_set_sampler.argtypes = [P, I]
            L.ck_set_prefill_gemm.argtypes = [P, I, I]
            L.ck_enqueue_decode_steps.argtypes = [P, I]
            L.ck_enqueue_decode_steps_sampled.argtypes = [P, I, pp(ck_sampling)]
            L.ck_sync.argtypes = [P]
            L.ck_step_bytes.argtypes = [P, pp(D), pp(D)]
            L.ck_dequant.argtypes = [I, P, S, I, I, P, I]
            L.ck_matvec.argtypes = [I, P, S, I, I, P, P, I]
            L.ck_bench_matvec.argtypes = [I, P, S, I, I, I, pp(D), I]
            L.ck_abi_info.argtypes = [pp(I), pp(I)]
            L.ck_io_bytes.argtypes = [P, pp(ctypes.c_uint64), pp(ctypes.c_uint64)]
            L.ck_matvec_noalloc.argtypes = [I, P, S, I, I, P, P, P]
            L.ck_trace.argtypes = [P, I]
            L.ck_trace_read.argtypes = [P, P, S]
            L.ck_matmul.argtypes = [I, P, S, I, I, P, I, P, I]
            L.ck_batch_create.argtypes = [P, I, I, pp(P)]
            L.ck_batch_add_seq.argtypes = [P, pp(U), I, I, pp(U), I, pp(I)]
            L.ck_batch_step.argtypes = [P, pp(I)]
            L.ck_batch_collect.argtypes = [P, I, pp(U), I, pp(I), pp(I)]
            L.ck_batch_stats.argtypes = [P, pp(ctypes.c_uint64), pp(ctypes.c_uint64), pp(ctypes.c_uint64)]
            L.ck_batch_last_error.argtypes = [P]
            L.ck_batch_last_error.restype = ctypes.c_char_p
            L.ck_batch_destroy.argtypes = [P]
            _lib = L
    return _lib


def _check(rc: int, h=None) -> None:
    if rc == CK_OK:
        return
    L = lib()
    msg = (L.ck_last_error(h) if h else L.ck_global_error()) or b""
    msg = msg.decode("utf-8", "replace")
    if rc == CK_ECONTEXT:
        raise ContextExhausted(rc, msg)
    raise CkError(rc, msg)


def _u32p(a: np.ndarray):
    return a.ctypes.data_as(ctypes.POINTER(ctypes.c_uint32))


def make_sampling(temperature: float = 0.0, top_p: float = 1.0, top_k: int = 0, repetition_penalty: float = 1.0,
                  seed: int = 0, offset: int = 0, penalized_ids: Optional[Sequence[int]] = None):
    s = ck_sampling()
    s.temperature = float(temperature or 0.0)
    s.top_p = float(1.0 if top_p is None else top_p)
    s.top_k = int(top_k or 0)
    s.repetition_penalty = float(1.0 if repetition_penalty is None else repetition_penalty)
    s.philox_seed = int(seed) & (2 ** 64 - 1)
    s.philox_offset = int(offset)
    keep = None
    if penalized_ids is not None:
        keep = np.ascontiguousarray(np.asarray(list(penalized_ids), dtype=np.uint32))
        s.penalized_ids = _u32p(keep) if keep.size else ctypes.cast(ctypes.c_void_p(0), ctypes.POINTER(ctypes.c_uint32))
        s.n_penalized = int(keep.size)
    return s, keep


class Engine:
    """One device engine (LlamaWgslEngine's device side)."""

    def __init__(self, cfg: ck_model_cfg, device: int = 0):
        self._L = lib()
        h = ctypes.c_void_p()
        _check(self._L.ck_create(ctypes.byref(cfg), device, ctypes.byref(h)))
        self.h = h
        self.cfg = cfg

    def upload(self, name: str, ggml_type: int, shape: Sequence[int], data: bytes) -> None:
        shp = (ctypes.c_int64 * len(shape))(*shape)
        buf = np.frombuffer(data, dtype=np.uint8) if not isinstance(data, np.ndarray) else data
        buf = np.ascontiguousarray(buf)
        _check(self._L.ck_upload_tensor(self.h, name.encode(), ggml_type, shp, len(shape), buf.ctypes.data,
                                        buf.nbytes), self.h)

    def finalize(self) -> None:
        _check(self._L.ck_finalize(self.h), self.h)

    def run_token(self, token: int, need_logits: bool, sampling=None) -> int:
        out = ctypes.c_uint32(0)
        _check(self._L.ck_run_token(self.h, int(token), 1 if need_logits else 0,
                                    ctypes.byref(sampling) if sampling is not None else None, ctypes.byref(out)),
               self.h)
        return int(out.value)

    def prefill(self, tokens: Sequence[int], need_logits_last: bool = True, sampling=None) -> int:
        arr = np.ascontiguousarray(np.asarray(list(tokens), dtype=np.uint32))
        out = ctypes.c_uint32(0)
        _check(self._L.ck_prefill(self.h, _u32p(arr), int(arr.size), 1 if need_logits_last else 0,
                                  ctypes.byref(sampling) if sampling is not None else None, ctypes.byref(out)),
               self.h)
        return int(out.value)

    def decode(self, first: int, max_new: int, sampling=None, eos_ids: Sequence[int] = ()) -> list:
        eos = np.ascontiguousarray(np.asarray(list(eos_ids) or [0], dtype=np.uint32))
        out = np.zeros(max(1, max_new), dtype=np.uint32)
        n = ctypes.c_int(0)
        _check(self._L.ck_decode(self.h, int(first), int(max_new),
                                 ctypes.byref(sampling) if sampling is not None else None, _u32p(eos),
                                 len(eos_ids), _u32p(out), ctypes.byref(n)), self.h)
        return out[:n.value].tolist()

    def logits(self) -> np.ndarray:
        out = np.empty(self.cfg.vocab, dtype=np.float32)
        _check(self._L.ck_get_logits(self.h, out.ctypes.data, out.size), self.h)
        return out

    def candidates(self) -> Tuple[np.ndarray, np.ndarray]:
        g = (self.cfg.vocab + 255) // 256
        v = np.empty(g, dtype=np.float32)
        i = np.empty(g, dtype=np.uint32)
        _check(self._L.ck_get_candidates(self.h, v.ctypes.data, i.ctypes.data, g), self.h)
        return v, i

    def reset(self) -> None:
        _check(self._L.ck_reset(self.h), self.h)

    @property
    def position(self) -> int:
        p = ctypes.c_int(0)
        _check(self._L.ck_position(self.h, ctypes.byref(p)), self.h)
        return p.value

    def truncate(self, pos: int) -> None:
        _check(self._L.ck_truncate(self.h, int(pos)), self.h)

    def set_stream(self, stream_handle: int) -> None:
        _check(self._L.ck_set_stream(self.h, ctypes.c_void_p(stream_handle)), self.h)

    def set_sampler(self, exact: bool) -> None:
        """ck_set_sampler: the reference's chunk-maxima candidates (False) or
        the exact top-K over the whole vocabulary (True)."""
        _check(self._L.ck_set_sampler(self.h, 1 if exact else 0), self.h)

    def set_mode(self, mode: int) -> None:
        _check(self._L.ck_set_mode(self.h, int(mode)), self.h)

    def set_prefill_gemm(self, min_tokens: int, chunk: int = 0) -> None:
        """Prompts of more than min_tokens ids (0: never) prefill on the
        tensor cores, chunk ids per pass (0: the largest)."""
        _check(self._L.ck_set_prefill_gemm(self.h, int(min_tokens), int(chunk)), self.h)

    def enqueue_decode_steps(self, n: int, sampling=None) -> None:
        """n chained decode steps, not synchronised: greedy, or sampling with
        `sampling` (a ck_sampling from make_sampling)."""
        if sampling is None:
            _check(self._L.ck_enqueue_decode_steps(self.h, int(n)), self.h)
        else:
            _check(self._L.ck_enqueue_decode_steps_sampled(self.h, int(n), ctypes.byref(sampling)), self.h)

    def sync(self) -> None:
        _check(self._L.ck_sync(self.h), self.h)

    def step_bytes(self) -> Tuple[float, float]:
        w, k = ctypes.c_double(), ctypes.c_double()
        _check(self._L.ck_step_bytes(self.h, ctypes.byref(w), ctypes.byref(k)), self.h)
        return w.value, k.value

    def trace(self, enable: bool) -> None:
        _check(self._L.ck_trace(self.h, 1 if enable else 0), self.h)

    def trace_read(self, n: int = 16384) -> np.ndarray:
        out = np.zeros(n, dtype=np.uint64)
        _check(self._L.ck_trace_read(self.h, out.ctypes.data, n), self.h)
        return out

    def io_bytes(self) -> Tuple[int, int]:
        a, b = ctypes.c_uint64(0), ctypes.c_uint64(0)
        _check(self._L.ck_io_bytes(self.h, ctypes.byref(a), ctypes.byref(b)), self.h)
        return a.value, b.value

    def close(self) -> None:
        if getattr(self, "h", None):
            self._L.ck_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def _check_batch(rc: int, b) -> None:
    if rc == CK_OK:
        return
    msg = (lib().ck_batch_last_error(b) or b"").decode("utf-8", "replace")
    raise CkError(rc, msg)


class Batch:
    """Batched decode over an Engine's weights (ck_batch_*): sequences are
    added, stepped together one position per step, and collected."""

    def __init__(self, engine: "Engine", max_seqs: int, kv_blocks: int = 0):
        self._L = lib()
        self.engine = engine   # keeps the weights alive
        b = ctypes.c_void_p()
        _check(self._L.ck_batch_create(engine.h, int(max_seqs), int(kv_blocks), ctypes.byref(b)), engine.h)
        self.b = b

    def add(self, prompt: Sequence[int], max_new: int, eos_ids: Sequence[int] = ()) -> int:
        arr = np.ascontiguousarray(np.asarray(prompt, dtype=np.uint32))
        eos = np.ascontiguousarray(np.asarray(list(eos_ids) or [0], dtype=np.uint32))
        sid = ctypes.c_int(0)
        _check_batch(self._L.ck_batch_add_seq(self.b, _u32p(arr), int(arr.size), int(max_new), _u32p(eos),
                                              len(eos_ids), ctypes.byref(sid)), self.b)
        return sid.value

    def step(self) -> int:
        n = ctypes.c_int(0)
        _check_batch(self._L.ck_batch_step(self.b, ctypes.byref(n)), self.b)
        return n.value

    def collect(self, seq_id: int, cap: int = 1 << 16) -> Tuple[List[int], bool]:
        """Ids so far and whether the sequence finished (a finished result is
        released by this call)."""
        out = np.zeros(max(cap, 1), dtype=np.uint32)
        n, done = ctypes.c_int(0), ctypes.c_int(0)
        _check_batch(self._L.ck_batch_collect(self.b, int(seq_id), _u32p(out), out.size, ctypes.byref(n),
                                              ctypes.byref(done)), self.b)
        return out[:min(n.value, out.size)].tolist(), bool(done.value)

    def stats(self) -> Tuple[int, int, int]:
        a, b, c = ctypes.c_uint64(0), ctypes.c_uint64(0), ctypes.c_uint64(0)
        _check_batch(self._L.ck_batch_stats(self.b, ctypes.byref(a), ctypes.byref(b), ctypes.byref(c)), self.b)
        return a.value, b.value, c.value

    def close(self) -> None:
        if getattr(self, "b", None):
            self._L.ck_batch_destroy(self.b)
            self.b = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def dequant(ggml_type: int, data: bytes, k: int, n: int, device: int = 0) -> np.ndarray:
    buf = np.ascontiguousarray(np.frombuffer(data, dtype=np.uint8))
    out = np.empty((n, k), dtype=np.float32)
    _check(lib().ck_dequant(ggml_type, buf.ctypes.data, buf.nbytes, k, n, out.ctypes.data, device))
    return out


def matvec(ggml_type: int, data: bytes, k: int, n: int, x: np.ndarray, device: int = 0) -> np.ndarray:
    buf = np.ascontiguousarray(np.frombuffer(data, dtype=np.uint8))
    xx = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty(n, dtype=np.float32)
    _check(lib().ck_matvec(ggml_type, buf.ctypes.data, buf.nbytes, k, n, xx.ctypes.data, y.ctypes.data, device))
    return y


def matmul(ggml_type: int, data: bytes, k: int, n: int, x: np.ndarray, device: int = 0) -> np.ndarray:
    """Y = X W^T for T rows of x (the batched path's tensor-core GEMM)."""
    buf = np.ascontiguousarray(np.frombuffer(data, dtype=np.uint8))
    xx = np.ascontiguousarray(np.asarray(x, dtype=np.float32))
    T = xx.shape[0]
    y = np.empty((T, n), dtype=np.float32)
    _check(lib().ck_matmul(ggml_type, buf.ctypes.data, buf.nbytes, k, n, xx.ctypes.data, T, y.ctypes.data, device))
    return y


def matvec_noalloc(ggml_type: int, w_dev: int, nbytes: int, k: int, n: int, x_dev: int, y_dev: int,
                   stream: int = 0) -> None:
    """ck_matvec_noalloc on caller-owned device buffers (raw integer device
    addresses): for callers that cannot allocate device memory themselves."""
    _check(lib().ck_matvec_noalloc(ggml_type, ctypes.c_void_p(w_dev), nbytes, k, n, ctypes.c_void_p(x_dev),
                                   ctypes.c_void_p(y_dev), ctypes.c_void_p(stream)))


def layout_row_bytes(ggml_type: int, k: int) -> int:
    """Bytes of one row of the engine's device layout (GGUF blocks re-laid
    into 16-byte units; equal to the GGUF row up to 16-byte padding)."""
    nb = k // (256 if ggml_type in (12, 14) else 32)
    r16 = lambda v: (v + 15) & ~15
    if ggml_type == 12:                       # Q4_K
        return 16 * nb + 128 * nb
    if ggml_type == 14:                       # Q6_K
        return 16 * nb + r16(2 * nb) + 128 * nb + 64 * nb
    if ggml_type == 8:                        # Q8_0
        return r16(2 * nb) + 32 * nb
    if ggml_type == 6:                        # Q5_0
        return r16(2 * nb) + r16(4 * nb) + 16 * nb
    if ggml_type == 7:                        # Q5_1
        return r16(2 * nb) + r16(2 * nb) + r16(4 * nb) + 16 * nb
    raise ValueError(f"type {ggml_type}")


def bench_matvec(ggml_type: int, data: bytes, k: int, n: int, reps: int = 200, device: int = 0) -> float:
    buf = np.ascontiguousarray(np.frombuffer(data, dtype=np.uint8))
    us = ctypes.c_double(0)
    _check(lib().ck_bench_matvec(ggml_type, buf.ctypes.data, buf.nbytes, k, n, reps, ctypes.byref(us), device))
    return us.value


def abi_info() -> Tuple[int, int]:
    a, b = ctypes.c_int(0), ctypes.c_int(0)
    lib().ck_abi_info(ctypes.byref(a), ctypes.byref(b))
    return a.value, b.value
