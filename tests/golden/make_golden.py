"""Generate the committed golden fixtures in this directory.

  dequant_golden.npz  for each block type: raw GGUF block bytes and the fp32
                      weights gguf-py 0.19.0 (llama.cpp's Python reader of the
                      block formats) decodes them to.  gguf-py's numpy decode
                      uses the same fp32 operation order as the reference's
                      WGSL dequantizers, so these vectors pin the oracle's
                      dequant bit for bit.  Blocks: seeded quantized normals,
                      seeded normals scaled so fp16 d/dmin are subnormal, and
                      hand-built known-answer blocks (fixed scales, every
                      6-bit scale/min packing position, every nibble value).
  tiny_logits.npz     oracle logits of the three tiny synthetic models on a
                      fixed token sequence (regression guard for the oracle).

Run from the repository root:  python tests/golden/make_golden.py
"""
import os
import struct
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

import torch  # noqa: E402

from chonklm_b200.gguf import GGML_TYPE  # noqa: E402
from chonklm_b200.quant import quantize  # noqa: E402

TYPES = {"Q4_K": GGML_TYPE.Q4_K, "Q6_K": GGML_TYPE.Q6_K, "Q8_0": GGML_TYPE.Q8_0, "Q5_0": GGML_TYPE.Q5_0,
         "Q5_1": GGML_TYPE.Q5_1}
ROW = {"Q4_K": 256, "Q6_K": 256, "Q8_0": 32, "Q5_0": 32, "Q5_1": 32}


def h(v: float) -> bytes:
    return np.float16(v).tobytes()


def kat_blocks(name: str) -> bytes:
    """Hand-built blocks whose decode is easy to state."""
    out = b""
    if name == "Q4_K":
        for variant in range(4):
            d, dmin = [(1.0, 0.5), (0.25, 2.0), (6.0e-5, 3.0e-6), (-0.5, 0.125)][variant]
            sc = [(variant * 7 + 9 * j) % 64 for j in range(8)]
            mn = [(variant * 5 + 13 * j + 1) % 64 for j in range(8)]
            s = bytearray(12)
            for j in range(4):
                s[j] = sc[j] & 63
                s[j + 4] = mn[j] & 63
            for j in range(4, 8):
                s[j + 4] = (sc[j] & 15) | ((mn[j] & 15) << 4)
                s[j - 4] |= (sc[j] >> 4) << 6
                s[j] |= (mn[j] >> 4) << 6
            qs = bytes(((i + variant) % 16) | (((i * 3 + variant) % 16) << 4) for i in range(128))
            out += h(d) + h(dmin) + bytes(s) + qs
    elif name == "Q6_K":
        for variant in range(4):
            ql = bytes(((i * 5 + variant) % 256) for i in range(128))
            qh = bytes(((i * 11 + 3 * variant) % 256) for i in range(64))
            sc = bytes(((j * 17 + variant * 31) % 256) for j in range(16))   # int8, both signs
            d = [1.0, 0.03125, 5.0e-6, -2.0][variant]
            out += ql + qh + sc + h(d)
    elif name == "Q8_0":
        for variant in range(4):
            d = [1.0, 0.0078125, 1.0e-6, -3.5][variant]
            out += h(d) + bytes(((i * 37 + variant * 101) % 256) for i in range(32))
    elif name == "Q5_0":
        for variant in range(4):
            d = [1.0, 0.0625, 2.0e-6, -0.75][variant]
            qh = [0xFFFFFFFF, 0x00000000, 0xA5A5A5A5, 0x12345678][variant]
            out += h(d) + struct.pack("<I", qh) + bytes(((i * 7 + variant) % 256) for i in range(16))
    elif name == "Q5_1":
        for variant in range(4):
            d, m = [(1.0, -8.0), (0.0625, 0.5), (2.0e-6, -1.0e-6), (-0.75, 3.0)][variant]
            qh = [0xFFFFFFFF, 0x00000000, 0x5A5A5A5A, 0x87654321][variant]
            out += h(d) + h(m) + struct.pack("<I", qh) + bytes(((i * 9 + variant) % 256) for i in range(16))
    return out


def main():
    import gguf
    from gguf import quants
    arrays = {}
    for name, t in TYPES.items():
        k = ROW[name]
        g = torch.Generator().manual_seed(100 + t)
        normal = quantize(torch.randn(6, k, generator=g) * 0.02, t)
        sub = quantize(torch.randn(2, k, generator=g) * 2e-6, t)
        raw = normal + sub + kat_blocks(name)
        bb = {"Q4_K": 144, "Q6_K": 210, "Q8_0": 34, "Q5_0": 22, "Q5_1": 24}[name]
        blocks = np.frombuffer(raw, dtype=np.uint8).reshape(-1, bb)
        deq = quants.dequantize(blocks, getattr(gguf.GGMLQuantizationType, name)).astype(np.float32)
        arrays[f"{name}_raw"] = blocks.reshape(-1)
        arrays[f"{name}_deq"] = deq.reshape(-1)
        arrays[f"{name}_k"] = np.array([k], dtype=np.int64)
    np.savez_compressed(os.path.join(HERE, "dequant_golden.npz"), **arrays)

    from chonklm_b200.synth import tiny_spec, write_synthetic_gguf
    from oracle import oracle
    import tempfile
    out = {}
    with tempfile.TemporaryDirectory() as d:
        for arch in ("llama", "qwen3", "gemma3"):
            p = os.path.join(d, f"{arch}.gguf")
            write_synthetic_gguf(tiny_spec(arch), p, seed=0, device="cpu")
            m = oracle.OracleModel(p, max_context=64)
            toks = [3, 141, 59, 265, 358, 979, 323, 846]
            lg = []
            ids = []
            for t in toks:
                ids.append(m.run_token(t, True))
                lg.append(m.logits())
            out[f"{arch}_tokens"] = np.array(toks, dtype=np.int64)
            out[f"{arch}_logits"] = np.stack(lg).astype(np.float32)
            out[f"{arch}_ids"] = np.array(ids, dtype=np.int64)
            m.close()
    np.savez_compressed(os.path.join(HERE, "tiny_logits.npz"), **out)
    print("wrote", sorted(os.listdir(HERE)))


if __name__ == "__main__":
    main()
