"""Block quantizers that write GGUF/ggml block layouts (synthetic-model tooling).

These produce the byte layouts the reference's WGSL dequantizers read:
  Q4_K  144 B / 256: fp16 d, fp16 dmin, 12 B packed 6-bit scales/mins, 128 B
        nibbles (low nibble = first 32 of each 64)   llama-wgsl-runtime.ts:2387-2410
  Q6_K  210 B / 256: ql 128 B, qh 64 B, int8 scales 16 B, fp16 d
                                                     llama-wgsl-runtime.ts:2560-2580
  Q8_0   34 B / 32 : fp16 d, 32 x int8               llama-wgsl-runtime.ts:2321-2327
  Q5_0   22 B / 32 : fp16 d, u32 qh, 16 B nibbles    llama-wgsl-runtime.ts:2234-2245
  Q5_1   24 B / 32 : fp16 d, fp16 m, u32 qh, 16 B    llama-wgsl-runtime.ts:2280-2289
The rounding choices are this project's own (simple min/max fits); any valid
block decodes identically on both sides of a parity test, which is what matters.
All functions take a float32 torch tensor [rows, k] and return uint8 [rows, bytes].
"""
from __future__ import annotations

import torch

from .gguf import GGML_TYPE, BLOCK_LAYOUT


def _f16_bytes(v: torch.Tensor) -> torch.Tensor:
    """[..] float -> [.., 2] uint8 (little-endian fp16)."""
    h = v.to(torch.float16).contiguous()
    return h.view(torch.uint8).reshape(*v.shape, 2)


def _u32_bytes(v: torch.Tensor) -> torch.Tensor:
    v = v.to(torch.int64) & 0xFFFFFFFF
    return torch.stack([(v >> (8 * i)) & 0xFF for i in range(4)], dim=-1).to(torch.uint8)


def quantize_q8_0(x: torch.Tensor) -> torch.Tensor:
    rows, k = x.shape
    b = x.reshape(rows, k // 32, 32)
    amax = b.abs().amax(-1)
    d = amax / 127.0
    d16 = d.to(torch.float16).to(torch.float32)
    inv = torch.where(d16 > 0, 1.0 / d16, torch.zeros_like(d16))
    q = torch.round(b * inv[..., None]).clamp(-127, 127).to(torch.int8)
    out = torch.cat([_f16_bytes(d), q.view(torch.uint8)], dim=-1)
    return out.reshape(rows, -1)


def quantize_q5_0(x: torch.Tensor) -> torch.Tensor:
    rows, k = x.shape
    b = x.reshape(rows, k // 32, 32)
    idx = b.abs().argmax(-1, keepdim=True)
    mx = torch.gather(b, -1, idx).squeeze(-1)
    d = mx / -16.0
    d16 = d.to(torch.float16).to(torch.float32)
    inv = torch.where(d16 != 0, 1.0 / d16, torch.zeros_like(d16))
    q = torch.floor(b * inv[..., None] + 16.5).clamp(0, 31).to(torch.int64)
    lo = q & 15
    hi = (q >> 4) & 1
    qs = (lo[..., :16] | (lo[..., 16:] << 4)).to(torch.uint8)
    qh = (hi << torch.arange(32, device=x.device)).sum(-1)
    out = torch.cat([_f16_bytes(d), _u32_bytes(qh), qs], dim=-1)
    return out.reshape(rows, -1)


def quantize_q5_1(x: torch.Tensor) -> torch.Tensor:
    rows, k = x.shape
    b = x.reshape(rows, k // 32, 32)
    mn = b.amin(-1)
    mx = b.amax(-1)
    d = (mx - mn) / 31.0
    d16 = d.to(torch.float16).to(torch.float32)
    m16 = mn.to(torch.float16).to(torch.float32)
    inv = torch.where(d16 > 0, 1.0 / d16, torch.zeros_like(d16))
    q = torch.round((b - m16[..., None]) * inv[..., None]).clamp(0, 31).to(torch.int64)
    lo = q & 15
    hi = (q >> 4) & 1
    qs = (lo[..., :16] | (lo[..., 16:] << 4)).to(torch.uint8)
    qh = (hi << torch.arange(32, device=x.device)).sum(-1)
    out = torch.cat([_f16_bytes(d), _f16_bytes(mn), _u32_bytes(qh), qs], dim=-1)
    return out.reshape(rows, -1)


def quantize_q4_k(x: torch.Tensor) -> torch.Tensor:
    rows, k = x.shape
    nsb = k // 256
    b = x.reshape(rows, nsb, 8, 32)
    mn = b.amin(-1).clamp(max=0.0)                 # sub-block minimum (<= 0)
    mx = b.amax(-1)
    scale = (mx - mn) / 15.0                       # per sub-block step
    d = scale.amax(-1) / 63.0                      # super-block scale of scales
    dmin = (-mn).amax(-1) / 63.0
    d16 = d.to(torch.float16).to(torch.float32)
    dm16 = dmin.to(torch.float16).to(torch.float32)
    sc = torch.where(d16[..., None] > 0, torch.round(scale / d16[..., None].clamp(min=1e-30)),
                     torch.zeros_like(scale)).clamp(0, 63).to(torch.int64)
    m = torch.where(dm16[..., None] > 0, torch.round(-mn / dm16[..., None].clamp(min=1e-30)),
                    torch.zeros_like(mn)).clamp(0, 63).to(torch.int64)
    # Reconstruct with the same fp32 steps the dequantizer uses.
    step = d16[..., None] * sc.to(torch.float32)
    off = dm16[..., None] * m.to(torch.float32)
    inv = torch.where(step > 0, 1.0 / step, torch.zeros_like(step))
    q = torch.round((b + off[..., None]) * inv[..., None]).clamp(0, 15).to(torch.int64)
    # 12-byte scale packing (inverse of scale_min_k4, llama-wgsl-runtime.ts:2387-2394)
    sb = torch.zeros(rows, nsb, 12, dtype=torch.int64, device=x.device)
    for j in range(4):
        sb[..., j] = sc[..., j] & 63
        sb[..., j + 4] = m[..., j] & 63
    for j in range(4, 8):
        sb[..., j + 4] = (sc[..., j] & 15) | ((m[..., j] & 15) << 4)
        sb[..., j - 4] |= (sc[..., j] >> 4) << 6
        sb[..., j] |= (m[..., j] >> 4) << 6
    qg = q.reshape(rows, nsb, 4, 2, 32)            # [group64][low/high][lane]
    qs = (qg[..., 0, :] | (qg[..., 1, :] << 4)).reshape(rows, nsb, 128)
    out = torch.cat([_f16_bytes(d), _f16_bytes(dmin), sb.to(torch.uint8), qs.to(torch.uint8)], dim=-1)
    return out.reshape(rows, -1)


def quantize_q6_k(x: torch.Tensor) -> torch.Tensor:
    rows, k = x.shape
    nsb = k // 256
    b = x.reshape(rows, nsb, 16, 16)
    amax = b.abs().amax(-1)
    s = amax / 31.0                                # per-16 step, positive
    d = s.amax(-1) / 127.0
    d16 = d.to(torch.float16).to(torch.float32)
    sc = torch.where(d16[..., None] > 0, torch.round(s / d16[..., None].clamp(min=1e-30)),
                     torch.zeros_like(s)).clamp(-127, 127).to(torch.int64)
    step = d16[..., None] * sc.to(torch.float32)
    inv = torch.where(step != 0, 1.0 / step, torch.zeros_like(step))
    q = (torch.round(b * inv[..., None]).clamp(-32, 31) + 32).to(torch.int64)   # 0..63
    q = q.reshape(rows, nsb, 2, 4, 32)             # [half][quarter][lane]
    lo = q & 15
    hi = (q >> 4) & 3
    # ql[half*64 + lane + 32*(quarter&1)]: quarters 0/1 in low nibbles, 2/3 in high
    ql0 = lo[:, :, :, 0, :] | (lo[:, :, :, 2, :] << 4)
    ql1 = lo[:, :, :, 1, :] | (lo[:, :, :, 3, :] << 4)
    ql = torch.cat([ql0, ql1], dim=-1).reshape(rows, nsb, 128)
    qh = (hi[:, :, :, 0, :] | (hi[:, :, :, 1, :] << 2) | (hi[:, :, :, 2, :] << 4) |
          (hi[:, :, :, 3, :] << 6)).reshape(rows, nsb, 64)
    scb = sc.to(torch.int8).view(torch.uint8)
    out = torch.cat([ql.to(torch.uint8), qh.to(torch.uint8), scb, _f16_bytes(d)], dim=-1)
    return out.reshape(rows, -1)


QUANTIZERS = {
    GGML_TYPE.Q8_0: quantize_q8_0,
    GGML_TYPE.Q5_0: quantize_q5_0,
    GGML_TYPE.Q5_1: quantize_q5_1,
    GGML_TYPE.Q4_K: quantize_q4_k,
    GGML_TYPE.Q6_K: quantize_q6_k,
}


def quantize(x: torch.Tensor, ggml_type: int, chunk_rows: int = 4096) -> bytes:
    """Quantize a [rows, k] float tensor to ggml block bytes (row-major)."""
    if ggml_type == GGML_TYPE.F32:
        return x.to(torch.float32).contiguous().cpu().numpy().tobytes()
    if ggml_type == GGML_TYPE.F16:
        return x.to(torch.float16).contiguous().cpu().numpy().tobytes()
    fn = QUANTIZERS[ggml_type]
    block, _ = BLOCK_LAYOUT[ggml_type]
    if x.shape[1] % block:
        raise ValueError(f"row length {x.shape[1]} is not a multiple of {block}")
    parts = []
    for r0 in range(0, x.shape[0], chunk_rows):
        parts.append(fn(x[r0:r0 + chunk_rows].to(torch.float32)).cpu())
    return torch.cat(parts, 0).numpy().tobytes()
