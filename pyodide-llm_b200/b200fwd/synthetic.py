"""Seeded synthetic int8 checkpoints of any size, made with torch on a device (or the CPU) in the checkpoint's own
byte layout: every matrix N(0, std) in float32, quantized per group of 32 exactly as quantize()
(public/llama2_convert.py:125-130: scale = max|w| / 127 in float32, inverse 0 where the scale is 0, round half to
even); norm weights 1.0. For the 8B-shape bench, where numpy on the host would take minutes.

The bytes differ from checkpoint.synthetic_checkpoint's (another generator), not their distribution.
"""
import struct

import numpy as np

from . import checkpoint as ck

CHUNK_ROWS_BYTES = 1 << 28  # floats made at once: 1 GiB of float32


def quantize_rows(values):
    """torch float32 [rows][n] -> (int8 [rows][n], float32 scales [rows][n/32]), quantize()'s arithmetic."""
    import torch

    rows, n = values.shape
    groups = values.reshape(-1, 32)
    scales = groups.abs().amax(dim=1) / 127.0
    inverse = torch.where(scales > 0, 1.0 / scales, torch.zeros_like(scales))
    q = torch.round(groups * inverse[:, None]).to(torch.int8)
    return q.reshape(rows, n), scales.reshape(rows, n // 32)


def make(header, seed=0, std=0.02, device="cuda", norm="ones"):
    """A uint8 torch tensor on `device` holding the whole checkpoint file (header, then the tensors in file order)."""
    import torch

    dim, hidden, layers, heads, kv_heads, vocab, seq_len = (int(v) for v in header)
    size = ck.checkpoint_size(header)
    out = torch.empty(size, dtype=torch.uint8, device=device)
    out[:28] = torch.frombuffer(bytearray(struct.pack("<7i", *header)), dtype=torch.uint8).to(device)
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    offset = 28
    for name, shape, matrix in ck.layout(dim, hidden, layers, heads, kv_heads, vocab, seq_len):
        count = int(np.prod(shape))
        if not matrix:
            vals = torch.ones(count, dtype=torch.float32, device=device) if norm == "ones" else \
                torch.randn(count, generator=gen, device=device, dtype=torch.float32) * std
            out[offset:offset + 4 * count] = vals.view(torch.uint8)
            offset += 4 * count
            continue
        n = shape[-1]
        rows = count // n
        values_at, scales_at = offset, offset + count
        step = max(1, CHUNK_ROWS_BYTES // (4 * n))
        for r0 in range(0, rows, step):
            r1 = min(rows, r0 + step)
            w = torch.randn((r1 - r0, n), generator=gen, device=device, dtype=torch.float32) * std
            q, s = quantize_rows(w)
            out[values_at + r0 * n:values_at + r1 * n] = q.view(torch.uint8).reshape(-1)
            out[scales_at + r0 * (n // 32) * 4:scales_at + r1 * (n // 32) * 4] = s.reshape(-1).view(torch.uint8)
            del w, q, s
        offset += count + 4 * (count // 32)
    assert offset == size
    return out


def plan_for(header, file_tensor, rope_theta, relaxed=True, half_kv=True, rms_norm_eps=ck.RMS_EPS):
    """make_plan() reading the final norm's bytes from the (device) file tensor."""
    def read(offset, length):
        return file_tensor[offset:offset + length].cpu().numpy().tobytes()

    return ck.make_plan(header, read, rope_theta=rope_theta, relaxed=relaxed, half_kv=half_kv,
                        rms_norm_eps=rms_norm_eps)
