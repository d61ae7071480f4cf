"""The int8 llama2.c "legacy" checkpoint this engine runs, and the plan Python hands the engine.

What Llama(external=...) computes on the Python side before it calls external.start(plan), restated for callers
that do not have public/llama2_numpy.py (the GPU boxes, bench.py): the tensor places of an int8 file
(`Places.take`, public/llama2_numpy.py:751-775, in the order of `llama_tensors`, :1149-1179), the RoPE tables
(`rope_tables`, :484-542), the outlier channels (`outlier_channels`, :807-813) and the plan dict
(`external_forward`, :1248-1270). The int8 format is quantize.py's (public/llama2_convert.py:25-29,125-130):
int8 values, then one float32 scale per group of 32 along the row.

With the reference importable (tests/golden/make_golden.py), tests hold these to the reference's own.
"""
import math
import struct

import numpy as np

KV_START = 256           # public/llama2_numpy.py:552
OUTLIER_CHANNELS = 8     # :561
OUTLIER_RATIO = 4.0      # :562
RMS_EPS = 1e-5           # :427

# (name, shape of the header's sizes, is a matrix) of a llama checkpoint in file order (llama2_convert.layout,
# public/llama2_convert.py:32-92; the RoPE tables are left out of an int8 file, :118)
def layout(dim, hidden_dim, n_layers, n_heads, n_kv_heads, vocab_size, seq_len, head_size=0):
    head_size = head_size or dim // n_heads
    q_dim, kv_dim = n_heads * head_size, n_kv_heads * head_size
    vocab = abs(vocab_size)
    tensors = [("token_embedding_table", (vocab, dim), True), ("rms_att_weight", (n_layers, dim), False),
               ("wq", (n_layers, q_dim, dim), True), ("wk", (n_layers, kv_dim, dim), True),
               ("wv", (n_layers, kv_dim, dim), True), ("wo", (n_layers, dim, q_dim), True),
               ("rms_ffn_weight", (n_layers, dim), False), ("w1", (n_layers, hidden_dim, dim), True),
               ("w2", (n_layers, dim, hidden_dim), True), ("w3", (n_layers, hidden_dim, dim), True),
               ("rms_final_weight", (dim,), False)]
    if vocab_size < 0:
        tensors.append(("wcls", (vocab, dim), True))
    return tensors


def group_size(row_length):
    """public/llama2_convert.py:25-29"""
    size = 32
    while row_length % size:
        size //= 2
    return size


def quantize(values):
    """public/llama2_convert.py:125-130: float32 rows -> (int8 values, float32 scales), one scale per group."""
    groups = values.reshape(-1, group_size(values.shape[-1]))
    scales = (np.abs(groups).max(axis=1) / 127.0).astype(np.float32)
    inverse = np.divide(1.0, scales, out=np.zeros_like(scales), where=scales > 0)
    return np.rint(groups * inverse[:, None]).astype(np.int8), scales


def places(header, head_size=0):
    """{name: Tensor.plan()} of an int8 checkpoint with this header (public/llama2_numpy.py:751-775)."""
    dim, hidden_dim, n_layers, n_heads, n_kv_heads, vocab_size, seq_len = (int(v) for v in header)
    offset, out = 28, {}
    for name, shape, matrix in layout(dim, hidden_dim, n_layers, n_heads, n_kv_heads, vocab_size, seq_len, head_size):
        count = math.prod(shape)
        if matrix:
            group = group_size(shape[-1])
            out[name] = {"kind": "int8", "offset": offset, "shape": list(shape), "group": group,
                         "scales": offset + count}
            offset += count + 4 * (count // group)
        else:
            out[name] = {"kind": "f32", "offset": offset, "shape": list(shape), "group": 0, "scales": 0}
            offset += 4 * count
    if vocab_size > 0:  # a shared classifier is the embedding table (public/llama2_numpy.py:1174)
        out["wcls"] = dict(out["token_embedding_table"])
    return out, offset


def checkpoint_size(header, head_size=0):
    return places(header, head_size)[1]


def rope_tables(seq_len, width, theta):
    """public/llama2_numpy.py:484-496,538-542 without scaling: float64 angles, cos and sin, as float32."""
    frequencies = 1.0 / theta ** (np.arange(0, width, 2, dtype=np.float64) / width)
    angles = np.arange(seq_len, dtype=np.float64)[:, None] * frequencies
    return np.cos(angles).astype(np.float32), np.sin(angles).astype(np.float32)


def outlier_channels(weight, count=OUTLIER_CHANNELS, ratio=OUTLIER_RATIO):
    """public/llama2_numpy.py:807-813"""
    size = np.abs(np.asarray(weight, dtype=np.float32))
    if size.max() < ratio * np.median(size):
        return np.zeros(0, dtype=np.intp)
    return np.sort(np.argsort(-size)[:count])


def header_of(data):
    return struct.unpack_from("<7i", bytes(data[:28]), 0)


def make_plan(header, read, rope_theta=10000.0, relaxed=True, half_kv=True, rms_norm_eps=RMS_EPS, head_size=0):
    """The plan dict Llama.external_forward builds for an int8 llama checkpoint (public/llama2_numpy.py:1248-1270).
    read(offset, length) -> bytes, as external.read."""
    dim, hidden_dim, n_layers, n_heads, n_kv_heads, vocab_size, seq_len = (int(v) for v in header)
    head_size = head_size or dim // n_heads
    tensors, _ = places(header, head_size)
    cos, sin = rope_tables(seq_len, head_size, rope_theta)
    final = tensors["rms_final_weight"]
    weight = np.frombuffer(bytes(read(final["offset"], dim * 4)), dtype=np.float32)
    # the int8 kernels take rows of whole groups of 32 (public/llama2_numpy.py:1058-1060,1066)
    q_dim, kv_dim = n_heads * head_size, n_kv_heads * head_size
    int8 = dim % 32 == 0 and q_dim % 32 == 0 and kv_dim % 32 == 0 and hidden_dim % 32 == 0
    channels = [int(c) for c in outlier_channels(weight, min(OUTLIER_CHANNELS, dim))] if int8 else []
    return {"arch": "llama", "dim": dim, "hidden_dim": hidden_dim, "n_layers": n_layers, "n_heads": n_heads,
            "n_kv_heads": n_kv_heads, "head_size": head_size, "vocab_size": abs(vocab_size), "seq_len": seq_len,
            "rotary": head_size, "parallel_residual": False, "kv_start": KV_START, "rms_norm_eps": float(rms_norm_eps),
            "shared_classifier": vocab_size > 0, "int8": int8, "relaxed": bool(relaxed), "tensors": tensors,
            "derived": {"freq_cis_real": np.ascontiguousarray(cos).tobytes(),
                        "freq_cis_imag": np.ascontiguousarray(sin).tobytes()},
            "outliers": channels, "half_kv": int8 and bool(half_kv),
            "form": {"interval": 0, "k_heads": 0, "v_heads": 0, "k_head": 0, "v_head": 0, "conv": 0, "hadamard": 0,
                     "head_dim": 0}}


def synthetic_checkpoint(header, seed=0, std=0.02, norm="ones"):
    """A seeded int8 checkpoint of this header: every matrix N(0, std) float32 (numpy.random.default_rng(seed)),
    quantized by quantize(); the norm weights 1.0 (norm="ones", llama2.c's convention) or N(0, std) too
    (norm="normal", which sets off the outlier channels). Small models only: it lives in host memory."""
    dim, hidden_dim, n_layers, n_heads, n_kv_heads, vocab_size, seq_len = (int(v) for v in header)
    rng = np.random.default_rng(seed)
    out = [struct.pack("<7i", dim, hidden_dim, n_layers, n_heads, n_kv_heads, vocab_size, seq_len)]
    for name, shape, matrix in layout(dim, hidden_dim, n_layers, n_heads, n_kv_heads, vocab_size, seq_len):
        if matrix:
            values = (rng.standard_normal(shape, dtype=np.float32) * np.float32(std)).astype(np.float32)
            q, s = quantize(values.reshape(-1, shape[-1]))
            out += [q.tobytes(), s.tobytes()]
        elif norm == "ones":
            out.append(np.ones(shape, dtype=np.float32).tobytes())
        else:
            out.append((rng.standard_normal(shape, dtype=np.float32) * np.float32(std)).astype(np.float32).tobytes())
    return b"".join(out)


# The headers of the configurations (dim, hidden_dim, n_layers, n_heads, n_kv_heads, vocab_size, seq_len)
STORIES15M = (288, 768, 6, 6, 6, 32000, 256)
LLAMA3_8B = (4096, 14336, 32, 32, 8, -128256, 8192)
