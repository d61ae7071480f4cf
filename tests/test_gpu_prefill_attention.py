"""Causal attention of whole prompts on the tensor cores (b200k_prefill_attention) against the reference's per-token
path: kernel.ts:344-357 rope on each token's query and key, then kernel.ts:447-566 attentionOf over positions 0..t
(the oracle's restatement, at small sizes), and against float64 at the prefill-attention config (4 sequences of 2048
tokens, 8 heads = 8 kv heads of 64, RoPE theta 1e4, Q/K/V N(0, 1) seed 1). The bar: every output within 1e-3 of the
reference's largest output value of its (sequence, head), and the norm of the error within 1e-3 of the reference's.
GPU only."""
import ctypes

import numpy as np
import pytest

import oracle
from b200fwd import abi
from b200fwd import checkpoint as ck
from gpu_util import dev, empty, full, host, ptr

pytestmark = pytest.mark.gpu
TOL = 1e-3


def run(q, k, v, theta=10000.0):
    lib = abi.load()
    B, S, H, D = q.shape
    KV = k.shape[2]
    cos, sin = ck.rope_tables(S, D, theta)
    size = ctypes.c_uint64()
    abi.check(lib.b200k_prefill_attention_scratch(B, S, H, KV, D, ctypes.byref(size)))
    scratch = empty(int(size.value) // 4 + 64, np.int32)
    held = [dev(a) for a in (q, k, v, np.ascontiguousarray(cos, np.float32), np.ascontiguousarray(sin, np.float32))]
    out = full((B, S, H, D), float("nan"))
    abi.check(lib.b200k_prefill_attention(ptr(out), *[ptr(t) for t in held], B, S, H, KV, D, ptr(scratch), None))
    abi.check(lib.b200k_prefill_attention_check(ptr(scratch), B, S, H, KV, D, None))
    return host(out), cos.astype(np.float32), sin.astype(np.float32)


def roped(x, cos, sin):
    """kernel.ts:344-357 rope in float32, every position: pairs (2i, 2i+1) turned by the row's tables"""
    x = x.astype(np.float32)
    v0, v1 = x[..., 0::2], x[..., 1::2]
    c, s = cos[None, :, None, :], sin[None, :, None, :]
    out = np.empty_like(x)
    out[..., 0::2] = v0 * c - v1 * s
    out[..., 1::2] = v0 * s + v1 * c
    return out


def within(got, ref):
    for b in range(ref.shape[0]):
        for h in range(ref.shape[2]):
            g, r = got[b, :, h].astype(np.float64), ref[b, :, h].astype(np.float64)
            assert np.abs(g - r).max() <= TOL * np.abs(r).max(), (b, h, np.abs(g - r).max() / np.abs(r).max())
            assert np.linalg.norm(g - r) <= TOL * np.linalg.norm(r), (b, h)


@pytest.mark.parametrize("B,S,H,KV", [(1, 256, 2, 2), (2, 512, 4, 1), (1, 256, 8, 2)])
def test_prefill_attention_is_the_references_per_token_attention(B, S, H, KV):
    rng = np.random.default_rng(B * 1000 + S + H)
    D = 64
    q = rng.standard_normal((B, S, H, D)).astype(np.float32)
    k = rng.standard_normal((B, S, KV, D)).astype(np.float32)
    v = rng.standard_normal((B, S, KV, D)).astype(np.float32)
    got, cos, sin = run(q, k, v)
    ref = np.zeros_like(got)
    for b in range(B):
        kc = np.ascontiguousarray(roped(k[b:b + 1], cos, sin)[0].reshape(S, KV * D))
        vc = np.ascontiguousarray(v[b].reshape(S, KV * D))
        qr = roped(q[b:b + 1], cos, sin)[0]
        for t in range(S):
            ref[b, t] = oracle.attention(qr[t].reshape(-1), kc, vc, t, H, KV, D)[0].reshape(H, D)
    within(got, ref)


def test_prefill_attention_at_the_prefill_config():
    """4 x 2048 tokens, 8 heads of 64, RoPE 1e4, seed 1, against float64 (torch on the device)."""
    import torch

    B, S, H, D = 4, 2048, 8, 64
    rng = np.random.default_rng(1)
    q = rng.standard_normal((B, S, H, D)).astype(np.float32)
    k = rng.standard_normal((B, S, H, D)).astype(np.float32)
    v = rng.standard_normal((B, S, H, D)).astype(np.float32)
    got, cos, sin = run(q, k, v)
    qr = torch.from_numpy(roped(q, cos, sin)).cuda().double().transpose(1, 2)
    kr = torch.from_numpy(roped(k, cos, sin)).cuda().double().transpose(1, 2)
    vv = torch.from_numpy(v).cuda().double().transpose(1, 2)
    s = (qr @ kr.transpose(-1, -2)) * np.float32(1.0 / np.sqrt(np.float32(D)))
    s = s.masked_fill(torch.triu(torch.ones(S, S, dtype=torch.bool, device="cuda"), 1), float("-inf"))
    ref = (torch.softmax(s, -1) @ vv).transpose(1, 2).cpu().numpy()
    within(got, ref)
