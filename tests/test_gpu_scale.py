"""Parity at the sizes the bench's numbers are quoted on, to the bit against the oracle (GPU only):

- the engine at the Llama-3-8B width (dim 4096, FFN 14336, 32/8 heads of 128, vocab 128256, RoPE theta 5e5, float16
  keys and values), two layers: 64 sequences whose 64-token prompts go through one run() (every matmul a 4096-token
  tensor-core GEMM, as the bench's prefill calls are), then 64 greedy tokens each on the device; the logits of the
  last prompt token and every greedy id of three of the sequences checked against the oracle's forward.js run();
- the int8 GEMM (b200k_matmul_q8s) on the 28672 x 4096 w1|w3 matrix at 512 and 4096 tokens;
- decode attention (b200k_attention_batch) at the 8B shape: 64 sequences, contexts drawn from U[512, 8192]
  (seed 2), 32 query / 8 key-value heads of 128, float16 cache, one query token each.
The reference functions: public/forward.js:1011-1090 (run), kernels/kernel_relaxed.ts:34-67,164-183 (matmul_q8r,
matmul_q8r_tile), kernels/kernel.ts:447-566 (attentionOf)."""
import os

import numpy as np
import pytest

import oracle
from b200fwd import abi, synthetic
from b200fwd.forward import Engine
from gpu_util import bits, dev, full, host, ptr
from test_gpu_kernels import matmul_signed

pytestmark = pytest.mark.gpu

HEADER_8B_2 = (4096, 14336, 2, 32, 8, -128256, 256)  # the 8B shape cut to two layers, its own classifier
THREADS = os.cpu_count() or 1


def test_engine_8b_width_batched_prefill_and_greedy():
    import torch

    vocab = abs(HEADER_8B_2[5])
    file = synthetic.make(HEADER_8B_2, seed=11, device="cuda")
    plan = synthetic.plan_for(HEADER_8B_2, file, 500000.0)
    host_ckpt = file.cpu().numpy()
    S, P, G = 64, 64, 64
    eng = Engine(file.data_ptr(), plan, checkpoint_on_device=True, size=file.numel(), half_keys=True, slots=S,
                 max_tokens=S * P, capacity=P + G)
    del file
    torch.cuda.empty_cache()
    rng = np.random.default_rng(5)
    prompts = rng.integers(0, vocab, size=(S, P), dtype=np.int32)
    prompts[:, 0] = 1
    slots = np.repeat(np.arange(S, dtype=np.int32), P)
    pos = np.tile(np.arange(P, dtype=np.int32), S)
    logits, first = eng.run(slots, prompts.reshape(-1), pos, want=pos == P - 1)
    ids = eng.generate_greedy(np.arange(S, dtype=np.int32), first, np.full(S, P, np.int32), G - 1)
    eng.release()
    for s in (0, 29, 63):
        ref = oracle.OracleEngine(host_ckpt, plan, half_keys=1, threads=THREADS)
        ref.forward_many(prompts[s, :-1], 0)
        want = ref.forward(int(prompts[s, -1]), P - 1)
        assert np.array_equal(bits(logits[s]), bits(want)), s
        token = int(np.argmax(want))
        assert token == first[s], s
        for i in range(G - 1):
            token = int(np.argmax(ref.forward(token, P + i)))
            assert token == ids[s, i], (s, i)
        ref.close()


@pytest.mark.parametrize("count", [512, 4096])
def test_gemm_w13_shape_large_token_counts(count):
    rows, n = 28672, 4096
    rng = np.random.default_rng(count)
    w = rng.integers(-127, 128, size=rows * n, dtype=np.int8)
    ws = rng.uniform(0.001, 0.02, rows * n // 32).astype(np.float32)
    x = rng.standard_normal((count, n)).astype(np.float32)
    xq = np.zeros((count, n), np.int8)
    xs = np.zeros((count, n // 32), np.float32)
    for t in range(count):
        xq[t], xs[t] = oracle.quantize_x(x[t], 64)
    got = matmul_signed(lib=abi.load(), xq7=xq, xs=xs, w=w, ws=ws, n=n, count=count)
    wc = oracle.int8_sums(w)
    # whole rows of tokens at the ends of tiles and of the grid ...
    for t in sorted({0, 1, 31, 32, 63, 64, count // 2 + 5, count - 1}):
        want = oracle.matmul_q8r(xq[t], xs[t], w, ws, wc, n)
        assert np.array_equal(bits(got[t]), bits(want)), t
    # ... and the first and last row tiles for every token
    for r0 in (0, rows - 128):
        for t in range(count):
            want = oracle.matmul_q8r(xq[t], xs[t], w, ws, wc, n, r0, r0 + 128)
            assert np.array_equal(bits(got[t, r0:r0 + 128]), bits(want[r0:r0 + 128])), (r0, t)


def test_decode_attention_8b_shape_long_contexts():
    lib = abi.load()
    nh, nkv, hs, seqs = 32, 8, 128, 64
    kvd = nkv * hs
    ctx = np.random.default_rng(2).integers(512, 8193, seqs).astype(np.int32)
    P = int(ctx.max())
    rng = np.random.default_rng(20)
    kc = np.zeros((seqs, P, kvd), np.uint16)
    vc = np.zeros((seqs, P, kvd), np.uint16)
    for s in range(seqs):
        kc[s, :ctx[s]] = rng.standard_normal((ctx[s], kvd)).astype(np.float16).view(np.uint16)
        vc[s, :ctx[s]] = rng.standard_normal((ctx[s], kvd)).astype(np.float16).view(np.uint16)
    q = rng.standard_normal((seqs, nh * hs)).astype(np.float32)
    seq = np.arange(seqs, dtype=np.int32)
    pos = ctx - 1
    out = full((seqs, nh * hs), float("nan"))
    att = full((seqs, nh, P), 0.0)
    held = [dev(a) for a in (q, kc, vc, seq, pos)]
    dq, dk, dv, dseq, dpos = held
    abi.check(lib.b200k_attention_batch(ptr(out), ptr(dq), ptr(dk), ptr(dv), ptr(att), ptr(dseq), ptr(dpos), seqs,
                                        P * kvd, P, nh, nkv, hs, 1, None))
    got = host(out)
    del held
    for s in range(seqs):
        ref, _ = oracle.attention(q[s], kc[s, :ctx[s]], vc[s, :ctx[s]], int(pos[s]), nh, nkv, hs, half=True)
        assert np.array_equal(bits(got[s]), bits(ref)), (s, int(ctx[s]))
