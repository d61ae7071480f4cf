"""The CUDA kernels through the C ABI (b200k_*) against the reference's own bit-exact checks (tests/formulas.py)
and against the oracle, to the bit. GPU only."""
import ctypes

import numpy as np
import pytest

import formulas as F
import oracle
from b200fwd import abi
from gpu_util import bits, dev, empty, full, host, ptr

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def lib():
    return abi.load()


def matmul(lib, xq, xs, w, ws, wc, n, r0, r1, count, relaxed=True, out_rows=None):
    """xq [count][n] int8, xs [count][n/32]; returns out [count][rows] (rows outside r0..r1 left at -7)."""
    rows = w.size // n if out_rows is None else out_rows
    # rows of 16-byte-aligned activations: pad each token's row to a multiple of 16 bytes
    qs = ((n + 15) // 16) * 16
    xqp = np.zeros((count, qs), np.int8)
    xqp[:, :n] = xq[:count]
    dq, ds = dev(xqp), dev(np.ascontiguousarray(xs[:count], np.float32))
    dw, dws = dev(w), dev(ws)
    dwc = dev(wc) if wc is not None else None
    out = full((count, rows), -7.0)
    if relaxed:
        rc = lib.b200k_matmul_q8r(ptr(out), ptr(dq), ptr(ds), ptr(dw), ptr(dws), ptr(dwc) if dwc is not None else None,
                                  n, r0, r1, count, rows, qs, xs.shape[1], None)
    else:
        rc = lib.b200k_matmul_q8(ptr(out), ptr(dq), ptr(ds), ptr(dw), ptr(dws), n, r0, r1, count, rows, qs,
                                 xs.shape[1], None)
    abi.check(rc)
    return host(out)


@pytest.fixture(scope="module")
def mm():
    return F.MatmulCase()


def test_int8_sums(lib):
    w, want = F.int8_sums_case()
    out, dw = empty(want.size, np.int32), dev(w)
    abi.check(lib.b200k_int8_sums(ptr(out), ptr(dw), want.size, None))
    assert np.array_equal(host(out), want)


def test_matmul_q8_lane_order(lib, mm):
    """tests/forward-check.mjs:165-176 on the GPU: matmul_q8's lane formula, to the bit."""
    for groups in mm.GROUPS:
        w = mm.q8_weights(groups)
        got = matmul(lib, mm.x8[None, :groups * 32], mm.xs[None, :groups], w, mm.ws[:mm.rows * groups], None,
                     groups * 32, 0, mm.rows, 1, relaxed=False)
        assert np.array_equal(bits(got[0]), bits(mm.q8_expected(w, groups))), groups


def test_matmul_q8r_formula_and_tile(lib, mm):
    """tests/forward-check.mjs:195-238 on the GPU: matmul_q8r's formula to the bit (with the int8_sums corrections
    and without them), and count tokens at once to the bit against one at a time, at 1-9 tokens and row ranges off
    the fours; rows outside left as they were."""
    for groups in mm.GROUPS:
        m = groups * 32
        w = mm.q8r_weights(groups)
        ws = mm.ws[:mm.rows * groups]
        wc = oracle.int8_sums(w)
        want = mm.q8r_expected(w, groups)
        for corrections in (wc, None):
            got = matmul(lib, mm.x7[None, :m], mm.xs[None, :groups], w, ws, corrections, m, 0, mm.rows, 1)
            assert np.array_equal(bits(got[0]), bits(want)), (groups, corrections is None)
        xq, xs = mm.tile_tokens(groups)
        for count in range(1, 10):
            for r0, r1 in mm.RANGES:
                tiles = matmul(lib, xq, xs, w, ws, wc, m, r0, r1, count)
                for t in range(count):
                    single = np.full(mm.rows, -7.0, np.float32)
                    oracle.matmul_q8r(xq[t], xs[t], w, ws, wc, m, r0, r1, out=single)
                    assert np.array_equal(bits(tiles[t]), bits(single)), (groups, count, r0, r1, t)


def test_matmul_q8r_ends_of_int8(lib):
    """tests/forward-check.mjs:240-276 on the GPU: exact against float64."""
    w, ws, xq, xs, want, n = F.ends_case()
    wc = oracle.int8_sums(w)
    for corrections in (wc, None):
        got = matmul(lib, xq, xs, w, ws, corrections, n, 0, 8, 4)
        assert np.array_equal(got.astype(np.float64), want)


def test_matmul_q8r_large_random(lib):
    """An 8B-shape slice (n = 4096 and 14336) at 1, 3, 8 and 13 tokens against the oracle, to the bit."""
    rng = np.random.default_rng(3)
    for n, rows in ((4096, 96), (14336, 40)):
        w = rng.integers(-127, 128, size=rows * n, dtype=np.int8)
        ws = rng.uniform(0.001, 0.02, rows * n // 32).astype(np.float32)
        x = rng.standard_normal((13, n)).astype(np.float32)
        xq = np.zeros((13, n), np.int8)
        xs = np.zeros((13, n // 32), np.float32)
        for t in range(13):
            xq[t], xs[t] = oracle.quantize_x(x[t], 64)
        wc = oracle.int8_sums(w)
        for count in (1, 3, 8, 13):
            got = matmul(lib, xq, xs, w, ws, None, n, 0, rows, count)
            for t in range(count):
                want = oracle.matmul_q8r(xq[t], xs[t], w, ws, wc, n)
                assert np.array_equal(bits(got[t]), bits(want)), (n, count, t)


def matmul_signed(lib, xq7, xs, w, ws, n, count, pad=16):
    """b200k_matmul_q8s: activations of quantize_x(bias 64) handed over less the bias; scale rows padded to a
    multiple of `pad` floats."""
    rows = w.size // n
    ng = n // 32
    ngp = (ng + pad - 1) // pad * pad
    qs = ((n + 15) // 16) * 16
    xsg = np.zeros((count, qs), np.int8)
    xsg[:, :n] = (xq7[:count].astype(np.int16) - 64).astype(np.int8)
    xsp = np.zeros((count, ngp), np.float32)
    xsp[:, :ng] = xs[:count, :ng]
    wsp = np.zeros((rows, ngp), np.float32)
    wsp[:, :ng] = ws.reshape(rows, ng)
    dq, ds, dw, dws = dev(xsg), dev(xsp), dev(w), dev(wsp)
    out = full((count, rows), -7.0)
    abi.check(lib.b200k_matmul_q8s(ptr(out), ptr(dq), ptr(ds), ptr(dw), ptr(dws), ngp, n, rows, count, rows, qs, ngp,
                                   None))
    return host(out)


@pytest.mark.parametrize("n,rows,pad", [(4096, 6144, 4), (14336, 300, 16), (288, 768, 4), (160, 200, 4),
                                        (4096, 1024, 16), (4096, 64, 4), (608, 384, 4)])
def test_matmul_tensor_cores(lib, n, rows, pad):
    """The tile tensor-core kernel (count >= 16 tokens, the natural group order) to the bit against the oracle's
    matmul_q8r, at the 8B and stories shapes and at widths with groups past the fours (288: 9 groups; 160: 5; 608:
    19), both token tile widths, scale rows padded to 4 or 16 floats; 64 rows take the CUDA cores."""
    rng = np.random.default_rng(n + rows)
    w = rng.integers(-128, 128, size=rows * n, dtype=np.int8)
    w[:32] = -128
    ws = rng.uniform(0.001, 0.02, rows * n // 32).astype(np.float32)
    wc = oracle.int8_sums(w)
    count_max = 200
    x = rng.standard_normal((count_max, n)).astype(np.float32) * rng.uniform(0.1, 10, (count_max, 1)).astype(np.float32)
    xq = np.zeros((count_max, n), np.int8)
    xs = np.zeros((count_max, n // 32), np.float32)
    for t in range(count_max):
        xq[t], xs[t] = oracle.quantize_x(x[t], 64)
    xq[0, :] = 127
    want = np.stack([oracle.matmul_q8r(xq[t], xs[t], w, ws, wc, n) for t in range(count_max)])
    for count in (16, 17, 33, 64, 100, 200):
        got = matmul_signed(lib, xq, xs, w, ws, n, count, pad)
        assert np.array_equal(bits(got), bits(want[:count])), count


@pytest.mark.parametrize("n,rows", [(4096, 256), (4096, 6144), (288, 256)])
def test_matmul_tensor_cores_extreme_scales(lib, n, rows):
    """Activation scales from subnormal (6e-39) to 1e29 and weight scales from 1e-32 to 1e18, through both
    tensor-core kernels (the lane split for 256 rows, the one-CTA kernel for 6144 and for 9 groups), to the bit
    against the oracle: subnormal scale products, products that underflow, and sums that overflow to infinity. Where
    an infinity meets one of the other sign the result is NaN on both sides; its bit pattern is the platform's (the
    GPU's canonical NaN, x86's default NaN; WASM leaves it unspecified), so NaNs are compared as NaNs. (Scales below
    about 3e-39 have no finite inverse: the reference then quantizes to -128, which the engine's activations less the
    bias of 64 do not hold; such groups are left out here.)"""
    rng = np.random.default_rng(n + 7 * rows)
    w = rng.integers(-128, 128, size=rows * n, dtype=np.int8)
    ws = rng.uniform(0.001, 0.02, rows * n // 32).astype(np.float32)
    ws.reshape(rows, -1)[::7] *= np.float32(1e-30)
    ws.reshape(rows, -1)[3::11] *= np.float32(1e20)
    wc = oracle.int8_sums(w)
    count = 64
    mags = np.array([3e-37, 1e-36, 1e-31, 1e-20, 1.0, 1e20, 1e30, 6e-37], np.float32)
    x = rng.standard_normal((count, n)).astype(np.float32) * mags[np.arange(count) % len(mags)][:, None]
    xq = np.zeros((count, n), np.int8)
    xs = np.zeros((count, n // 32), np.float32)
    for t in range(count):
        xq[t], xs[t] = oracle.quantize_x(x[t], 64)
    assert (xs[xs > 0] < np.float32(1.2e-38)).any() and (xq != -128).all()  # subnormal scales among them
    got = matmul_signed(lib, xq, xs, w, ws, n, count, 4)
    want = np.stack([oracle.matmul_q8r(xq[t], xs[t], w, ws, wc, n) for t in range(count)])
    assert np.isnan(want).any() and (np.abs(want) < np.float32(1.2e-38)).any()  # both ends reached
    assert np.array_equal(np.isnan(got), np.isnan(want))
    finite = ~np.isnan(want)
    assert np.array_equal(bits(got)[finite], bits(want)[finite])


def test_matmul_tensor_cores_formula(lib, mm):
    """forward-check.mjs's matmul_q8r formula through the tensor-core path: its activations repeated to 24 tokens."""
    for groups in mm.GROUPS:
        m = groups * 32
        w = mm.q8r_weights(groups)
        ws = mm.ws[:mm.rows * groups]
        want = mm.q8r_expected(w, groups)
        xq = np.tile(mm.x7[:m], (24, 1))
        xs = np.tile(mm.xs[:groups], (24, 1))
        got = matmul_signed(lib, xq, xs, w, ws, m, 24)
        for t in range(24):
            assert np.array_equal(bits(got[t]), bits(want)), (groups, t)


def test_quantize_x(lib):
    rng = np.random.default_rng(4)
    n, count = 4096 + 96, 5
    x = (rng.standard_normal((count, n)) * rng.uniform(0.01, 100, (count, 1))).astype(np.float32)
    x[1, :32] = 0.0           # a group of zeros: scale 0, inverse 0
    x[2, 32:64] = 1e-39       # subnormal amax: the inverse overflows (T136)
    x[3, 64:96] = -5.0        # all the same value
    for bias in (0, 64):
        dq, ds, dx = empty((count, n), np.int8), empty((count, n // 32), np.float32), dev(x)
        abi.check(lib.b200k_quantize_x(ptr(dq), ptr(ds), ptr(dx), n, bias, count, n, n, n // 32, None))
        gq, gs = host(dq), host(ds)
        for t in range(count):
            wq, wss = oracle.quantize_x(x[t], bias)
            assert np.array_equal(gq[t], wq), (bias, t)
            assert np.array_equal(bits(gs[t]), bits(wss)), (bias, t)


def attention_gpu(lib, q, kc, vc, pos, nh, nkv, hs, half, h0=0, h1=None):
    h1 = nh if h1 is None else h1
    out = full(nh * hs, float("nan"))
    att = full(nh * (pos + 1), 0.0)
    dq, dk, dv = dev(q), dev(kc), dev(vc)  # held until the kernel has run
    abi.check(lib.b200k_attention(ptr(out), ptr(dq), ptr(dk), ptr(dv), ptr(att), pos, nh, nkv, hs, h0, h1,
                                  1 if half else 0, None))
    return host(out), host(att)


@pytest.mark.parametrize("half", [False, True])
def test_attention_far_leading(lib, half):
    """tests/attention-check.mjs on the GPU (a sample of its cases): to the bit against the oracle, and within
    1e-3 of float64."""
    table = F.half_table()
    for i, (count, a, b, q, kc, vc) in enumerate(F.attention_cases()):
        if i % 13:
            continue
        if half:
            kc, vc = oracle.to_f16(kc).reshape(count, 16), oracle.to_f16(vc).reshape(count, 16)
            want_keys, want_vals = table[kc], table[vc]
        else:
            want_keys, want_vals = kc, vc
        got, _ = attention_gpu(lib, q, kc, vc, count - 1, 2, 2, 8, half)
        ref, _ = oracle.attention(q, kc, vc, count - 1, 2, 2, 8, half=half)
        assert np.array_equal(bits(got), bits(ref)), (count, a, b)
        assert np.abs(got.astype(np.float64) - F.attention_expected(q, want_keys, want_vals, count)).max() <= 1e-3


@pytest.mark.parametrize("nh,nkv,hs", [(8, 8, 64), (32, 8, 64), (4, 2, 6), (3, 3, 10), (32, 8, 128), (6, 6, 48)])
@pytest.mark.parametrize("half", [False, True])
def test_attention_shapes(lib, nh, nkv, hs, half):
    """tests/attention-compare.mjs's shapes at positions 0-9, 130 and 700; the heads split in two ranges give the
    numbers of all at once (attention-compare.mjs:165-177); the weights left in att are the oracle's."""
    rng = np.random.default_rng(nh * 100 + hs)
    for pos in (0, 1, 2, 3, 4, 5, 6, 7, 8, 9, 130, 700):
        count = pos + 1
        q = rng.standard_normal(nh * hs).astype(np.float32)
        kc = rng.standard_normal((count, nkv * hs)).astype(np.float32)
        vc = rng.standard_normal((count, nkv * hs)).astype(np.float32)
        if half:
            kc, vc = oracle.to_f16(kc).reshape(count, -1), oracle.to_f16(vc).reshape(count, -1)
        got, att = attention_gpu(lib, q, kc, vc, pos, nh, nkv, hs, half)
        ref, ref_att = oracle.attention(q, kc, vc, pos, nh, nkv, hs, half=half)
        assert np.array_equal(bits(got), bits(ref)), pos
        assert np.array_equal(bits(att), bits(ref_att)), pos
        split = nh // 2 or 1
        lo, _ = attention_gpu(lib, q, kc, vc, pos, nh, nkv, hs, half, 0, split)
        hi, _ = attention_gpu(lib, q, kc, vc, pos, nh, nkv, hs, half, split, nh)
        both = np.where(np.arange(nh * hs) < split * hs, lo, hi)
        assert np.array_equal(bits(both), bits(ref)), pos


@pytest.mark.parametrize("hs", [64, 128])
def test_attention_half_values_of_every_bit_pattern(lib, hs):
    """Float16 value caches of arbitrary bit patterns (subnormals, zeros of both signs, the top exponent that the
    reference's half() widens to finite numbers) through the decode kernels, to the bit against the oracle: the
    values kernel folds half()'s 2^112 into the weights."""
    rng = np.random.default_rng(hs)
    nh, nkv = 32, 8
    for pos in (2, 3, 130, 301):
        count = pos + 1
        q = rng.standard_normal(nh * hs).astype(np.float32)
        kc = oracle.to_f16((rng.standard_normal((count, nkv * hs)) * 0.05).astype(np.float32)).reshape(count, -1)
        vc = rng.integers(0, 65536, (count, nkv * hs)).astype(np.uint16)
        vc[0, :8] = [0x0000, 0x8000, 0x0001, 0x83ff, 0x7c00, 0xfc00, 0x7e01, 0x7bff]
        got, att = attention_gpu(lib, q, kc, vc, pos, nh, nkv, hs, True)
        ref, ref_att = oracle.attention(q, kc, vc, pos, nh, nkv, hs, half=True)
        assert np.array_equal(bits(att), bits(ref_att)), pos
        assert np.array_equal(bits(got), bits(ref)), pos


def test_attention_batch_is_per_token(lib):
    """b200k_attention_batch: each token against its own sequence's cache gives b200k_attention's numbers."""
    rng = np.random.default_rng(9)
    nh, nkv, hs, seqs, P = 8, 2, 64, 3, 300
    kvd = nkv * hs
    kc = oracle.to_f16(rng.standard_normal((seqs, P, kvd)).astype(np.float32)).reshape(seqs, P, kvd)
    vc = oracle.to_f16(rng.standard_normal((seqs, P, kvd)).astype(np.float32)).reshape(seqs, P, kvd)
    seq = np.array([2, 0, 1, 1, 2], np.int32)
    pos = np.array([0, 299, 17, 18, 255], np.int32)
    q = rng.standard_normal((5, nh * hs)).astype(np.float32)
    out = full((5, nh * hs), float("nan"))
    att = full((5, nh, P), 0.0)
    held = [dev(a) for a in (q, kc, vc, seq, pos)]
    dq, dk, dv, dseq, dpos = held
    abi.check(lib.b200k_attention_batch(ptr(out), ptr(dq), ptr(dk), ptr(dv), ptr(att), ptr(dseq), ptr(dpos), 5,
                                        P * kvd, P, nh, nkv, hs, 1, None))
    got = host(out)
    for i in range(5):
        ref, _ = oracle.attention(q[i], kc[seq[i]], vc[seq[i]], int(pos[i]), nh, nkv, hs, half=True)
        assert np.array_equal(bits(got[i]), bits(ref)), i


def test_f16_conversions(lib):
    halves = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    out, dh = empty(65536, np.float32), dev(halves)
    abi.check(lib.b200k_from_f16(ptr(out), ptr(dh), 65536, None))
    assert np.array_equal(bits(host(out)), bits(oracle.from_f16(halves)))
    rng = np.random.default_rng(0)
    x = np.concatenate([rng.standard_normal(50000).astype(np.float32) * np.float32(10) ** rng.integers(-9, 6, 50000),
                        np.float32([0, -0.0, 65504, 65519, 65520, 1e6, 6e-8, 3e-8, 2.9e-8, np.inf, -np.inf])])
    x = x.astype(np.float32)
    h, dx = empty(x.size, np.uint16), dev(x)
    abi.check(lib.b200k_to_f16(ptr(h), ptr(dx), x.size, None))
    assert np.array_equal(host(h).view(np.uint16), oracle.to_f16(x))


def test_small_kernels(lib):
    rng = np.random.default_rng(5)
    n = 1003
    h1 = (rng.standard_normal(n) * 40).astype(np.float32)
    h3 = rng.standard_normal(n).astype(np.float32)
    out, d1, d3 = empty(n, np.float32), dev(h1), dev(h3)
    abi.check(lib.b200k_swiglu(ptr(out), ptr(d1), ptr(d3), n, None))
    assert np.array_equal(bits(host(out)), bits(oracle.swiglu(h1, h3)))
    for dim in (288, 4096, 99):
        x = rng.standard_normal((3, dim)).astype(np.float32)
        w = rng.standard_normal(dim).astype(np.float32)
        o, dx, dw = empty((3, dim), np.float32), dev(x), dev(w)
        abi.check(lib.b200k_rmsnorm(ptr(o), ptr(dx), ptr(dw), dim, np.float32(1e-5), 3, dim, None))
        g = host(o)
        for t in range(3):
            assert np.array_equal(bits(g[t]), bits(oracle.rmsnorm(x[t], w))), (dim, t)
    v = rng.standard_normal(6 * 48).astype(np.float32)
    c, s = rng.standard_normal(24).astype(np.float32), rng.standard_normal(24).astype(np.float32)
    for rot in (0, 16):
        dv, dc, ds = dev(v), dev(c), dev(s)
        abi.check(lib.b200k_rope(ptr(dv), ptr(dc), ptr(ds), 6, 48, rot, None))
        assert np.array_equal(bits(host(dv)), bits(oracle.rope(v, c, s, 6, 48, rot)))
    y = rng.standard_normal(32000).astype(np.float32)
    rows = rng.standard_normal((8, 32000)).astype(np.float32)
    a = rng.standard_normal(8).astype(np.float32)
    dy, drows, da = dev(y), dev(rows), dev(a)
    abi.check(lib.b200k_add_columns(ptr(dy), ptr(drows), ptr(da), 8, 32000, None))
    assert np.array_equal(bits(host(dy)), bits(oracle.add_columns(y, rows, a)))
    xx, yy = rng.standard_normal(777).astype(np.float32), rng.standard_normal(777).astype(np.float32)
    dx, dyy = dev(xx), dev(yy)
    abi.check(lib.b200k_add_inplace(ptr(dx), ptr(dyy), 777, None))
    assert np.array_equal(bits(host(dx)), bits(xx + yy))
    for z in (rng.standard_normal(128256).astype(np.float32), np.float32([1, 5, 5, 2]), np.float32([np.nan, 1, 2])):
        r, dz = empty(1, np.int32), dev(z)
        abi.check(lib.b200k_argmax(ptr(r), ptr(dz), z.size, None))
        assert host(r)[0] == oracle.argmax(z)


def test_bad_arguments_are_refused(lib):
    rc = lib.b200k_matmul_q8r(None, None, None, None, None, None, 32, 0, 1, 1, 1, 32, 1, None)
    assert rc == abi.EINVAL and "null" in abi.last_error()
    rc = lib.b200k_quantize_x(None, None, None, 32, 7, 1, 32, 32, 1, None)
    assert rc == abi.EINVAL and "bias" in abi.last_error()


def test_penalize_and_sample_are_the_oracles(lib):
    """kernel.ts:705-868 penalize and sample (b200k_penalize, b200k_sample) against the oracle's restatement, to the
    bit and the id, on the NumPy-sampler fixture's logits (tests/golden/sample.npz: temperatures 0.3-1.6, top-p 0.5,
    0.9, 0.95 and 1, with their random numbers), on a 128256-wide vocabulary, and on the edges (NaN, +inf)."""
    from conftest import GOLDEN

    g = np.load(GOLDEN / "sample.npz")
    size = ctypes.c_uint64()

    def draw(x, t, p, r):
        abi.check(lib.b200k_sample_scratch(x.size, ctypes.byref(size)))
        scratch = empty(int(size.value) // 4 + 2, np.int32)
        out, dx = full(1, -9, np.int32), dev(np.ascontiguousarray(x, np.float32))
        abi.check(lib.b200k_sample(ptr(out), ptr(dx), x.size, float(t), float(p), float(r), ptr(scratch), None))
        return int(host(out)[0])

    for i in range(0, g["chosen"].size, 3):
        hist = np.ascontiguousarray(g["history"][i][-64:], np.int32)
        dx, dh = dev(g["logits"][i]), dev(hist)
        abi.check(lib.b200k_penalize(ptr(dx), ptr(dh), hist.size, np.float32(1.3), None))
        pen = host(dx)
        assert np.array_equal(bits(pen), bits(oracle.penalize(g["logits"][i], hist, 1.3))), i
        want = oracle.sample(pen, g["temperature"][i], g["topp"][i], g["random"][i])
        assert draw(pen, g["temperature"][i], g["topp"][i], g["random"][i]) == want, i
    rng = np.random.default_rng(8)
    for scale, t, p in ((6.0, 0.8, 0.9), (0.5, 1.0, 0.95), (3.0, 0.7, 1.0)):
        x = (rng.standard_normal(128256) * scale).astype(np.float32)
        for r in (0.0, 0.37, 0.999):
            assert draw(x, t, p, r) == oracle.sample(x, t, p, r), (scale, t, p, r)
    x = np.zeros(100, np.float32)
    x[3] = np.nan
    assert draw(x, 1.0, 0.9, 0.5) == -1
    x[3] = np.inf
    assert draw(x, 1.0, 0.9, 0.5) == -1
