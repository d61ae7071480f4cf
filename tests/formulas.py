"""The reference's bit-exact kernel checks, restated in Python: inputs made by the same LCG and the expected numbers
by the same formulas, so that the oracle (CPU) and the CUDA kernels (GPU) are held to what the reference holds its
WASM kernels to.

  - tests/forward-check.mjs:119-238: matmul_q8's lane order (dot32's lanes, each scaled on its own, lanes summed
    last); matmul_q8r's grouping (lane g % 4, lanes summed in order, groups past the fours one by one, the bias taken
    out of each group's integer); matmul_q8r_tile bit-identical to matmul_q8r at 1-9 tokens and odd row ranges.
  - tests/forward-check.mjs:240-276: the ends of int8 (-128, 127 against 127 and 1) with power-of-two scales,
    exact in float64.
  - tests/forward-check.mjs:38-68: int8_sums, including all -128 (262144) and all 127 (-260096).
  - tests/attention-check.mjs:30-87: two positions far above the rest, 1, 4 and 32 apart, 2 to 72 positions, one
    head above zero and one below, float32 and float16 caches, within 1e-3 of float64.
"""
import math

import numpy as np

f32 = np.float32


class LCG:
    """seed = Math.imul(seed, 1103515245) + 12345 >>> 0; next() = seed >>> 8 (tests/forward-check.mjs)."""

    def __init__(self, seed):
        self.seed = seed & 0xFFFFFFFF

    def next(self):
        self.seed = (self.seed * 1103515245 + 12345) & 0xFFFFFFFF
        return self.seed >> 8

    def random(self):  # tests/attention-check.mjs:27, [0, 1)
        return self.next() / 2 ** 24


def fround(x):
    return f32(x)


# ------------------------------------------------------------------------------------ int8_sums (forward-check :38-68)
def int8_sums_case():
    groups = 2000 * 24 // 32
    u = np.array([((i * 2654435761) & 0xFFFFFFFF) >> 7 & 255 for i in range(groups * 32)], dtype=np.uint8)
    w = u.view(np.int8).copy()
    w[:32] = -128
    w[32:64] = 127
    want = (-64 * w.reshape(-1, 32).astype(np.int64).sum(axis=1)).astype(np.int32)
    assert want[0] == 262144 and want[1] == -260096
    return w, want


# ------------------------------------------------------------------- matmul_q8 / q8r / tile (forward-check :119-238)
class MatmulCase:
    rows, ng = 24, 41
    n = 32 * 41
    GROUPS = [1, 2, 3, 4, 5, 6, 7, 8, 11, 41]
    RANGES = [(0, 24), (1, 23), (2, 5), (3, 10), (4, 8), (5, 6), (7, 7)]

    def __init__(self):
        rows, n, ng = self.rows, self.n, self.ng
        r = LCG(7)
        self.pool = np.array([(r.next() & 255) - 128 for _ in range(rows * n)], dtype=np.int8)
        x = np.array([(r.next() % 255) - 127 for _ in range(n)], dtype=np.int8)
        x[:32] = 127
        x[32:64] = -127
        self.x8 = x
        self.ws = np.array([fround(1e-3 * (1 + (r.next() % 1000))) for _ in range(rows * ng)], dtype=np.float32)
        self.xs = np.array([fround(1e-2 * (1 + (r.next() % 1000))) for _ in range(ng)], dtype=np.float32)
        self.u6 = np.array([r.next() & 255 for _ in range(rows * ng * 24)], dtype=np.uint8)
        self.x7 = np.array([r.next() % 128 for _ in range(n)], dtype=np.int8)
        self.lcg = r  # continues into the tile's tokens, in the order of GROUPS

    # the int8 value of int6 weight j of row i of `groups` groups (forward-check.mjs:132-136)
    def six(self, i, j, groups):
        at = (i * groups + (j >> 5)) * 24
        m = j & 31
        low = self.u6[at + m] & 15 if m < 16 else self.u6[at + m - 16] >> 4
        top = (self.u6[at + 16 + (m % 8)] >> (2 * (m // 8))) & 3
        v = ((int(low) | (int(top) << 4)) << 2) & 255
        return v - 256 if v >= 128 else v

    def q8_weights(self, groups):
        m = groups * 32
        w = np.zeros((self.rows, m), np.int8)
        for i in range(self.rows):
            w[i] = self.pool[i * self.n:i * self.n + m]
        w = w.reshape(-1)
        w[:32] = 127
        start = m + (32 if groups > 1 else 0)
        w[start:start + 32] = -128
        return w

    def q8_expected(self, w, groups):
        """matmul_q8's formula: lane k of each group holds products 2k, 2k+1, 2k+8, 2k+9, +16..."""
        m = groups * 32
        out = np.zeros(self.rows, np.float32)
        x = self.x8.astype(np.int64)
        for i in range(self.rows):
            lanes = [f32(0)] * 4
            for g in range(groups):
                s = f32(self.ws[i * groups + g] * self.xs[g])
                for lane in range(4):
                    idx = [2 * lane, 2 * lane + 1, 2 * lane + 8, 2 * lane + 9, 2 * lane + 16, 2 * lane + 17,
                           2 * lane + 24, 2 * lane + 25]
                    total = sum(int(w[i * m + g * 32 + j]) * int(x[g * 32 + j]) for j in idx)
                    lanes[lane] = f32(lanes[lane] + f32(f32(total) * s))
            out[i] = f32(f32(f32(lanes[0] + lanes[1]) + lanes[2]) + lanes[3])
        return out

    def q8r_weights(self, groups):
        m = groups * 32
        return np.array([self.six(i, j, groups) for i in range(self.rows) for j in range(m)], dtype=np.int8)

    def q8r_expected(self, w, groups, x=None, xs=None):
        """matmul_q8r's formula (forward-check.mjs:208-221): each group's exact dot(w, q - 64) scaled once, into lane
        g % 4 for the groups in fours, lanes summed in order, the groups past the fours one at a time."""
        x = self.x7 if x is None else x
        xs = self.xs if xs is None else xs
        m, fours = groups * 32, groups & ~3
        out = np.zeros(self.rows, np.float32)
        wi = w.astype(np.int64).reshape(self.rows, m)
        xi = x.astype(np.int64)[:m] - 64
        for i in range(self.rows):
            def part(g):
                dot = int((wi[i, g * 32:(g + 1) * 32] * xi[g * 32:(g + 1) * 32]).sum())
                return f32(f32(dot) * f32(self.ws[i * groups + g] * xs[g]))

            lanes = [f32(0)] * 4
            for g in range(fours):
                lanes[g & 3] = f32(lanes[g & 3] + part(g))
            total = f32(f32(f32(lanes[0] + lanes[1]) + lanes[2]) + lanes[3])
            for g in range(fours, groups):
                total = f32(total + part(g))
            out[i] = total
        return out

    def tile_tokens(self, groups):
        """Nine tokens' activations (0..127) and scales for the tile check (forward-check.mjs:225-228); the LCG
        continues from the previous group count's, so call in the order of GROUPS."""
        m = groups * 32
        xq = np.zeros((9, m), np.int8)
        xs = np.zeros((9, groups), np.float32)
        for t in range(9):
            for j in range(m):
                xq[t, j] = self.lcg.next() % 128
            for g in range(groups):
                xs[t, g] = fround(1e-2 * (1 + (self.lcg.next() % 1000)))
        return xq, xs


def ends_case():
    """forward-check.mjs:240-276: weights -128/127 against activations 127/1 (and mixes), power-of-two scales."""
    rows, groups = 8, 5
    n = groups * 32
    r = LCG(11)
    patterns = [lambda j: -128, lambda j: 127, lambda j: 127 if j & 1 else -128, lambda j: -128 if (j & 31) < 16 else 127]
    w = np.zeros((rows, n), np.int8)
    for i in range(rows):
        for j in range(n):
            w[i, j] = patterns[i](j) if i < 4 else (r.next() & 255) - 128
    acts = [lambda j: 127, lambda j: 1, lambda j: 1 if j & 1 else 127, lambda j: 1 + (r.next() % 127)]
    xq = np.zeros((4, n), np.int8)
    xs = np.zeros((4, groups), np.float32)
    for t in range(4):
        for j in range(n):
            xq[t, j] = acts[t](j)
        xs[t, :] = 2.0 ** -(2 + t)
    ws = np.full(rows * groups, 2.0 ** -7, np.float32)
    want = np.zeros((4, rows), np.float64)
    for t in range(4):
        for i in range(rows):
            want[t, i] = float(np.sum(w[i].astype(np.float64) * (xq[t].astype(np.float64) - 64))) * 2.0 ** -7 * 2.0 ** -(2 + t)
    return w.reshape(-1), ws, xq, xs, want, n


# -------------------------------------------------------------------------------------- attention (attention-check)
def half_to_float(h):
    h = int(h)
    sign = -1.0 if h & 0x8000 else 1.0
    e, m = (h >> 10) & 31, h & 1023
    if e == 0:
        return sign * m * 2.0 ** -24
    return sign * (1 + m / 1024) * 2.0 ** (e - 15)


def attention_cases(most=72):
    """Yields (count, a, b, q, kc, vc): the cache of `count` positions, 2 heads of 8, one kv head each."""
    nh, hs = 2, 8
    kv_dim = nh * hs
    r = LCG(12345)
    u = [r.random() * 2 - 1 for _ in range(hs)]
    uu = sum(x * x for x in u)
    q = np.array(u * nh, dtype=np.float32)
    levels = [((-2, 2), 110), ((-260, -250), -100)]
    for count in range(2, most + 1):
        for apart in (1, 4, 32):
            for a in range(count - apart):
                b = a + apart
                kc = np.zeros((count, kv_dim), np.float32)
                vc = np.zeros((count, kv_dim), np.float32)
                for h in range(nh):
                    (low, high), top = levels[h]
                    for t in range(count):
                        score = top if t == a else top - 3 if t == b else low + (high - low) * r.random()
                        for i in range(hs):
                            kc[t, h * hs + i] = (score * math.sqrt(hs) / uu) * u[i]
                            vc[t, h * hs + i] = 1 if t == a else -1 if t == b else r.random() * 2 - 1
                yield count, a, b, q, kc, vc


def attention_expected(q, keys, values, count, nh=2, hs=8):
    """float64 softmax-weighted sum from the numbers the kernel reads (attention-check.mjs:63-75)."""
    out = np.zeros(nh * hs)
    for h in range(nh):
        qh = q[h * hs:(h + 1) * hs].astype(np.float64)
        scores = keys[:count, h * hs:(h + 1) * hs].astype(np.float64) @ qh / math.sqrt(hs)
        wts = np.exp(scores - scores.max())
        wts /= wts.sum()
        out[h * hs:(h + 1) * hs] = wts @ values[:count, h * hs:(h + 1) * hs].astype(np.float64)
    return out


def half_table():
    """The float32 value of every float16 bit pattern as the reference reads it (kernel.ts:383-392): exact, except
    that an infinity reads as 65536 and a NaN as a number."""
    out = np.zeros(65536, np.float32)
    for h in range(65536):
        v = np.int32(np.int16(np.uint16(h)))
        bits = np.uint32((int(v) << 13) & 0x8FFFFFFF)
        out[h] = f32(np.array([bits], np.uint32).view(np.float32)[0] * f32(5.192296858534828e33))
    return out
