"""The oracle (oracle/oracle.cpp) pinned to the reference: its own bit-exact kernel checks (restated in
tests/formulas.py) and fixtures made from the reference's Python (tests/golden/make_golden.py). CPU only."""
import json

import numpy as np
import pytest

import formulas as F
import oracle
from conftest import GOLDEN


def test_int8_sums_ends():
    w, want = F.int8_sums_case()
    assert np.array_equal(oracle.int8_sums(w), want)


@pytest.fixture(scope="module")
def mm():
    return F.MatmulCase()


def test_matmul_q8_lane_order(mm):
    """tests/forward-check.mjs:165-176: matmul_q8 to the bit against its lane formula at 1-8, 11 and 41 groups."""
    for groups in mm.GROUPS:
        w = mm.q8_weights(groups)
        ws = mm.ws[:mm.rows * groups]
        got = oracle.matmul_q8(mm.x8, mm.xs, w, ws, groups * 32)
        assert np.array_equal(got, mm.q8_expected(w, groups)), groups


def test_matmul_q8r_and_tile(mm):
    """tests/forward-check.mjs:195-238: matmul_q8r to the bit against its formula; the tile to the bit against
    matmul_q8r token by token, at 1-9 tokens and row ranges off the fours; rows outside left as they were."""
    for groups in mm.GROUPS:
        m = groups * 32
        w = mm.q8r_weights(groups)
        ws = mm.ws[:mm.rows * groups]
        wc = oracle.int8_sums(w)
        got = oracle.matmul_q8r(mm.x7, mm.xs, w, ws, wc, m)
        assert np.array_equal(got, mm.q8r_expected(w, groups)), groups
        xq, xs = mm.tile_tokens(groups)
        for count in range(1, 10):
            for r0, r1 in mm.RANGES:
                tiles = np.full((9, mm.rows), -7.0, np.float32)
                oracle.matmul_q8r_tile(xq, xs, w, ws, wc, m, r0, r1, count, tiles)
                singles = np.full((9, mm.rows), -7.0, np.float32)
                for t in range(count):
                    oracle.matmul_q8r(xq[t], xs[t], w, ws, wc, m, r0, r1, out=singles[t])
                assert np.array_equal(tiles.view(np.uint32), singles.view(np.uint32)), (groups, count, r0, r1)


def test_matmul_q8r_ends_of_int8():
    """tests/forward-check.mjs:240-276: exact against float64 at the ends of int8."""
    w, ws, xq, xs, want, n = F.ends_case()
    wc = oracle.int8_sums(w)
    tiles = np.full((4, 8), -7.0, np.float32)
    oracle.matmul_q8r_tile(xq, xs, w, ws, wc, n, 0, 8, 4, tiles)
    for t in range(4):
        single = oracle.matmul_q8r(xq[t], xs[t], w, ws, wc, n)
        assert np.array_equal(single.astype(np.float64), want[t])
        assert np.array_equal(tiles[t].astype(np.float64), want[t])


@pytest.mark.parametrize("half", [False, True])
def test_attention_far_leading(half):
    """tests/attention-check.mjs: two positions far above the rest; within 1e-3 of float64."""
    table = F.half_table() if half else None
    worst, cases = 0.0, 0
    for count, a, b, q, kc, vc in F.attention_cases():
        if half:
            kh, vh = oracle.to_f16(kc), oracle.to_f16(vc)
            out, _ = oracle.attention(q, kh, vh, count - 1, 2, 2, 8, half=True)
            want = F.attention_expected(q, table[kh].reshape(count, 16), table[vh].reshape(count, 16), count)
        else:
            out, _ = oracle.attention(q, kc, vc, count - 1, 2, 2, 8)
            want = F.attention_expected(q, kc, vc, count)
        off = np.abs(out.astype(np.float64) - want).max()
        worst = max(worst, off)
        cases += 1
        assert off <= 1e-3, (count, a, b, off)
    assert cases > 5000


def test_fexp_vexp():
    xs = np.concatenate([np.linspace(-100, 100, 20001, dtype=np.float32), np.float32([-87.5, -87, 88, 89, 0, -0.0])])
    for x in xs:
        f, v = oracle.fexp(x), oracle.vexp(x)
        if x >= -87:
            assert f == v, x
            ref = np.exp(np.float64(min(x, 88.0)))
            assert abs(f - ref) <= 2e-7 * ref, x
        else:
            assert f == 0 and v == oracle.vexp(np.float32(-87))


def test_to_from_f16_numpy_exact():
    """to_f16 is NumPy's astype(float16) (kernel.ts:568-569); from_f16 reads every half exactly."""
    rng = np.random.default_rng(0)
    x = np.concatenate([rng.standard_normal(20000).astype(np.float32) * np.float32(10) ** rng.integers(-9, 6, 20000),
                        np.float32([0, -0.0, 65504, 65519, 65520, 1e6, -1e6, 6e-8, 3e-8, 2.9e-8, 1e-12])]).astype(np.float32)
    with np.errstate(over="ignore"):
        want = x.astype(np.float16).view(np.uint16)
    assert np.array_equal(oracle.to_f16(x), want)
    halves = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    got = oracle.from_f16(halves)
    finite = np.isfinite(halves.view(np.float16))
    assert np.array_equal(got[finite], halves.view(np.float16)[finite].astype(np.float32))
    assert np.array_equal(got, F.half_table())


def test_quantize_x_is_the_converters_quantize():
    """quantize_x(bias 0) gives the bits of llama2_convert.quantize() (kernel.ts:130-133); golden from the
    reference's own quantize() (tests/golden/quantize.npz)."""
    g = np.load(GOLDEN / "quantize.npz")
    from b200fwd.checkpoint import quantize

    q, s = quantize(g["values"])
    assert np.array_equal(q, g["q"]) and np.array_equal(s, g["s"])
    for row in range(g["values"].shape[0]):
        xq, xs = oracle.quantize_x(g["values"][row], 0)
        assert np.array_equal(xq, g["q"].reshape(37, 96)[row]) and np.array_equal(xs, g["s"].reshape(37, 3)[row])


def test_quantize_x_bias64_range():
    rng = np.random.default_rng(1)
    x = rng.standard_normal(4096).astype(np.float32)
    xq, xs = oracle.quantize_x(x, 64)
    assert xq.min() >= 1 and xq.max() <= 127
    back = (xq.astype(np.float32) - 64).reshape(-1, 32) * xs[:, None]
    assert np.abs(back.reshape(-1) - x).max() <= xs.max() * 0.5 + 1e-7


def test_rope_tables_golden():
    from b200fwd.checkpoint import rope_tables

    g = np.load(GOLDEN / "rope.npz")
    cos, sin = rope_tables(300, 48, 10000.0)
    assert np.array_equal(cos, g["cos"]) and np.array_equal(sin, g["sin"])
    cos, sin = rope_tables(64, 128, 500000.0)
    assert np.array_equal(cos, g["cos8b"]) and np.array_equal(sin, g["sin8b"])


def test_swiglu_rmsnorm_rope_add_columns_argmax():
    rng = np.random.default_rng(2)
    h1 = rng.standard_normal(103).astype(np.float32) * 30
    h3 = rng.standard_normal(103).astype(np.float32)
    got = oracle.swiglu(h1, h3)
    want = (h1.astype(np.float64) / (1 + np.exp(-h1.astype(np.float64))) * h3).astype(np.float32)
    assert np.allclose(got, want, rtol=1e-5, atol=1e-6)
    x = rng.standard_normal(99).astype(np.float32)
    w = rng.standard_normal(99).astype(np.float32)
    got = oracle.rmsnorm(x, w)
    want = w * x / np.sqrt(np.mean(x.astype(np.float64) ** 2) + 1e-5)
    assert np.allclose(got, want, rtol=1e-5)
    v = rng.standard_normal(3 * 16).astype(np.float32)
    c, s = np.cos([0.1 * i for i in range(8)]).astype(np.float32), np.sin([0.1 * i for i in range(8)]).astype(np.float32)
    out = oracle.rope(v, c, s, 3, 16)
    pairs = v.reshape(3, 8, 2)
    assert np.allclose(out.reshape(3, 8, 2)[..., 0], pairs[..., 0] * c - pairs[..., 1] * s, atol=1e-6)
    y = rng.standard_normal(37).astype(np.float32)
    rows = rng.standard_normal((3, 37)).astype(np.float32)
    a = rng.standard_normal(3).astype(np.float32)
    want = y.copy()
    for c_ in range(3):
        want = (want + a[c_] * rows[c_]).astype(np.float32)
    assert np.array_equal(oracle.add_columns(y, rows, a), want)
    z = np.float32([1, 3, 3, 2])
    assert oracle.argmax(z) == 1


def golden_model(name):
    from b200fwd import checkpoint as ck
    import hashlib

    g = np.load(GOLDEN / f"numpy_{name}.npz")
    header = tuple(int(v) for v in g["header"])
    data = ck.synthetic_checkpoint(header, seed=int(g["seed"]), norm=str(g["norm"]))
    assert hashlib.sha256(data).digest() == g["sha256"].tobytes(), "the synthetic checkpoint is not the golden one"
    plan = json.loads((GOLDEN / f"plan_{name}.json").read_text())
    d = np.load(GOLDEN / f"plan_{name}.npz")
    plan["derived"] = {k: d[k].tobytes() for k in d.files}
    return data, plan, g


@pytest.mark.parametrize("name", ["tiny_gqa", "tiny_mha", "tiny_mqa"])
def test_plan_is_the_references(name):
    """b200fwd.checkpoint.make_plan builds the plan Llama.external_forward builds (captured from the reference)."""
    from b200fwd import checkpoint as ck

    data, plan, g = golden_model(name)
    mine = ck.make_plan(ck.header_of(data), lambda o, n: data[o:o + n])
    for key in plan:
        if key == "derived":
            for k in plan["derived"]:
                assert mine["derived"][k] == plan["derived"][k], k
        else:
            assert mine[key] == plan[key], key


@pytest.mark.parametrize("name", ["tiny_gqa", "tiny_mha", "tiny_mqa"])
def test_oracle_engine_against_numpy(name):
    """forward.js's line against the NumPy engine on int8 (tests/forward-check.mjs:2-9,437): the most likely token
    the same at >= 85% of 128 positions and the perplexity within 5%; forwardMany in blocks bit-identical to
    token-by-token (forward-check.mjs:440-451), over a cache that grows past kv_start."""
    data, plan, g = golden_model(name)
    plan = dict(plan, kv_start=16)
    e = oracle.OracleEngine(data, plan, threads=3)
    tokens, ref = g["tokens"], g["logits"]
    same, nll_mine, nll_ref = 0, 0.0, 0.0
    for pos in range(len(tokens)):
        logits = e.forward(int(tokens[pos]), pos)
        same += int(np.argmax(logits) == np.argmax(ref[pos]))
        if pos + 1 < len(tokens):
            nxt = int(tokens[pos + 1])
            for lg, acc in ((logits, 0), (ref[pos], 1)):
                lp = lg.astype(np.float64) - np.log(np.sum(np.exp(lg.astype(np.float64) - lg.max()))) - lg.max()
                if acc == 0:
                    nll_mine -= lp[nxt]
                else:
                    nll_ref -= lp[nxt]
    assert same / len(tokens) >= 0.85
    ppl_mine, ppl_ref = np.exp(nll_mine / (len(tokens) - 1)), np.exp(nll_ref / (len(tokens) - 1))
    assert abs(ppl_mine / ppl_ref - 1) <= 0.05
    last = e.forward(int(tokens[-1]), len(tokens) - 1)
    # blocks of 37 from a fresh engine, then the last token: bit-identical
    e2 = oracle.OracleEngine(data, plan, threads=2)
    e2.forward_many(tokens[:-1], 0)
    last2 = e2.forward(int(tokens[-1]), len(tokens) - 1)
    e3 = oracle.OracleEngine(data, plan, threads=1)
    for start in range(0, len(tokens) - 1, 37):
        e3.forward_many(tokens[start:min(start + 37, len(tokens) - 1)], start)
    last3 = e3.forward(int(tokens[-1]), len(tokens) - 1)
    assert np.array_equal(last.view(np.uint32), last2.view(np.uint32))
    assert np.array_equal(last.view(np.uint32), last3.view(np.uint32))
    k1, v1 = e.keys_values(0, len(tokens))
    k3, v3 = e3.keys_values(0, len(tokens))
    assert np.array_equal(k1, k3) and np.array_equal(v1, v3)


def generate_like_the_reference(engine, prompt, steps, bos=1, stops=(1,)):
    """public/llama2_numpy.py:1565-1671 generate(prompt, temperature=0) as it drives an engine with forwardMany
    (`Llama.external_forward`, :1276-1283): [BOS] + prompt[:-1] through forwardMany in blocks of promptBlock, then
    forward(token, pos) and greedy sampling (np.argmax, :1521-1527) from the last prompt token, until `steps`
    positions or a stop token. `engine` has forward.js's members and a bound logits array `engine.bound_logits`.
    Returns (the blocks fed as (pos, tokens) pairs, the chosen ids)."""
    fed, calls = [bos] + list(prompt[:-1]), []
    at = 0
    while at < len(fed):
        block = fed[at:at + int(engine.promptBlock)]
        engine.forwardMany(block, at)
        calls.append((at, list(block)))
        at += len(block)
    token, pos, chosen = prompt[-1], len(fed), []
    while pos < steps:
        engine.forward(token, pos)
        calls.append((pos, [token]))
        nxt = int(np.argmax(engine.bound_logits))
        assert np.isfinite(engine.bound_logits[nxt]), "NOT_FINITE"
        chosen.append(nxt)
        if nxt in stops:
            break
        token, pos = nxt, pos + 1
    return calls, chosen


class OracleAsEngine:
    """forward.js's members over the oracle (test infrastructure), for generate_like_the_reference."""

    def __init__(self, data, plan, block):
        self.ref = oracle.OracleEngine(data, plan, half_keys=-1, threads=2)
        self.promptBlock = block
        self.bound_logits = np.zeros(plan["vocab_size"], np.float32)

    def forwardMany(self, tokens, pos):
        self.ref.forward_many(tokens, pos)

    def forward(self, token, pos, needLogits=True):
        self.bound_logits[:] = self.ref.forward(token, pos)


def test_generate_fixture_is_the_oracles():
    """generate_tiny_gqa.npz was made by the unmodified reference Llama.generate() driving an oracle-backed engine
    (tests/golden/make_golden.py): the same driving loop restated here, on the oracle, feeds the same blocks and
    chooses the same ids; and it matches the calls the reference made."""
    data, plan, _ = golden_model("tiny_gqa")
    g = np.load(GOLDEN / "generate_tiny_gqa.npz")
    prompt, steps = [int(t) for t in g["prompt"]], int(g["steps"])
    calls, chosen = generate_like_the_reference(OracleAsEngine(data, plan, int(g["prompt_block"])), prompt, steps)
    assert chosen == [int(t) for t in g["ids"]]
    assert np.array_equal(np.concatenate([[p + i for i in range(len(t))] for p, t in calls]), g["fed_pos"])
    assert np.array_equal(np.concatenate([t for _, t in calls]), g["fed_tok"])
    assert len(calls) == int(g["fed_call"].max()) + 1


def test_penalize_and_sample_against_the_numpy_sampler():
    """kernel.ts penalize/sample (restated in the oracle) against the reference's NumPy sampler (Llama.penalize and
    Llama.sample, public/llama2_numpy.py:1514-1563) on the same logits, temperatures, top-p values and random
    numbers (tests/golden/sample.npz): penalize the same to the bit (the same float32 operations); sample draws the
    same token for all but the draws whose random number falls within rounding of a boundary between two tokens (the
    kernel's exponentials are float32, NumPy's float64)."""
    g = np.load(GOLDEN / "sample.npz")
    same = 0
    for i in range(g["chosen"].size):
        pen = oracle.penalize(g["logits"][i], g["history"][i][-64:], 1.3)
        assert np.array_equal(pen.view(np.uint32), g["penalized"][i].view(np.uint32)), i
        token = oracle.sample(pen, g["temperature"][i], g["topp"][i], g["random"][i])
        same += int(token == g["chosen"][i])
    assert same >= 0.99 * g["chosen"].size, same


def test_sample_edges():
    """sample()'s own rules (kernel.ts:801-868): logits whose largest is NaN or +inf give -1; the nucleus of a token
    far above the rest is that token alone, whatever the random number; without a nucleus (topp 1) the last
    cumulative step covers random numbers up to 1."""
    x = np.zeros(50, np.float32)
    x[7] = np.nan
    assert oracle.sample(x, 1.0, 0.9, 0.5) == -1
    x[7] = np.inf
    assert oracle.sample(x, 1.0, 0.9, 0.5) == -1
    y = np.zeros(50, np.float32)
    y[31] = 40.0
    assert all(oracle.sample(y, 1.0, 0.9, r) == 31 for r in (0.0, 0.5, 0.999999))
    z = np.zeros(8, np.float32)
    assert [oracle.sample(z, 1.0, 1.0, r) for r in (0.0, 0.13, 0.99999)] == [0, 1, 7]
