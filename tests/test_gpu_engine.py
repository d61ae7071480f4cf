"""The engine (include/b200fwd.h b200fwd_*) against the oracle's forward.js run(), to the bit, through the
reference's engine interface. GPU only."""
import hashlib
import json

import numpy as np
import pytest

import oracle
from b200fwd import abi, checkpoint as ck
from b200fwd.forward import Engine, external
from conftest import GOLDEN
from gpu_util import bits

pytestmark = pytest.mark.gpu


def golden_model(name):
    g = np.load(GOLDEN / f"numpy_{name}.npz")
    header = tuple(int(v) for v in g["header"])
    data = ck.synthetic_checkpoint(header, seed=int(g["seed"]), norm=str(g["norm"]))
    assert hashlib.sha256(data).digest() == g["sha256"].tobytes()
    plan = json.loads((GOLDEN / f"plan_{name}.json").read_text())
    d = np.load(GOLDEN / f"plan_{name}.npz")
    plan["derived"] = {k: d[k].tobytes() for k in d.files}
    return data, plan, g


MODELS = ["tiny_gqa", "tiny_mha", "tiny_mqa"]


@pytest.mark.parametrize("name", MODELS)
@pytest.mark.parametrize("half_keys", [True, False])
def test_forward_bit_identical_to_oracle(name, half_keys):
    """forward() at every position of the NumPy engine's greedy text: the logits of the oracle's run(), to the bit,
    over a cache that grows from 16 positions; keysAndValues the oracle's."""
    data, plan, g = golden_model(name)
    plan = dict(plan, kv_start=16)
    eng = Engine(data, plan, half_keys=half_keys)
    ref = oracle.OracleEngine(data, plan, half_keys=1 if half_keys else 0, threads=2)
    assert ("float16" in eng.backend) == (half_keys and plan["half_kv"])
    logits = np.zeros(plan["vocab_size"], np.float32)
    eng.bind(logits)
    tokens = g["tokens"]
    for pos in range(len(tokens)):
        eng.forward(int(tokens[pos]), pos)
        want = ref.forward(int(tokens[pos]), pos)
        assert np.array_equal(bits(logits), bits(want)), pos
    kv = eng.keysAndValues(0, len(tokens))
    rk, rv = ref.keys_values(0, len(tokens))
    assert np.array_equal(bits(kv["keys"]), bits(rk)) and np.array_equal(bits(kv["values"]), bits(rv))
    eng.release()


@pytest.mark.parametrize("name", MODELS)
def test_forward_many_blocks_are_tokens(name):
    """tests/forward-check.mjs:440-451: the prompt in blocks of 37 (and of the engine's own block) is bit-identical
    to token by token."""
    data, plan, g = golden_model(name)
    plan = dict(plan, kv_start=16)
    tokens = [int(t) for t in g["tokens"]]
    one = Engine(data, plan)
    for pos, t in enumerate(tokens[:-1]):
        one.forward(t, pos, False)
    one.forward(tokens[-1], len(tokens) - 1)
    a = one.logits()
    blocks = Engine(data, plan)
    for start in range(0, len(tokens) - 1, 37):
        blocks.forwardMany(tokens[start:min(start + 37, len(tokens) - 1)], start)
    blocks.forward(tokens[-1], len(tokens) - 1)
    b = blocks.logits()
    whole = Engine(data, plan, max_tokens=64)
    whole.forwardMany(tokens[:-1], 0)
    whole.forward(tokens[-1], len(tokens) - 1)
    c = whole.logits()
    assert np.array_equal(bits(a), bits(b)) and np.array_equal(bits(a), bits(c))


def test_numpy_line_through_llama_style_driver():
    """The engine against the reference's NumPy engine at forward.js's own line (tests/forward-check.mjs:437): the
    most likely token the same at >= 85% of 128 positions, perplexity within 5%."""
    for name in MODELS:
        data, plan, g = golden_model(name)
        ext = external(data)
        eng = ext.start(plan)
        logits = np.zeros(plan["vocab_size"], np.float32)
        eng.bind(logits)
        tokens, ref = g["tokens"], g["logits"]
        same, nll, nll_ref = 0, 0.0, 0.0
        for pos in range(len(tokens)):
            eng.forward(int(tokens[pos]), pos, True)
            same += int(np.argmax(logits) == np.argmax(ref[pos]))
            if pos + 1 < len(tokens):
                for lg, which in ((logits, 0), (ref[pos], 1)):
                    x = lg.astype(np.float64)
                    lp = x - x.max() - np.log(np.exp(x - x.max()).sum())
                    if which == 0:
                        nll -= lp[tokens[pos + 1]]
                    else:
                        nll_ref -= lp[tokens[pos + 1]]
        assert same / len(tokens) >= 0.85, name
        assert abs(np.exp((nll - nll_ref) / (len(tokens) - 1)) - 1) <= 0.05, name


def stories_plan(data, seq_len=256):
    return ck.make_plan(ck.header_of(data), lambda o, n: data[o:o + n])


@pytest.fixture(scope="module")
def stories():
    """The stories15M shape (288 dims, 6 layers, 6 heads, vocab 32000), N(0, 0.02) weights (seed 0) quantized by
    quantize()."""
    data = ck.synthetic_checkpoint(ck.STORIES15M, seed=0)
    return data, stories_plan(data)


def test_stories15m_greedy_identical(stories):
    """64 seeded prompt tokens, then 128 greedy tokens: the ids and every step's logits the oracle's to the bit
    (forward.js's float16 cache: stories15M is multi-head)."""
    data, plan = stories
    rng = np.random.default_rng(0)
    prompt = [1] + [int(t) for t in rng.integers(0, 32000, 63)]
    eng = Engine(data, plan)
    ref = oracle.OracleEngine(data, plan, threads=4)
    eng.forwardMany(prompt[:-1], 0)
    ref.forward_many(prompt[:-1], 0)
    logits = np.zeros(32000, np.float32)
    eng.bind(logits)
    token, ids, ref_ids = prompt[-1], [], []
    rtoken = token
    for pos in range(63, 63 + 128):
        eng.forward(token, pos)
        want = ref.forward(rtoken, pos)
        assert np.array_equal(bits(logits), bits(want)), pos
        token, rtoken = int(np.argmax(logits)), int(np.argmax(want))
        ids.append(token)
        ref_ids.append(rtoken)
    assert ids == ref_ids


def test_slots_are_independent(stories):
    """The batched extension: three sequences in one run, token by token and in prompt blocks, each bit-identical
    to the same sequence alone; generate_greedy on the device gives run()'s argmax ids."""
    data, plan = stories
    rng = np.random.default_rng(1)
    prompts = [[1] + [int(t) for t in rng.integers(0, 32000, n)] for n in (20, 33, 7)]
    alone = []
    for p in prompts:
        e = Engine(data, plan)
        e.forwardMany(p[:-1], 0)
        e.forward(p[-1], len(p) - 1)
        alone.append(e.logits())
        e.release()
    eng = Engine(data, plan, slots=3)
    # the prompts in one run (every slot's tokens in order), then the last tokens together
    slots = np.concatenate([[i] * (len(p) - 1) for i, p in enumerate(prompts)])
    toks = np.concatenate([p[:-1] for p in prompts])
    pos = np.concatenate([np.arange(len(p) - 1) for p in prompts])
    eng.run(slots, toks, pos)
    last, am = eng.run([0, 1, 2], [p[-1] for p in prompts], [len(p) - 1 for p in prompts], want=[1, 1, 1])
    for i in range(3):
        assert np.array_equal(bits(last[i]), bits(alone[i])), i
        assert am[i] == int(np.argmax(alone[i]))
    # 12 greedy steps on the device from there, against run() step by step on a second engine
    first = [int(a) for a in am]
    p0 = [len(p) for p in prompts]
    ids = eng.generate_greedy([0, 1, 2], first, p0, 12)
    other = Engine(data, plan, slots=3)
    other.run(slots, toks, pos)
    other.run([0, 1, 2], [p[-1] for p in prompts], [len(p) - 1 for p in prompts])
    cur, steps = list(first), []
    for s in range(12):
        _, am2 = other.run([0, 1, 2], cur, [p + s for p in p0], want=[1, 1, 1], logits=False)
        steps.append(list(am2))
        cur = [int(a) for a in am2]
    assert np.array_equal(ids, np.array(steps).T)


def test_errors_are_raised_not_crashed(stories):
    data, plan = stories
    eng = Engine(data, plan)
    with pytest.raises(abi.EngineError, match="vocabulary"):
        eng.forward(32000, 0)
    with pytest.raises(abi.EngineError, match="context"):
        eng.forward(5, 256)
    bad = dict(plan, dim=320)
    with pytest.raises(abi.EngineError):
        Engine(data, bad)


def test_not_finite_logits_stop_greedy(stories):
    """llama2_numpy.greedy's NOT_FINITE (public/llama2_numpy.py:1521-1527): a classifier whose scales are NaN
    gives logits that are no numbers; generate_greedy says so, and the engine is still usable."""
    data, plan = stories
    broken = bytearray(data)
    t = plan["tensors"]["token_embedding_table"]
    nan = np.full(32000 * 288 // 32, np.nan, np.float32).tobytes()
    broken[t["scales"]:t["scales"] + len(nan)] = nan
    eng = Engine(bytes(broken), plan)
    with pytest.raises(abi.EngineError) as err:
        eng.generate_greedy([0], [1], [0], 2)
    assert err.value.code == abi.ENOTFINITE
    eng.forward(1, 0)  # still answers


def test_time_matmuls_leaves_the_sequence_alone(stories):
    """b200fwd_time_matmuls (the bench's roofline leg) writes only scratch: a sequence continued after it gives the
    logits it gives without it, to the bit; one pass is every layer's four matmuls and the classifier."""
    data, plan = stories
    rng = np.random.default_rng(2)
    prompt = [1] + [int(t) for t in rng.integers(0, 32000, 40)]
    runs = []
    for timed in (False, True):
        eng = Engine(data, plan, slots=2)
        eng.run([0] * 40 + [1] * 40, prompt[:-1] * 2, list(range(40)) * 2)
        if timed:
            ms, nbytes, launches = eng.time_matmuls(32, reps=2)
            assert ms > 0 and launches == 4 * plan["n_layers"] + 1
            assert nbytes > plan["vocab_size"] * plan["dim"]
        last, _ = eng.run([0, 1], [prompt[-1]] * 2, [40, 40], want=[1, 1])
        runs.append(last)
        eng.release()
    assert np.array_equal(bits(runs[0]), bits(runs[1]))


def test_generate_drives_the_engine_like_the_reference():
    """The reference's generate() (public/llama2_numpy.py:1565-1671), unmodified, drove an oracle-backed engine to
    make generate_tiny_gqa.npz (tests/golden/make_golden.py): 54 prompt tokens in forwardMany blocks, then 66 greedy
    steps through forward(). The same loop over b200fwd.forward.external(...).start(plan) (this engine's promptBlock:
    one block) chooses the same 66 ids."""
    from test_oracle_golden import generate_like_the_reference

    data, plan, _ = golden_model("tiny_gqa")
    g = np.load(GOLDEN / "generate_tiny_gqa.npz")
    eng = external(data).start(plan)
    logits = np.zeros(plan["vocab_size"], np.float32)
    eng.bind(logits)
    eng.bound_logits = logits
    calls, chosen = generate_like_the_reference(eng, [int(t) for t in g["prompt"]], int(g["steps"]))
    assert chosen == [int(t) for t in g["ids"]]
    assert calls[0] == (0, [1] + [int(t) for t in g["prompt"][:-1]])  # the whole prompt in one block here
    eng.release()


def oracle_generate(data, plan, prompt, steps, temperature, topp, penalty, randoms, stops):
    """generate()'s sampling loop (public/llama2_numpy.py:1612-1650, with the kernel sampler of :1468-1512) on the
    oracle: forward, penalize over the last 64 tokens of the history, sample (or argmax), stop tokens."""
    ref = oracle.OracleEngine(data, plan, threads=2)
    ref.forward_many([1] + prompt[:-1], 0)
    history, token, pos, ids = [1] + prompt, prompt[-1], len(prompt), []
    while pos < steps:
        logits = ref.forward(token, pos)
        if penalty != 1.0:
            logits = oracle.penalize(logits, history[-64:], penalty)
        nxt = int(np.argmax(logits)) if temperature == 0 else oracle.sample(logits, temperature, topp,
                                                                            randoms[len(ids)])
        ids.append(nxt)
        if nxt in stops:
            break
        history.append(nxt)
        token, pos = nxt, pos + 1
    ref.close()
    return ids


def engine_generate(eng, prompt, steps, temperature, topp, penalty, randoms, stops):
    """generate()'s loop over an engine with generateMany (public/llama2_numpy.py:1612-1650): blocks of tokenBlock
    steps, a random number per step, the history's last 64 tokens and its length, stop tokens."""
    eng.forwardMany([1] + prompt[:-1], 0)
    history, token, pos, ids = [1] + prompt, prompt[-1], len(prompt), []
    while pos < steps:
        many = min(eng.tokenBlock, steps - pos)
        rs = list(randoms[len(ids):len(ids) + many]) if temperature != 0 else []
        chosen = eng.generateMany(token, pos, history[-64:], len(history), many, temperature, topp, penalty, rs,
                                  sorted(stops))
        ended = False
        for nxt in chosen:
            ids.append(nxt)
            if nxt in stops:
                ended = True
                break
            history.append(nxt)
            token, pos = nxt, pos + 1
        if ended:
            break
    return ids


@pytest.mark.parametrize("temperature,topp,penalty", [(0.0, 0.9, 1.3), (0.8, 0.9, 1.2), (1.0, 1.0, 1.0),
                                                      (0.6, 0.5, 1.0)])
def test_generate_many_is_generates_loop(temperature, topp, penalty):
    """generateMany on the device (b200fwd_generate_many: forward, penalize, sample or argmax, in one CUDA graph a
    step) gives the ids of generate()'s loop on the oracle with the same random numbers, to the id, over 70 steps in
    blocks of tokenBlock; then again with the 9th id made a stop token: the run ends there, that id last."""
    data, plan, _ = golden_model("tiny_gqa")
    rng = np.random.default_rng(4)
    prompt = [int(t) for t in rng.integers(3, 320, 20)]
    randoms = [float(v) for v in rng.random(80)]
    steps = len(prompt) + 70
    want = oracle_generate(data, plan, prompt, steps, temperature, topp, penalty, randoms, set())
    eng = Engine(data, plan)
    assert eng.tokenBlock > 0
    got = engine_generate(eng, prompt, steps, temperature, topp, penalty, randoms, set())
    eng.release()
    assert got == want
    stop = {want[8]}
    want2 = oracle_generate(data, plan, prompt, steps, temperature, topp, penalty, randoms, stop)
    eng = Engine(data, plan)
    got2 = engine_generate(eng, prompt, steps, temperature, topp, penalty, randoms, stop)
    eng.release()
    assert got2 == want2 and got2[-1] in stop and len(got2) <= 9


def test_generate_many_slots_are_independent():
    """Three slots sampled in one b200fwd_generate_many call give each slot's ids alone."""
    data, plan, _ = golden_model("tiny_gqa")
    rng = np.random.default_rng(6)
    prompts = [[1] + [int(t) for t in rng.integers(3, 320, n)] for n in (9, 17, 4)]
    randoms = rng.random((3, 12))
    alone = []
    for i, p in enumerate(prompts):
        e = Engine(data, plan)
        e.forwardMany(p[:-1], 0)
        alone.append(e.generateMany(p[-1], len(p) - 1, p[-64:], len(p), 12, 0.9, 0.9, 1.1, list(randoms[i]), []))
        e.release()
    eng = Engine(data, plan, slots=3)
    for i, p in enumerate(prompts):
        eng.run([i] * (len(p) - 1), p[:-1], list(range(len(p) - 1)))
    ids, made = eng.generate_many([0, 1, 2], [p[-1] for p in prompts], [len(p) - 1 for p in prompts], 12, 0.9, 0.9,
                                  1.1, [p for p in prompts], [len(p) for p in prompts], randoms, [])
    for i in range(3):
        assert list(ids[i][:made[i]]) == alone[i], i


@pytest.mark.parametrize("heads,kv_heads", [(4, 4), (4, 2), (8, 2), (8, 1)])
@pytest.mark.parametrize("half_keys", [True, False])
def test_prompt_blocks_of_wide_heads(heads, kv_heads, half_keys):
    """Prompt blocks of heads of 64 values (the register-blocked prompt attention: 1, 2, 4 and 8 query heads per kv
    head): three sequences' prompts of ragged lengths, run in two calls of several sequences each, so that tiles of
    up to 16 tokens read keys and values past three 64-position chunks and the last tile of a run is short; each
    sequence's last logits against the oracle's token-by-token forward, to the bit. Then four greedy steps of all
    three on the device (the single-token attention kernels, which quantize their rows themselves): the ids, and the
    second layer's keys and values at the new positions (they depend on the first layer's quantized attention rows),
    to the bit."""
    dim = 64 * heads
    header = (dim, 2 * dim, 2, heads, kv_heads, 320, 512)
    data = ck.synthetic_checkpoint(header, seed=heads * 10 + kv_heads, norm="normal")
    plan = ck.make_plan(header, lambda o, n: data[o:o + n])
    lengths = [150, 83, 211]
    rng = np.random.default_rng(heads + kv_heads)
    prompts = [rng.integers(0, 320, n).astype(np.int32) for n in lengths]
    eng = Engine(data, plan, half_keys=half_keys, slots=3, max_tokens=512, capacity=256)
    got = {}
    for lo, hi in ((0, 100), (100, 256)):
        slots, tokens, pos, want = [], [], [], []
        for s, p in enumerate(prompts):
            n = min(hi, len(p)) - lo
            if n <= 0:
                continue
            slots += [s] * n
            tokens += list(p[lo:lo + n])
            pos += list(range(lo, lo + n))
            want += [lo + i == len(p) - 1 for i in range(n)]
        logits, _ = eng.run(np.array(slots), np.array(tokens), np.array(pos), want=np.array(want))
        ends = [s for s, w in zip(slots, want) if w]
        for s, row in zip(ends, logits):
            got[s] = row.copy()
    steps = 4
    first = np.array([int(np.argmax(got[s])) for s in range(3)], np.int32)
    ids = eng.generate_greedy(np.arange(3, dtype=np.int32), first, np.array(lengths, np.int32), steps)
    kv = [eng.keysAndValues(len(p), steps, slot=s) for s, p in enumerate(prompts)]
    eng.release()
    for s, p in enumerate(prompts):
        ref = oracle.OracleEngine(data, plan, half_keys=1 if half_keys else 0, threads=2)
        ref.forward_many([int(t) for t in p[:-1]], 0)
        want = ref.forward(int(p[-1]), len(p) - 1)
        assert np.array_equal(bits(got[s]), bits(want)), s
        token = int(np.argmax(want))
        for i in range(steps):
            token = int(np.argmax(ref.forward(token, len(p) + i)))
            assert token == ids[s, i], (s, i)
        rk, rv = ref.keys_values(len(p), steps)
        ref.close()
        assert np.array_equal(bits(kv[s]["keys"]), bits(rk)) and np.array_equal(bits(kv[s]["values"]), bits(rv)), s
