"""Makes the golden fixtures of tests/golden/ from the reference's own Python (public/llama2_numpy.py,
public/llama2_convert.py), which runs in a container that has the reference checked out:

    python tests/golden/make_golden.py /path/to/pyodide-llm

For each model of MODELS (a seeded int8 checkpoint from b200fwd.checkpoint.synthetic_checkpoint, whose sha256 is
recorded so that the tests can make it again without the reference):
  - plan_<name>.json / .npz: the plan `Llama(None, tokenizer, dtype="int8", external=...)` hands to
    external.start(plan) (public/llama2_numpy.py:1248-1270), captured by a stand-in external;
  - numpy_<name>.npz: the reference NumPy engine's logits (`Llama.forward`, public/llama2_numpy.py:1310-1465) on
    its own greedy text from BOS, at POSITIONS positions: forward.js is held to these by the line of
    tests/forward-check.mjs:2-9,437 (the most likely token the same at >= 85% of positions, perplexity within 5%).
Besides: quantize.npz (the reference's quantize() of a seeded matrix), rope.npz (its rope_tables()), and
generate_tiny_gqa.npz: the unmodified `Llama(None, tokenizer, dtype="int8", external=...).generate(prompt,
temperature=0)` (public/llama2_numpy.py:1565-1671) driving a stand-in engine that serves forward.js's members from the
oracle (OracleExternal below): the prompt's token ids, every block and token it fed the engine (forwardMany blocks of
promptBlock, then forward), and the ids its greedy sampling chose.
"""
import hashlib
import json
import struct
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO / "pyodide-llm_b200"))

from b200fwd import checkpoint as ck  # noqa: E402

# name: (header, seed, norm, positions)
MODELS = {
    # GQA, a hidden width of 5 groups (one group past the fours), outlier channels from N(0, 0.02) norm weights
    "tiny_gqa": ((64, 160, 2, 4, 2, 320, 160), 0, "normal", 128),
    # MHA, unshared classifier, norm weights 1.0
    "tiny_mha": ((96, 224, 3, 3, 3, -320, 160), 1, "ones", 128),
    # MQA
    "tiny_mqa": ((64, 128, 2, 2, 1, 320, 160), 2, "ones", 128),
}


def tokenizer_bin(vocab):
    """A llama2.c tokenizer.bin of `vocab` pieces (the format of public/llama2_numpy.py:950-967)."""
    pieces = [b"<unk>", b"<s>", b"</s>"] + [b"<0x%02X>" % b for b in range(256)]
    while len(pieces) < vocab:
        pieces.append(b"p%d" % len(pieces))
    out = [struct.pack("<i", max(len(p) for p in pieces))]
    out += [struct.pack("<fi", -1e9 if i < 259 else -float(i), len(p)) + p for i, p in enumerate(pieces[:vocab])]
    return b"".join(out)


class Capture:
    """A stand-in for forward.js's external(): size, read(), and start(plan), which keeps the plan."""

    def __init__(self, data):
        self.data, self.size, self.plan = data, len(data), None

    def read(self, offset, length):
        return self.data[offset:offset + length]

    def start(self, plan):
        self.plan = plan

        class Stub:
            backend = "capture"

            def bind(self, array):
                pass

            def forward(self, token, pos, need_logits=True):
                pass

        return Stub()


class OracleExternal:
    """TEST INFRASTRUCTURE: forward.js's external() (public/forward.js:571-590) whose engine answers from the oracle
    (oracle/oracle.py: the C++ restatement of forward.js run()), recording every call the caller makes."""

    def __init__(self, data, prompt_block=16):
        self.data, self.size, self.prompt_block, self.fed = data, len(data), prompt_block, []

    def read(self, offset, length):
        return self.data[offset:offset + length]

    def start(self, plan):
        sys.path.insert(0, str(REPO / "oracle"))
        import oracle

        outer = self

        class Engine:
            backend = "oracle (test stand-in)"
            promptBlock = outer.prompt_block

            def __init__(self):
                self.ref = oracle.OracleEngine(outer.data, plan, half_keys=-1, threads=2)
                self.logits = None

            def bind(self, array):
                self.logits = array

            def forward(self, token, pos, needLogits=True):
                outer.fed.append((int(pos), [int(token)], bool(needLogits)))
                out = self.ref.forward(int(token), int(pos), needLogits)
                if needLogits:
                    self.logits[:] = out

            def forwardMany(self, tokens, pos):
                outer.fed.append((int(pos), [int(t) for t in tokens], False))
                self.ref.forward_many(list(tokens), int(pos))

        return Engine()


PROMPT = "Once upon a time, there was a little girl named Lily."
GENERATE_STEPS = 120


def generate_fixture(llama2_numpy, name="tiny_gqa"):
    header, seed, norm, _ = MODELS[name]
    data = ck.synthetic_checkpoint(header, seed=seed, norm=norm)
    ext = OracleExternal(data)
    model = llama2_numpy.Llama(None, tokenizer_bin(abs(header[5])), dtype="int8", external=ext)
    chosen = []
    sample = model.sample

    def recording(logits, temperature, topp, rng):
        token = sample(logits, temperature, topp, rng)
        chosen.append(int(token))
        return token

    model.sample = recording
    text = "".join(model.generate(PROMPT, steps=GENERATE_STEPS, temperature=0.0))
    prompt = model.tokenizer.encode(PROMPT, model.specials)
    fed_pos = np.array([p + i for p, toks, _ in ext.fed for i in range(len(toks))], np.int32)
    fed_tok = np.array([t for _, toks, _ in ext.fed for t in toks], np.int32)
    fed_call = np.array([i for i, (_, toks, _) in enumerate(ext.fed) for _ in toks], np.int32)
    np.savez_compressed(HERE / f"generate_{name}.npz", prompt=np.array(prompt, np.int32), ids=np.array(chosen, np.int32),
                        steps=np.array(GENERATE_STEPS), prompt_block=np.array(ext.prompt_block), fed_pos=fed_pos,
                        fed_tok=fed_tok, fed_call=fed_call, sha256=np.frombuffer(hashlib.sha256(data).digest(), np.uint8))
    print(name, "generate:", len(prompt), "prompt tokens,", len(chosen), "chosen,", len(ext.fed), "engine calls,",
          len(text), "characters")


class Drawn:
    """A generator whose random() gives the numbers it was made with, in order (so that a test can give the same)."""

    def __init__(self, numbers):
        self.numbers = list(numbers)

    def random(self):
        return self.numbers.pop(0)


def sample_fixture(llama2_numpy):
    """sample.npz: the reference's NumPy sampler (Llama.sample and Llama.penalize, public/llama2_numpy.py:1529-1563,
    1514-1518) on seeded logits at several temperatures and top-p values, with the random numbers it drew."""
    rng = np.random.default_rng(17)
    logits, temps, topps, randoms, chosen, penalized, histories = [], [], [], [], [], [], []
    for case in range(48):
        vocab = 1000
        x = (rng.standard_normal(vocab) * rng.choice([0.3, 1.0, 3.0, 8.0])).astype(np.float32)
        t = float(rng.choice([0.3, 0.7, 1.0, 1.6]))
        p = float(rng.choice([0.5, 0.9, 0.95, 1.0]))
        history = [int(v) for v in rng.integers(0, vocab, 80)]
        pen = x.copy()
        llama2_numpy.Llama.penalize(None, pen, history, 1.3)
        for _ in range(8):
            r = float(rng.random())
            token = llama2_numpy.Llama.sample(None, pen.copy(), t, p, Drawn([r]))
            logits.append(x)
            temps.append(t)
            topps.append(p)
            randoms.append(r)
            chosen.append(token)
            penalized.append(pen)
            histories.append(history)
    np.savez_compressed(HERE / "sample.npz", logits=np.stack(logits), temperature=np.array(temps, np.float32),
                        topp=np.array(topps, np.float32), random=np.array(randoms), chosen=np.array(chosen, np.int32),
                        penalized=np.stack(penalized), history=np.array(histories, np.int32))
    print("sample:", len(chosen), "draws")


def main(reference):
    sys.path.insert(0, str(Path(reference) / "public"))
    import llama2_convert
    import llama2_numpy

    for name, (header, seed, norm, positions) in MODELS.items():
        data = ck.synthetic_checkpoint(header, seed=seed, norm=norm)
        vocab = abs(header[5])
        tok = tokenizer_bin(vocab)
        capture = Capture(data)
        llama2_numpy.Llama(None, tok, dtype="int8", external=capture)
        plan = capture.plan
        derived = {k: np.frombuffer(v, dtype=np.float32) for k, v in plan["derived"].items()}
        meta = {k: v for k, v in plan.items() if k != "derived"}
        (HERE / f"plan_{name}.json").write_text(json.dumps(meta, indent=1, sort_keys=True))
        np.savez_compressed(HERE / f"plan_{name}.npz", **derived)
        model = llama2_numpy.Llama(data, tok, dtype="int8")
        token, tokens, logits = llama2_numpy.BOS, [], []
        for pos in range(positions):
            out = np.array(model.forward(token, pos), dtype=np.float32)
            logits.append(out)
            tokens.append(token)
            token = int(np.argmax(out))
        np.savez_compressed(HERE / f"numpy_{name}.npz", tokens=np.array(tokens, np.int32),
                            logits=np.stack(logits), header=np.array(header, np.int32),
                            sha256=np.frombuffer(hashlib.sha256(data).digest(), np.uint8),
                            seed=np.array(seed), norm=np.array(norm))
        print(name, "plan outliers", plan["outliers"], "positions", positions)
    rng = np.random.default_rng(5)
    values = (rng.standard_normal((37, 96)) * 0.02).astype(np.float32)
    values[3, :32] = 0  # a group of zeros: scale 0, inverse 0
    q, s = llama2_convert.quantize(values)
    np.savez_compressed(HERE / "quantize.npz", values=values, q=q, s=s)
    cos, sin = llama2_numpy.rope_tables(300, 48, 10000.0)
    cos8, sin8 = llama2_numpy.rope_tables(64, 128, 500000.0)
    np.savez_compressed(HERE / "rope.npz", cos=cos.astype(np.float32), sin=sin.astype(np.float32),
                        cos8b=cos8.astype(np.float32), sin8b=sin8.astype(np.float32))
    generate_fixture(llama2_numpy)
    sample_fixture(llama2_numpy)


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py /path/to/pyodide-llm")
    main(sys.argv[1])
