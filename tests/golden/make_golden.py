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
Besides: quantize.npz (the reference's quantize() of a seeded matrix), rope.npz (its rope_tables()).
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


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py /path/to/pyodide-llm")
    main(sys.argv[1])
