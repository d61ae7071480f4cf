"""TEST INFRASTRUCTURE: ctypes bindings of oracle/liboracle.so, the C++ restatement of the reference's CPU path
(kernels/kernel.ts, kernels/kernel_relaxed.ts, public/forward.js run()). Only tests/, __graft_entry__.smoke() and
bench.py's CPU baseline use it, as the checker; the product path never does.

Parity pins: tests/test_oracle_golden.py holds these functions to the reference's own bit-exact formula checks
(tests/forward-check.mjs:119-276, tests/attention-check.mjs) and to fixtures made from the reference's Python
(tests/golden/make_golden.py).
"""
import ctypes
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent / "pyodide-llm_b200"))

from b200fwd.abi import Plan, plan_struct  # noqa: E402

_lib = None
_native = False


def use_native():
    """Load the oracle built on and for this host's CPU (-march=native; built now, before the first call): the
    timed CPU baseline. Same numbers as the portable build."""
    global _native
    if _lib is not None and not _native:
        raise RuntimeError("the portable oracle is already loaded in this process")
    _native = True


def load():
    global _lib
    if _lib is None:
        sys.path.insert(0, str(HERE))
        from build_oracle import build

        path = build(native=_native)
        lib = ctypes.CDLL(str(path))
        P, I32, I64 = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64
        sigs = {
            "oracle_quantize_x": ((P, P, P, I32, I32), None),
            "oracle_int8_sums": ((P, P, I64), None),
            "oracle_matmul_q8": ((P, P, P, P, P, I32, I32, I32), None),
            "oracle_matmul_q8r": ((P, P, P, P, P, P, I32, I32, I32), None),
            "oracle_matmul_q8r_tile": ((P, P, P, P, P, P, I32, I32, I32, I32, I64, I64, I64), None),
            "oracle_matmul_f32": ((P, P, P, I32, I32, I32), None),
            "oracle_rmsnorm": ((P, P, P, I32, ctypes.c_float), None),
            "oracle_rope": ((P, P, P, I32, I32, I32), None),
            "oracle_attention": ((P, P, P, P, P, I32, I32, I32, I32, I32, I32, I32), None),
            "oracle_to_f16": ((P, P, I64), None),
            "oracle_from_f16": ((P, P, I64), None),
            "oracle_swiglu": ((P, P, P, I64), None),
            "oracle_add_columns": ((P, P, P, I32, I32), None),
            "oracle_add_inplace": ((P, P, I64), None),
            "oracle_argmax": ((P, I32), ctypes.c_int),
            "oracle_penalize": ((P, P, I32, ctypes.c_float), None),
            "oracle_sample": ((P, I32, ctypes.c_float, ctypes.c_float, ctypes.c_double, P, P), ctypes.c_int),
            "oracle_fexp": ((ctypes.c_float,), ctypes.c_float),
            "oracle_vexp": ((ctypes.c_float,), ctypes.c_float),
            "oracle_create": ((P, ctypes.c_size_t, ctypes.POINTER(Plan), I32, I32), P),
            "oracle_destroy": ((P,), None),
            "oracle_half_kv": ((P,), ctypes.c_int),
            "oracle_forward": ((P, I32, I32, I32, P), ctypes.c_int),
            "oracle_forward_many": ((P, P, I32, I32), ctypes.c_int),
            "oracle_keys_values": ((P, I32, I32, P, P), ctypes.c_int),
            "oracle_threads": ((P,), ctypes.c_int),
        }
        for name, (args, res) in sigs.items():
            fn = getattr(lib, name)
            fn.argtypes = list(args)
            fn.restype = res
        _lib = lib
    return _lib


def _p(a):
    return a.ctypes.data_as(ctypes.c_void_p)


# ---- the kernels, on NumPy arrays (each returns its outputs)
def quantize_x(x, bias):
    x = np.ascontiguousarray(x, dtype=np.float32)
    n = x.size
    xq, xs = np.zeros(n, np.int8), np.zeros(n // 32, np.float32)
    load().oracle_quantize_x(_p(xq), _p(xs), _p(x), n, bias)
    return xq, xs


def int8_sums(w):
    w = np.ascontiguousarray(w, dtype=np.int8).reshape(-1)
    out = np.zeros(w.size // 32, np.int32)
    load().oracle_int8_sums(_p(out), _p(w), out.size)
    return out


def matmul_q8r(xq, xs, wq, ws, wc, n, r0=0, r1=None, out=None):
    rows = wq.size // n
    r1 = rows if r1 is None else r1
    out = np.full(rows, -7.0, np.float32) if out is None else out
    load().oracle_matmul_q8r(_p(out), _p(xq), _p(xs), _p(wq), _p(ws), _p(wc), n, r0, r1)
    return out


def matmul_q8(xq, xs, wq, ws, n, r0=0, r1=None, out=None):
    rows = wq.size // n
    r1 = rows if r1 is None else r1
    out = np.full(rows, -7.0, np.float32) if out is None else out
    load().oracle_matmul_q8(_p(out), _p(xq), _p(xs), _p(wq), _p(ws), n, r0, r1)
    return out


def matmul_q8r_tile(xq, xs, wq, ws, wc, n, r0, r1, count, out):
    """xq [count][n] int8, xs [count][n/32], out [count][rows] (token rows contiguous)."""
    rows = out.shape[1]
    load().oracle_matmul_q8r_tile(_p(out), _p(xq), _p(xs), _p(wq), _p(ws), _p(wc), n, r0, r1, count, rows,
                                  xq.shape[1], xs.shape[1])
    return out


def rmsnorm(x, w, eps=1e-5):
    x = np.ascontiguousarray(x, np.float32)
    out = np.zeros_like(x)
    load().oracle_rmsnorm(_p(out), _p(x), _p(np.ascontiguousarray(w, np.float32)), x.size, eps)
    return out


def rope(v, fcr, fci, nh, hs, rot=0):
    v = np.array(v, dtype=np.float32)
    load().oracle_rope(_p(v), _p(np.ascontiguousarray(fcr, np.float32)), _p(np.ascontiguousarray(fci, np.float32)),
                       nh, hs, rot)
    return v


def attention(q, kc, vc, pos, nh, nkv, hs, h0=0, h1=None, half=False):
    h1 = nh if h1 is None else h1
    out = np.full(nh * hs, np.nan, np.float32)
    att = np.zeros(nh * (pos + 1), np.float32)
    load().oracle_attention(_p(out), _p(np.ascontiguousarray(q, np.float32)), _p(kc), _p(vc), _p(att), pos, nh, nkv,
                            hs, h0, h1, 1 if half else 0)
    return out, att


def to_f16(x):
    x = np.ascontiguousarray(x, np.float32)
    out = np.zeros(x.size, np.uint16)
    load().oracle_to_f16(_p(out), _p(x), x.size)
    return out


def from_f16(h):
    h = np.ascontiguousarray(h, np.uint16)
    out = np.zeros(h.size, np.float32)
    load().oracle_from_f16(_p(out), _p(h), h.size)
    return out


def swiglu(h1, h3):
    h1, h3 = np.ascontiguousarray(h1, np.float32), np.ascontiguousarray(h3, np.float32)
    out = np.zeros_like(h1)
    load().oracle_swiglu(_p(out), _p(h1), _p(h3), h1.size)
    return out


def add_columns(y, rows, a):
    y = np.array(y, dtype=np.float32)
    rows, a = np.ascontiguousarray(rows, np.float32), np.ascontiguousarray(a, np.float32)
    load().oracle_add_columns(_p(y), _p(rows), _p(a), a.size, y.size)
    return y


def argmax(x):
    x = np.ascontiguousarray(x, np.float32)
    return load().oracle_argmax(_p(x), x.size)


def penalize(logits, tokens, penalty):
    """kernel.ts:705-719 on a copy of logits"""
    out = np.array(logits, dtype=np.float32)
    t = np.ascontiguousarray(tokens, np.int32)
    load().oracle_penalize(_p(out), _p(t), t.size, float(penalty))
    return out


def sample(logits, temperature, topp, random):
    """kernel.ts:808-868: the token drawn with `random` in [0, 1), -1 for logits whose largest is not finite"""
    x = np.ascontiguousarray(logits, np.float32)
    probs, index = np.zeros(x.size, np.float32), np.zeros(x.size, np.int32)
    return int(load().oracle_sample(_p(x), x.size, float(temperature), float(topp), float(random), _p(probs),
                                    _p(index)))


def fexp(x):
    return np.float32(load().oracle_fexp(float(x)))


def vexp(x):
    return np.float32(load().oracle_vexp(float(x)))


class OracleEngine:
    """The oracle's forward.js engine on one sequence: forward(), forward_many(), keys_values()."""

    def __init__(self, checkpoint, plan, half_keys=-1, threads=1):
        self._ckpt = np.frombuffer(bytes(checkpoint), dtype=np.uint8) if not isinstance(checkpoint, np.ndarray) \
            else np.ascontiguousarray(checkpoint).view(np.uint8)
        self._plan, self._keep = plan_struct(plan)
        self.vocab = int(plan["vocab_size"])
        self.layers, self.kv_dim = int(plan["n_layers"]), int(plan["n_kv_heads"]) * int(plan["head_size"])
        self._h = load().oracle_create(_p(self._ckpt), self._ckpt.size, ctypes.byref(self._plan), half_keys, threads)
        if not self._h:
            raise RuntimeError("oracle_create failed")
        self.half_kv = bool(load().oracle_half_kv(self._h))

    def forward(self, token, pos, need_logits=True):
        logits = np.zeros(self.vocab, np.float32)
        rc = load().oracle_forward(self._h, int(token), int(pos), 1 if need_logits else 0, _p(logits))
        if rc:
            raise RuntimeError("oracle_forward failed")
        return logits if need_logits else None

    def forward_many(self, tokens, pos):
        t = np.ascontiguousarray(tokens, np.int32)
        if load().oracle_forward_many(self._h, _p(t), t.size, int(pos)):
            raise RuntimeError("oracle_forward_many failed")

    def keys_values(self, start, count):
        k = np.zeros((self.layers, count, self.kv_dim), np.float32)
        v = np.zeros_like(k)
        if load().oracle_keys_values(self._h, start, count, _p(k), _p(v)):
            raise RuntimeError("oracle_keys_values failed")
        return k, v

    def close(self):
        if self._h:
            load().oracle_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
