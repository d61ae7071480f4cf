"""The engine interface of public/forward.js over the C ABI of include/b200fwd.h.

`external(checkpoint)` is what forward.js's `external({memory, base, size, kernels, ...})` is to
`llama2_numpy.Llama(None, tokenizer, external=...)` (public/forward.js:571-590): `size`, `read(offset, length)` and
`start(plan)`, which returns the engine. The engine has forward.js's members (public/forward.js:1676-1955) under the
same names — backend, bind, forward, forwardMany, promptBlock, tokenBlock, release, logits, keysAndValues,
memoryBytes — so the unmodified Python model code drives it. It adds the batched members of the B200 build (run,
generate_greedy) for many independent sequences.

Errors are raised as EngineError with the library's message (forward.js throws an Error). There is no CPU path.
"""
import ctypes

import numpy as np

from . import abi


def _p(a):
    return ctypes.c_void_p(a.ctypes.data) if a is not None else None


class Engine:
    """forward.js's engine (createForward's return value) on one B200."""

    def __init__(self, checkpoint, plan, half_keys=None, slots=1, device=0, max_tokens=0, capacity=0,
                 checkpoint_on_device=False, size=None):
        lib = abi.load()
        self._lib = lib
        self._plan_struct, self._keep = abi.plan_struct(plan)
        opts = abi.Options()
        opts.half_keys = -1 if half_keys is None else int(bool(half_keys))
        opts.slots = int(slots)
        opts.device = int(device)
        opts.max_tokens = int(max_tokens)
        opts.capacity = int(capacity)
        opts.checkpoint_on_device = int(bool(checkpoint_on_device))
        if checkpoint_on_device:
            ptr, nbytes = int(checkpoint), int(size)
        else:
            buf = checkpoint if isinstance(checkpoint, np.ndarray) else np.frombuffer(memoryview(checkpoint), np.uint8)
            buf = np.ascontiguousarray(buf).view(np.uint8).reshape(-1)
            self._ckpt_host = buf  # only needed during create; dropped below
            ptr, nbytes = buf.ctypes.data, buf.size
        handle = ctypes.c_void_p()
        abi.check(lib.b200fwd_create(ctypes.c_void_p(ptr), nbytes, ctypes.byref(self._plan_struct), ctypes.byref(opts),
                                     ctypes.byref(handle)), "create")
        self._h = handle
        self._ckpt_host = None
        self.vocab_size = int(plan["vocab_size"])
        self.n_layers = int(plan["n_layers"])
        self.kv_dim = int(plan["n_kv_heads"]) * int(plan["head_size"])
        self.slots = int(slots)
        self._bound = None
        buf = ctypes.create_string_buffer(512)
        abi.check(lib.b200fwd_backend(self._h, buf, len(buf)), "backend")
        self.backend = buf.value.decode()
        pb = ctypes.c_int32()
        abi.check(lib.b200fwd_prompt_block(self._h, ctypes.byref(pb)), "promptBlock")
        self._prompt_block = pb.value

    # ---- forward.js's members
    def bind(self, array):
        """forward.js:1745-1748: the float32 array forward() fills with the logits."""
        if not (isinstance(array, np.ndarray) and array.dtype == np.float32 and array.flags.c_contiguous
                and array.size >= self.vocab_size):
            raise ValueError("bind() takes a contiguous float32 array of vocab_size values")
        self._bound = array
        abi.check(self._lib.b200fwd_bind_logits(self._h, ctypes.c_void_p(array.ctypes.data)), "bind")

    def forward(self, token, pos, needLogits=True):
        """forward.js:1891-1912"""
        abi.check(self._lib.b200fwd_forward(self._h, int(token), int(pos), 1 if needLogits else 0), "forward")

    def forwardMany(self, tokens, pos):
        """forward.js:1755-1769: a prompt's tokens at pos, pos + 1, ..., no logits"""
        t = np.ascontiguousarray(np.asarray(list(tokens), dtype=np.int32))
        abi.check(self._lib.b200fwd_forward_many(self._h, _p(t), t.size, int(pos)), "forwardMany")

    @property
    def promptBlock(self):
        """forward.js:1773-1778: how many prompt tokens Python hands forwardMany at once"""
        return self._prompt_block

    TOKEN_BLOCK = 16
    REPETITION_WINDOW = 64  # public/llama2_numpy.py:545

    @property
    def tokenBlock(self):
        """forward.js:1837-1840: how many steps generate() hands generateMany at once (public/llama2_numpy.py:1612-1620)"""
        return self.TOKEN_BLOCK

    def generateMany(self, token, pos, history, length, count, temperature, topp, penalty, randoms, stops):
        """forward.js:1830-1890 generateMany: count steps of generate() from token at pos on the device (slot 0): the
        forward pass, the repetition penalty over the last 64 tokens of the history (the last of `history`, whose
        whole length is `length`), then greedy argmax (temperature 0) or kernel.ts's sample with one of `randoms` a
        step. Returns the ids (a stop token last where one came); their keys and values are in the cache as forward()
        would have written them."""
        ids, made = self.generate_many([0], [token], [pos], count, temperature, topp, penalty, [list(history)],
                                       [length], [list(randoms)] if temperature != 0 else None, list(stops))
        return [int(t) for t in ids[0][:made[0]]]

    def generate_many(self, slots, first, pos0, steps, temperature, topp, penalty, histories, lengths, randoms,
                      stops):
        """generateMany for several slots at once: returns (ids [n][steps], made [n])."""
        n, W = len(slots), self.REPETITION_WINDOW
        recent = np.zeros((n, W), np.int32)
        for i, h in enumerate(histories):
            last = list(h)[-min(int(lengths[i]), W):] if lengths[i] else []
            recent[i, :len(last)] = last
        r = None
        if temperature != 0:
            r = np.zeros((n, steps), np.float64)
            for i, row in enumerate(randoms):
                row = list(row)[:steps]
                r[i, :len(row)] = row
        st = np.ascontiguousarray(stops, np.int32)
        # (the arrays are held in locals until the call returns: the library reads them through bare pointers)
        sl, fi = np.ascontiguousarray(slots, np.int32), np.ascontiguousarray(first, np.int32)
        po, le = np.ascontiguousarray(pos0, np.int32), np.ascontiguousarray(lengths, np.int32)
        out, made = np.zeros((n, steps), np.int32), np.zeros(n, np.int32)
        abi.check(self._lib.b200fwd_generate_many(
            self._h, n, _p(sl), _p(fi), _p(po), int(steps), float(temperature), float(topp), float(penalty),
            _p(recent), _p(le), _p(r), _p(st) if st.size else None, st.size, _p(out), _p(made)), "generateMany")
        return out, made

    def release(self):
        """forward.js:1915-1934"""
        if getattr(self, "_h", None):
            self._lib.b200fwd_destroy(self._h)
            self._h = None
        self._bound = None
        return True

    def logits(self):
        """forward.js:1936"""
        out = np.zeros(self.vocab_size, np.float32)
        abi.check(self._lib.b200fwd_logits(self._h, _p(out)), "logits")
        return out

    def keysAndValues(self, start, count, slot=0):
        """forward.js:1939-1953: {keys, values}, float32 [layers][count][kvDim] each"""
        k = np.zeros((self.n_layers, count, self.kv_dim), np.float32)
        v = np.zeros_like(k)
        abi.check(self._lib.b200fwd_keys_values(self._h, int(slot), int(start), int(count), _p(k), _p(v)),
                  "keysAndValues")
        return {"keys": k, "values": v}

    def memoryBytes(self):
        out = ctypes.c_uint64()
        abi.check(self._lib.b200fwd_memory_bytes(self._h, ctypes.byref(out)), "memoryBytes")
        return out.value

    # ---- the batched extension
    def run(self, slots, tokens, pos, want=None, logits=True):
        """n tokens of any slots at their positions; returns (logits [W][vocab] or None, argmax [W]) of the
        tokens with want[i] (default: none)."""
        slots = np.ascontiguousarray(slots, np.int32)
        tokens = np.ascontiguousarray(tokens, np.int32)
        pos = np.ascontiguousarray(pos, np.int32)
        n = tokens.size
        w = None if want is None else np.ascontiguousarray(np.asarray(want, dtype=bool).astype(np.uint8))
        W = 0 if w is None else int(w.sum())
        out = np.zeros((W, self.vocab_size), np.float32) if (W and logits) else None
        am = np.zeros(W, np.int32) if W else None
        abi.check(self._lib.b200fwd_run(self._h, n, _p(slots), _p(tokens), _p(pos), _p(w), _p(out), _p(am)), "run")
        return out, am

    def generate_greedy(self, slots, first, pos0, steps):
        """steps greedy steps of each slot on the device; returns the ids [n][steps]."""
        slots = np.ascontiguousarray(slots, np.int32)
        first = np.ascontiguousarray(first, np.int32)
        pos0 = np.ascontiguousarray(pos0, np.int32)
        out = np.zeros((slots.size, steps), np.int32)
        abi.check(self._lib.b200fwd_generate_greedy(self._h, slots.size, _p(slots), _p(first), _p(pos0), int(steps),
                                                    _p(out)), "generate_greedy")
        return out

    def launch_count(self):
        out = ctypes.c_uint64()
        abi.check(self._lib.b200fwd_launch_count(self._h, ctypes.byref(out)), "launch_count")
        return out.value

    def time_matmuls(self, count, reps=3):
        """(ms, bytes, launches) of one pass of every matmul at `count` tokens (b200fwd_time_matmuls)."""
        ms, nbytes, launches = ctypes.c_float(), ctypes.c_double(), ctypes.c_int32()
        abi.check(self._lib.b200fwd_time_matmuls(self._h, count, reps, ctypes.byref(ms), ctypes.byref(nbytes),
                                                 ctypes.byref(launches)), "time_matmuls")
        return ms.value, nbytes.value, launches.value

    KINDS = ("qkv", "o", "w13", "w2", "classifier")

    def time_matmul_kinds(self, count, reps=3):
        """{kind: (us per launch, algorithmic bytes per launch)} of each weight-matrix kind at `count` tokens, every
        layer's copy in turn (b200fwd_time_matmul_kinds)."""
        us, nbytes = (ctypes.c_float * 5)(), (ctypes.c_double * 5)()
        abi.check(self._lib.b200fwd_time_matmul_kinds(self._h, count, reps, us, nbytes), "time_matmul_kinds")
        return {k: (us[i], nbytes[i]) for i, k in enumerate(self.KINDS)}

    def stream(self):
        out = ctypes.c_void_p()
        abi.check(self._lib.b200fwd_stream_of(self._h, ctypes.byref(out)), "stream")
        return out.value or 0

    # snake_case names for Python callers
    forward_many = forwardMany
    keys_and_values = keysAndValues
    memory_bytes = memoryBytes

    def __del__(self):
        try:
            self.release()
        except Exception:
            pass


class External:
    """forward.js's external() (public/forward.js:571-590): size, read(offset, length), start(plan)."""

    def __init__(self, checkpoint, **options):
        self._data = checkpoint if isinstance(checkpoint, (bytes, bytearray)) else bytes(checkpoint)
        self.size = len(self._data)
        self.options = options
        self.engine = None

    def read(self, offset, length):
        return self._data[offset:offset + length]

    def start(self, plan):
        self.engine = Engine(self._data, plan, **self.options)
        return self.engine


def external(checkpoint, **options):
    """What Llama(None, tokenizer, external=...) takes. options: half_keys, slots, device, max_tokens, capacity."""
    return External(checkpoint, **options)
