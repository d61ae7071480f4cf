"""The C ABI of include/b200fwd.h as ctypes: the plan structs and the library loader.

The library is pyodide-llm_b200/b200fwd/libb200fwd.so, built in-tree by pyodide-llm_b200/build.py. Loading it is
the only way this package runs a forward pass: there is no CPU fallback, and a missing library raises.
"""
import ctypes
from pathlib import Path

HERE = Path(__file__).resolve().parent
LIBRARY = HERE / "libb200fwd.so"

TENSOR_ABSENT, TENSOR_INT8, TENSOR_F32, TENSOR_F16 = 0, 1, 2, 3
KINDS = {"int8": TENSOR_INT8, "f32": TENSOR_F32, "f16": TENSOR_F16}
MAX_OUTLIERS = 16

OK, EINVAL, ECUDA, ENOMEM, EUNSUPPORTED, ENOTFINITE, ETIMEOUT = 0, -1, -2, -3, -4, -5, -6


class Tensor(ctypes.Structure):
    _fields_ = [("kind", ctypes.c_int32), ("group", ctypes.c_int32), ("offset", ctypes.c_int64),
                ("scales", ctypes.c_int64), ("ndim", ctypes.c_int32), ("pad_", ctypes.c_int32),
                ("shape", ctypes.c_int64 * 4)]


TENSOR_FIELDS = ("token_embedding_table", "rms_att_weight", "wq", "wk", "wv", "wo", "rms_ffn_weight", "w1", "w2",
                 "w3", "rms_final_weight", "wcls")


class Plan(ctypes.Structure):
    _fields_ = ([(name, ctypes.c_int32) for name in ("dim", "hidden_dim", "n_layers", "n_heads", "n_kv_heads",
                                                      "head_size", "vocab_size", "seq_len", "rotary", "kv_start")]
                + [("rms_norm_eps", ctypes.c_float)]
                + [(name, ctypes.c_int32) for name in ("shared_classifier", "int8", "relaxed", "half_kv",
                                                        "n_outliers")]
                + [("outliers", ctypes.c_int32 * MAX_OUTLIERS)]
                + [(name, Tensor) for name in TENSOR_FIELDS]
                + [("freq_cis_real", ctypes.POINTER(ctypes.c_float)),
                   ("freq_cis_imag", ctypes.POINTER(ctypes.c_float))])


class Options(ctypes.Structure):
    _fields_ = [("half_keys", ctypes.c_int32), ("slots", ctypes.c_int32), ("device", ctypes.c_int32),
                ("max_tokens", ctypes.c_int32), ("capacity", ctypes.c_int32),
                ("checkpoint_on_device", ctypes.c_int32), ("reserved", ctypes.c_int32 * 6)]


class PlanError(ValueError):
    pass


def plan_struct(plan):
    """The plan dict of Llama.external_forward (public/llama2_numpy.py:1261-1270) as a Plan struct. Returns the
    struct and the arrays it points into (keep them alive while the struct is used)."""
    import numpy as np

    if plan.get("arch", "llama") != "llama":
        raise PlanError(f"This engine runs the llama arch only, not {plan.get('arch')!r}.")
    if not plan.get("int8"):
        raise PlanError("This engine runs int8 checkpoints on the int8 kernels only (plan.int8 is false).")
    form = plan.get("form") or {}
    if int(form.get("interval", 0) or 0) or int(form.get("hadamard", 0) or 0):
        raise PlanError("A Qwen3.5 form is not run by this engine.")
    tensors = plan["tensors"]
    for name in ("bq", "bk", "bv", "q_norm", "k_norm", "positions"):
        if name in tensors:
            raise PlanError(f"The tensor {name} (a Qwen2/Qwen3/GPT-2 form) is not run by this engine.")
    s = Plan()
    for name in ("dim", "hidden_dim", "n_layers", "n_heads", "n_kv_heads", "head_size", "vocab_size", "seq_len",
                 "rotary", "kv_start"):
        setattr(s, name, int(plan[name]))
    s.rms_norm_eps = float(plan.get("rms_norm_eps", 1e-5))
    s.shared_classifier = int(bool(plan["shared_classifier"]))
    s.int8 = int(bool(plan["int8"]))
    s.relaxed = int(bool(plan.get("relaxed", True)))
    s.half_kv = int(bool(plan.get("half_kv", False)))
    outliers = [int(c) for c in plan.get("outliers", [])]
    if len(outliers) > MAX_OUTLIERS:
        raise PlanError(f"More than {MAX_OUTLIERS} outlier channels.")
    s.n_outliers = len(outliers)
    for i, c in enumerate(outliers):
        s.outliers[i] = c
    for name in TENSOR_FIELDS:
        t = tensors.get(name)
        if name == "wcls" and plan["shared_classifier"]:
            t = tensors["token_embedding_table"]
        if t is None:
            raise PlanError(f"The plan has no tensor {name}.")
        ts = getattr(s, name)
        ts.kind = KINDS[t["kind"]]
        ts.group = int(t.get("group", 0) or 0)
        ts.offset = int(t["offset"])
        ts.scales = int(t.get("scales", 0) or 0)
        shape = list(t["shape"])
        ts.ndim = len(shape)
        for i, d in enumerate(shape):
            ts.shape[i] = int(d)
    derived = plan.get("derived", {})
    keep = []
    table = (int(plan["seq_len"]), int(plan["head_size"]) // 2)
    for field, name in (("freq_cis_real", "freq_cis_real"), ("freq_cis_imag", "freq_cis_imag")):
        raw = derived.get(name)
        if raw is None:
            raise PlanError(f"The plan has no derived {name} table.")
        arr = np.frombuffer(bytes(raw), dtype=np.float32) if not isinstance(raw, np.ndarray) else raw
        arr = np.ascontiguousarray(arr, dtype=np.float32).reshape(-1)
        if arr.size != table[0] * table[1]:
            raise PlanError(f"The derived {name} table has {arr.size} floats, not {table[0] * table[1]}.")
        keep.append(arr)
        setattr(s, field, arr.ctypes.data_as(ctypes.POINTER(ctypes.c_float)))
    return s, keep


_lib = None


def load():
    """The engine library, loaded once. Raises when it is not built: nothing else runs the forward pass."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIBRARY.exists():
        raise RuntimeError(f"{LIBRARY} is not built: run `python pyodide-llm_b200/build.py` (no CPU fallback).")
    lib = ctypes.CDLL(str(LIBRARY))
    P, I32, I64, U64 = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.c_uint64
    sig = {
        "b200fwd_create": (P, ctypes.c_size_t, ctypes.POINTER(Plan), ctypes.POINTER(Options), ctypes.POINTER(P)),
        "b200fwd_bind_logits": (P, P),
        "b200fwd_forward": (P, I32, I32, I32),
        "b200fwd_forward_many": (P, P, I32, I32),
        "b200fwd_prompt_block": (P, ctypes.POINTER(I32)),
        "b200fwd_keys_values": (P, I32, I32, I32, P, P),
        "b200fwd_logits": (P, P),
        "b200fwd_backend": (P, ctypes.c_char_p, ctypes.c_size_t),
        "b200fwd_memory_bytes": (P, ctypes.POINTER(U64)),
        "b200fwd_destroy": (P,),
        "b200fwd_last_error": (ctypes.c_char_p, ctypes.c_size_t),
        "b200fwd_abi_version": (),
        "b200fwd_run": (P, I32, P, P, P, P, P, P),
        "b200fwd_generate_greedy": (P, I32, P, P, P, I32, P),
        "b200fwd_reset_slot": (P, I32),
        "b200fwd_stream_of": (P, ctypes.POINTER(P)),
        "b200fwd_launch_count": (P, ctypes.POINTER(U64)),
        "b200fwd_time_matmuls": (P, I32, I32, ctypes.POINTER(ctypes.c_float), ctypes.POINTER(ctypes.c_double),
                                 ctypes.POINTER(I32)),
        "b200fwd_time_matmul_kinds": (P, I32, I32, ctypes.POINTER(ctypes.c_float), ctypes.POINTER(ctypes.c_double)),
        "b200k_quantize_x": (P, P, P, I32, I32, I32, I64, I64, I64, P),
        "b200k_int8_sums": (P, P, I64, P),
        "b200k_matmul_q8r": (P, P, P, P, P, P, I32, I32, I32, I32, I64, I64, I64, P),
        "b200k_matmul_q8": (P, P, P, P, P, I32, I32, I32, I32, I64, I64, I64, P),
        "b200k_matmul_q8s": (P, P, P, P, P, I64, I32, I32, I32, I64, I64, I64, P),
        "b200k_rmsnorm": (P, P, P, I32, ctypes.c_float, I32, I64, P),
        "b200k_rope": (P, P, P, I32, I32, I32, P),
        "b200k_attention": (P, P, P, P, P, I32, I32, I32, I32, I32, I32, I32, P),
        "b200k_attention_static": (P, P, P, P, I32, I32, I32, I32, I32, I32, I32, P),
        "b200k_to_f16": (P, P, I64, P),
        "b200k_from_f16": (P, P, I64, P),
        "b200k_swiglu": (P, P, P, I64, P),
        "b200k_add_inplace": (P, P, I64, P),
        "b200k_add_columns": (P, P, P, I32, I32, P),
        "b200k_argmax": (P, P, I32, P),
        "b200k_penalize": (P, P, I32, ctypes.c_float, P),
        "b200k_prefill_attention": (P, P, P, P, P, P, I32, I32, I32, I32, I32, P, P),
        "b200k_prefill_attention_scratch": (I32, I32, I32, I32, I32, ctypes.POINTER(U64)),
        "b200k_prefill_attention_check": (P, I32, I32, I32, I32, I32, P),
        "b200k_sample": (P, P, I32, ctypes.c_float, ctypes.c_float, ctypes.c_double, P, P),
        "b200k_sample_scratch": (I32, ctypes.POINTER(U64)),
        "b200fwd_generate_many": (P, I32, P, P, P, I32, ctypes.c_float, ctypes.c_float, ctypes.c_float, P, P, P, P,
                                  I32, P, P),
        "b200k_attention_batch": (P, P, P, P, P, P, P, I32, I64, I32, I32, I32, I32, I32, P),
        "b200k_matmul_plan": (I32, I32, I32, I32, I32, P, P),
    }
    for name, args in sig.items():
        fn = getattr(lib, name)
        fn.argtypes = list(args)
        fn.restype = ctypes.c_int
    _lib = lib
    return lib


def last_error():
    lib = load()
    buf = ctypes.create_string_buffer(4096)
    lib.b200fwd_last_error(buf, len(buf))
    return buf.value.decode("utf-8", "replace")


class EngineError(RuntimeError):
    def __init__(self, code, message):
        super().__init__(message)
        self.code = code


def check(rc, what=""):
    """Raise the library's message for a non-zero status (forward.js throws an Error with its message)."""
    if rc != OK:
        raise EngineError(rc, f"{what}: {last_error()}" if what else last_error())
    return rc


def exported_symbols():
    """The function names include/b200fwd.h declares (read from the header, for the export check)."""
    import re

    header = (HERE.parent.parent / "include" / "b200fwd.h").read_text()
    return sorted(set(re.findall(r"^int (b200(?:fwd|k)_\w+)\(", header, flags=re.M)))
