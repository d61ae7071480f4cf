"""The C ABI without a GPU: the library loads, exports every function include/b200fwd.h declares, and the plan
checks of the host side refuse what the engine does not run. No compute call (there is no GPU here)."""
import ctypes
import json

import numpy as np
import pytest

from b200fwd import abi, checkpoint as ck
from conftest import GOLDEN, ROOT


@pytest.fixture(scope="module")
def lib():
    import sys

    sys.path.insert(0, str(ROOT / "pyodide-llm_b200"))
    import build

    build.build()
    return abi.load()


def test_exports_every_declared_symbol(lib):
    names = abi.exported_symbols()
    assert len(names) >= 30
    for name in names:
        assert hasattr(lib, name), name


def test_abi_version_and_errors(lib):
    assert lib.b200fwd_abi_version() == 1
    # a null engine is refused with a message, never a crash
    rc = lib.b200fwd_forward(None, 1, 0, 1)
    assert rc == abi.EINVAL
    assert "engine" in abi.last_error()
    assert lib.b200fwd_destroy(None) == 0


def test_struct_layout_matches_header():
    # the C struct sizes as the header lays them out (x86-64)
    assert ctypes.sizeof(abi.Tensor) == 64
    assert ctypes.sizeof(abi.Options) == 48
    assert abi.Plan.freq_cis_real.offset % 8 == 0


def golden_plan(name):
    plan = json.loads((GOLDEN / f"plan_{name}.json").read_text())
    d = np.load(GOLDEN / f"plan_{name}.npz")
    plan["derived"] = {k: d[k].tobytes() for k in d.files}
    return plan


def test_plan_struct_from_the_references_plan():
    plan = golden_plan("tiny_gqa")
    s, keep = abi.plan_struct(plan)
    assert (s.dim, s.n_layers, s.n_heads, s.n_kv_heads, s.head_size) == (64, 2, 4, 2, 16)
    assert s.n_outliers == 8 and list(s.outliers)[:8] == plan["outliers"]
    assert s.wq.kind == abi.TENSOR_INT8 and s.wq.group == 32 and s.wq.ndim == 3
    assert s.wcls.offset == s.token_embedding_table.offset  # shared classifier
    assert s.rms_final_weight.kind == abi.TENSOR_F32


@pytest.mark.parametrize("change,words", [
    ({"arch": "gpt2"}, "llama"),
    ({"int8": False}, "int8"),
    ({"form": {"interval": 4}}, "Qwen3.5"),
])
def test_plan_refusals(change, words):
    plan = dict(golden_plan("tiny_gqa"), **change)
    with pytest.raises(abi.PlanError, match=words):
        abi.plan_struct(plan)


def test_plan_refuses_bias_tensors():
    plan = golden_plan("tiny_gqa")
    plan["tensors"] = dict(plan["tensors"], bq={"kind": "f32", "offset": 0, "shape": [2, 64]})
    with pytest.raises(abi.PlanError, match="bq"):
        abi.plan_struct(plan)


def test_make_plan_8b_shape():
    """The plan of the Llama-3-8B-shaped int8 checkpoint (its places without the bytes)."""
    tensors, size = ck.places(ck.LLAMA3_8B)
    assert tensors["wq"]["shape"] == [32, 4096, 4096] and tensors["wk"]["shape"] == [32, 1024, 4096]
    assert "wcls" in tensors and tensors["wcls"]["shape"] == [128256, 4096]
    weights = sum(np.prod(t["shape"]) for n, t in tensors.items() if t["kind"] == "int8")
    assert weights == 8_029_995_008  # layers 6.98e9 + embedding and classifier 0.525e9 each
    assert size == 28 + weights * 9 // 8 + 4 * (32 * 4096 * 2 + 4096)


# the engine's matmul choices for the 8B projections on 148 SMs, as measured per launch (every layer's copy in turn):
# (lane split, tile tokens) by token count, for q|k|v 6144x4096, o 4096x4096, w1|w3 28672x4096, w2 4096x14336 and the
# classifier 128256x4096
MATMUL_PLANS = {
    2: [(1, 16), (1, 16), (0, 16), (1, 16), (0, 16)],
    8: [(1, 16), (1, 16), (0, 16), (1, 16), (0, 16)],
    32: [(1, 32), (1, 32), (0, 32), (1, 32), (0, 32)],
    48: [(0, 16), (1, 64), (0, 64), (1, 64), (0, 64)],
    64: [(1, 64), (1, 64), (0, 64), (1, 64), (0, 64)],
    128: [(0, 64), (1, 64), (0, 64), (1, 64), (0, 64)],
    512: [(0, 64), (0, 64), (0, 64), (0, 64), (0, 64)],
}
SHAPES_8B = [(6144, 4096), (4096, 4096), (28672, 4096), (4096, 14336), (128256, 4096)]


@pytest.mark.parametrize("count", sorted(MATMUL_PLANS))
def test_matmul_plan_of_the_8b_shapes(lib, count):
    """b200k_matmul_plan: the kernel and tile width the engine takes per matrix, from the measured stage times (at 64
    tokens, q|k|v, o and w2 on the lane split, w1|w3 and the classifier on one CTA a tile of 64 tokens)."""
    lane, tile = ctypes.c_int32(), ctypes.c_int32()
    got = []
    for rows, n in SHAPES_8B:
        assert lib.b200k_matmul_plan(rows, n, count, 148, 64, ctypes.byref(lane), ctypes.byref(tile)) == 0
        got.append((lane.value, tile.value))
    assert got == MATMUL_PLANS[count]


def test_matmul_plan_refusals(lib):
    lane, tile = ctypes.c_int32(), ctypes.c_int32()
    assert lib.b200k_matmul_plan(4096, 4096, 1, 148, 64, ctypes.byref(lane), ctypes.byref(tile)) == abi.EINVAL
    assert lib.b200k_matmul_plan(4096, 100, 64, 148, 64, ctypes.byref(lane), ctypes.byref(tile)) == abi.EINVAL
    assert lib.b200k_matmul_plan(4096, 4096, 64, 148, 48, ctypes.byref(lane), ctypes.byref(tile)) == abi.EINVAL
    # tiles of at most 32 tokens (activations of fewer than 64 tokens): no lane split; o's 32 row tiles x four
    # 16-token tiles still fit the SMs in one round, and a 16-token stage is the cheaper (23.2 against 27.7 us)
    assert lib.b200k_matmul_plan(4096, 4096, 64, 148, 32, ctypes.byref(lane), ctypes.byref(tile)) == 0
    assert (lane.value, tile.value) == (0, 16)
