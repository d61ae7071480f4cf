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
