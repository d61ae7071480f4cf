"""b200k_attention_static, the entry point that allocates nothing: for callers that cannot allocate device memory
where they call (inside a stream capture, on a path that must not stall the device, under a fixed budget). It must
give b200k_attention's numbers (to the bit, the tolerance of these tests), call after call, while its scratch is the
library's own array shared by every call. This file is collected last (its name), so that a run stopping at its
first failure has run every other test before it."""
import numpy as np
import pytest

import oracle
from b200fwd import abi
from gpu_util import bits, dev, full, host, ptr

pytestmark = pytest.mark.gpu


def both(lib, q, kc, vc, pos, nh, nkv, hs, half):
    """(b200k_attention's output, b200k_attention_static's output) on the same inputs."""
    dq, dk, dv = dev(q), dev(kc), dev(vc)
    ref = full(nh * hs, float("nan"))
    att = full(nh * (pos + 1), 0.0)
    abi.check(lib.b200k_attention(ptr(ref), ptr(dq), ptr(dk), ptr(dv), ptr(att), pos, nh, nkv, hs, 0, nh,
                                  1 if half else 0, None))
    got = full(nh * hs, float("nan"))
    abi.check(lib.b200k_attention_static(ptr(got), ptr(dq), ptr(dk), ptr(dv), pos, nh, nkv, hs, 0, nh,
                                         1 if half else 0, None))
    return host(ref), host(got)


def test_no_alloc_attention_matches_the_allocating_one():
    lib = abi.load()
    rng = np.random.default_rng(77)
    # two calls in a row, the second shorter than the first (the array keeps the first call's weights)
    for nh, nkv, hs, pos, half in ((32, 8, 128, 700, True), (8, 8, 64, 90, False)):
        q = rng.standard_normal(nh * hs).astype(np.float32)
        kc = rng.standard_normal((pos + 1, nkv * hs)).astype(np.float32)
        vc = rng.standard_normal((pos + 1, nkv * hs)).astype(np.float32)
        if half:
            kc, vc = oracle.to_f16(kc).reshape(pos + 1, -1), oracle.to_f16(vc).reshape(pos + 1, -1)
        ref, got = both(lib, q, kc, vc, pos, nh, nkv, hs, half)
        assert np.array_equal(bits(got), bits(ref)), (nh, pos)
        want, _ = oracle.attention(q, kc, vc, pos, nh, nkv, hs, half=half)
        assert np.array_equal(bits(got), bits(want)), (nh, pos)


def test_no_alloc_attention_refuses_past_its_array():
    lib = abi.load()
    rc = lib.b200k_attention_static(None, None, None, None, 40000, 32, 8, 128, 0, 32, 1, None)
    assert rc == abi.EINVAL
    q = full(32 * 128, 0.0)
    rc = lib.b200k_attention_static(ptr(q), ptr(q), ptr(q), ptr(q), 40000, 32, 8, 128, 0, 32, 1, None)
    assert rc == abi.EINVAL and "1048576" in abi.last_error()
    # one head of 60000 positions fits the array but not one softmax row of a block: refused before any launch
    rc = lib.b200k_attention_static(ptr(q), ptr(q), ptr(q), ptr(q), 59999, 1, 1, 128, 0, 1, 1, None)
    assert rc == abi.EINVAL and "51200" in abi.last_error()
