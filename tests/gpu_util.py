"""Device buffers for the GPU tests (torch holds the memory; the kernels are called through the C ABI)."""
import ctypes

import numpy as np


def torch():
    import torch as t

    return t


_DT = {np.float32: "float32", np.int8: "int8", np.int32: "int32", np.uint16: "int16", np.uint8: "uint8"}


def dev(a):
    """A numpy array's bytes on cuda:0 (a torch tensor of the same bytes)."""
    t = torch()
    a = np.ascontiguousarray(a)
    if a.dtype == np.uint16:
        a = a.view(np.int16)
    return t.from_numpy(a.copy()).to("cuda:0")


def empty(shape, dtype):
    t = torch()
    tt = {np.float32: t.float32, np.int8: t.int8, np.int32: t.int32, np.uint16: t.int16, np.uint8: t.uint8}[dtype]
    return t.empty(shape, dtype=tt, device="cuda:0")


def full(shape, value, dtype=np.float32):
    x = empty(shape, dtype)
    x.fill_(value)
    return x


def ptr(t):
    return ctypes.c_void_p(t.data_ptr())


def host(t, dtype=None):
    torch().cuda.synchronize()
    a = t.cpu().numpy()
    if dtype is not None:
        a = a.view(dtype)
    return a


def bits(a):
    a = np.ascontiguousarray(a, dtype=np.float32)
    return a.view(np.uint32)
