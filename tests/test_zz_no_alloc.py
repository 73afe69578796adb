"""The allocation-free decode entry point, called through its exported C
symbol, must give the same attention output as the regular binding.

Why it exists: some callers of this library cannot allocate GPU memory while
they run (an embedding runtime that owns every device allocation, a plugin
host that forbids cudaMalloc on its hot path, or a plain C caller with no
PyTorch allocator). For them ``swift_paged_decode_noalloc`` takes only inputs
and outputs and keeps its split-KV scratch in a fixed array inside the
library. This file is named so that pytest collects it last.
"""

import ctypes
import math

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _lib():
    from swiftllm_b200.ops import cuda_ext
    lib = ctypes.CDLL(cuda_ext().__file__)
    fn = lib.swift_paged_decode_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64,
                   ctypes.c_int64, ctypes.c_int64, ctypes.c_int, ctypes.c_int, ctypes.c_void_p,
                   ctypes.c_int64, ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                   ctypes.c_int, ctypes.c_float, ctypes.c_int, ctypes.c_void_p]
    return fn


def _case(lens, Hq, Hkv, D, bs=16, L=2, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    nbs = [(l + bs - 1) // bs for l in lens]
    total = sum(nbs) + 2
    kv = torch.randn(total, L, 2, Hkv, bs, D, device="cuda", generator=g).to(torch.bfloat16)
    perm = torch.randperm(total, device="cuda", generator=g).to(torch.int32)
    bt = torch.zeros(len(lens), max(nbs) + 1, dtype=torch.int32, device="cuda")
    o = 0
    for i, n in enumerate(nbs):
        bt[i, :n] = perm[o:o + n]
        o += n
    q = torch.randn(len(lens), Hq, D, device="cuda", generator=g).to(torch.bfloat16)
    sl = torch.tensor(lens, dtype=torch.int32, device="cuda")
    return kv, bt, q, sl


def _run_both(fn, C, lens, Hq, Hkv, D, splits, layer, seed):
    kv, bt, q, sl = _case(lens, Hq, Hkv, D, seed=seed)
    rows = len(lens)
    scale = 1.0 / math.sqrt(D)
    ws = torch.empty(rows * Hq * splits * (D + 2), dtype=torch.float32, device="cuda")
    ref = torch.empty_like(q)
    C.paged_decode(ref, q, kv, layer, bt, sl, rows, splits, scale, 0, ws)
    out = torch.full_like(q, float("nan"))
    stream = torch.cuda.current_stream().cuda_stream
    rc = fn(out.data_ptr(), q.data_ptr(), kv.data_ptr(), kv.stride(0), layer * kv.stride(1),
            kv.stride(2), kv.size(4), D, bt.data_ptr(), bt.stride(0), sl.data_ptr(), rows, Hq,
            Hkv, splits, scale, 0, stream)
    torch.cuda.synchronize()
    assert rc == 0
    torch.testing.assert_close(out.float(), ref.float(), rtol=2e-2, atol=2e-2)
    lib = ctypes.CDLL(C.__file__)
    code, site = ctypes.c_int(-1), ctypes.c_int(-1)
    assert lib.swift_noalloc_status(ctypes.byref(code), ctypes.byref(site), 1) == 0
    assert code.value == 0, (code.value, site.value)


def test_noalloc_decode_matches_regular_entry_twice():
    from swiftllm_b200.ops import cuda_ext
    C = cuda_ext()
    fn = _lib()
    # two calls in a row with different shapes: the shared scratch keeps the
    # previous call's contents, which must not leak into the next result
    _run_both(fn, C, [1, 17, 200, 1000, 33], 32, 8, 128, splits=4, layer=1, seed=1)
    _run_both(fn, C, [5, 64, 300], 8, 8, 128, splits=3, layer=0, seed=2)
    assert C.read_status(True)[0] == 0


def test_noalloc_rejects_oversized_request():
    fn = _lib()
    # rows * Hq * splits * (D + 2) * 4 bytes far above the 8 MiB scratch
    dummy = torch.zeros(16, dtype=torch.int32, device="cuda")
    rc = fn(dummy.data_ptr(), dummy.data_ptr(), dummy.data_ptr(), 8, 0, 8, 16, 128,
            dummy.data_ptr(), 1, dummy.data_ptr(), 4096, 64, 8, 16, 1.0, 0,
            torch.cuda.current_stream().cuda_stream)
    assert rc == 1


def test_noalloc_rejects_unaligned_arguments():
    fn = _lib()
    dummy = torch.zeros(64, dtype=torch.int32, device="cuda")
    p = dummy.data_ptr()
    stream = torch.cuda.current_stream().cuda_stream
    # a KV pointer off the 16-byte grid, then a stride that is not a
    # multiple of 8 elements: rejected before any launch
    assert fn(p, p, p + 2, 8, 0, 8, 16, 128, p, 1, p, 1, 8, 8, 1, 1.0, 0, stream) == 4
    assert fn(p, p, p, 12, 0, 8, 16, 128, p, 1, p, 1, 8, 8, 1, 1.0, 0, stream) == 4


def test_noalloc_status_word_reads_clean():
    from swiftllm_b200.ops import cuda_ext
    lib = ctypes.CDLL(cuda_ext().__file__)
    st = lib.swift_noalloc_status
    st.restype = ctypes.c_int
    st.argtypes = [ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_int), ctypes.c_int]
    code, site = ctypes.c_int(-1), ctypes.c_int(-1)
    assert st(ctypes.byref(code), ctypes.byref(site), 1) == 0
    assert code.value == 0
