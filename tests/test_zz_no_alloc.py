"""The allocation-free embedding-gradient entry point
(nsb_op_embedding_bwd_noalloc): for callers that cannot allocate device
memory at the point they need the gradient (allocator callbacks, hosts whose
device memory is all in their own pool). Checked through the C-ABI against
the regular entry point, which takes caller-allocated scratch, on two
consecutive calls (the fixed scratch keeps the previous call's contents, so
the second call proves the counters are cleared), and for the size limit.
This file is collected last so a failure here cannot stop the other tests.
"""
import ctypes as C

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import neuralscript_b200 as nsb  # noqa: E402


def _lib():
    L = nsb.lib()
    L.nsb_op_embedding_bwd_noalloc.restype = C.c_int
    L.nsb_op_embedding_bwd_noalloc.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_void_p,
                                               C.c_void_p]
    L.nsb_op_embedding_bwd.restype = C.c_int
    L.nsb_op_embedding_bwd.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_void_p,
                                       C.c_void_p]
    L.nsb_op_embedding_bwd_scratch_bytes.restype = C.c_size_t
    L.nsb_op_embedding_bwd_scratch_bytes.argtypes = [C.c_int, C.c_int]
    return L


def _ptr(t):
    return C.c_void_p(t.data_ptr())


def _case(seed, M, V, D):
    g = torch.Generator(device="cuda").manual_seed(seed)
    ids = torch.randint(0, V, (M,), device="cuda", generator=g).float()
    ids[:3] = torch.tensor([-1.0, float(V), 2.5], device="cuda")  # skipped, skipped, truncated to 2
    dout = torch.randn(M, D, device="cuda", generator=g)
    return ids, dout


def test_noalloc_matches_regular_entry_point_twice():
    L = _lib()
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    for seed, (M, V, D) in enumerate([(16384, 8192, 512), (5000, 300, 64)]):
        ids, dout = _case(seed, M, V, D)
        scratch = torch.empty(L.nsb_op_embedding_bwd_scratch_bytes(M, V), dtype=torch.uint8, device="cuda")
        ref = torch.empty(V, D, device="cuda")
        assert L.nsb_op_embedding_bwd(_ptr(dout), _ptr(ids), M, V, D, _ptr(ref), _ptr(scratch), stream) == 0
        got = torch.full((V, D), float("nan"), device="cuda")
        assert L.nsb_op_embedding_bwd_noalloc(_ptr(dout), _ptr(ids), M, V, D, _ptr(got), stream) == 0
        torch.cuda.synchronize()
        assert torch.equal(got, ref)  # deterministic: identical bits


def test_noalloc_at_its_limits_after_larger_and_smaller_calls():
    """The whole scratch in use (M = 262144 rows, V = 65536 vocabulary rows),
    then a small call, then the full size again: each bit-for-bit equal to
    the regular entry point, so no counter survives from an earlier call
    anywhere in the shared array."""
    L = _lib()
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    for seed, (M, V, D) in enumerate([(262144, 65536, 32), (700, 50, 16), (262144, 65536, 32)]):
        ids, dout = _case(10 + seed, M, V, D)
        ids[M // 2:M // 2 + 5000] = 7.0  # a bucket far larger than a warp
        scratch = torch.empty(L.nsb_op_embedding_bwd_scratch_bytes(M, V), dtype=torch.uint8, device="cuda")
        ref = torch.empty(V, D, device="cuda")
        assert L.nsb_op_embedding_bwd(_ptr(dout), _ptr(ids), M, V, D, _ptr(ref), _ptr(scratch), stream) == 0
        got = torch.full((V, D), float("nan"), device="cuda")
        assert L.nsb_op_embedding_bwd_noalloc(_ptr(dout), _ptr(ids), M, V, D, _ptr(got), stream) == 0
        torch.cuda.synchronize()
        assert torch.equal(got, ref), (M, V)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs a second GPU")
def test_noalloc_rejects_a_stream_of_another_device():
    L = _lib()
    with torch.cuda.device(1):
        other = torch.cuda.Stream()
    d = torch.zeros(4, 8, device="cuda:0")
    ids = torch.zeros(4, device="cuda:0")
    out = torch.zeros(16, 8, device="cuda:0")
    assert L.nsb_op_embedding_bwd_noalloc(_ptr(d), _ptr(ids), 4, 16, 8, _ptr(out), C.c_void_p(other.cuda_stream)) == -4


def test_noalloc_rejects_sizes_beyond_its_scratch():
    L = _lib()
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    d = torch.zeros(4, 8, device="cuda")
    ids = torch.zeros(4, device="cuda")
    out = torch.zeros(70000, 8, device="cuda")
    assert L.nsb_op_embedding_bwd_noalloc(_ptr(d), _ptr(ids), 4, 70000, 8, _ptr(out), stream) == -2
    big = torch.zeros(300000, device="cuda")
    assert L.nsb_op_embedding_bwd_noalloc(_ptr(d), _ptr(big), 300000, 16, 8, _ptr(out), stream) == -2
    torch.cuda.synchronize()
    assert float(out.abs().sum()) == 0.0
