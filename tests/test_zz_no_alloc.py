"""The allocation-free dedup entry point, called through its exported C symbol.

``flare_unique_first_occurrence_noalloc`` serves callers that cannot allocate
device memory themselves (a host program that owns all device memory through
a fixed pool, or a latency-critical call site).  It must return exactly what
the allocating entry point ``unique_first_occurrence`` returns, on two calls in
a row (the shared scratch keeps the previous call's contents, so the second
call checks that the entry point clears what it needs), and must reject a key
count beyond its fixed scratch with an error code instead of running.

This file is named so that pytest collects it last.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

MAX_KEYS = 1 << 18


def _entry_point():
    from flare_b200 import _C

    lib = ctypes.CDLL(_C.__file__)
    fn = lib.flare_unique_first_occurrence_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                   ctypes.c_void_p, ctypes.c_void_p]
    return fn


def test_noalloc_dedup_matches_allocating_entry_point():
    from flare_b200.ops.sparse import unique_first_occurrence

    fn = _entry_point()
    dev = torch.device("cuda", 0)
    stream = torch.cuda.current_stream(dev)
    for call, (n, hi) in enumerate([(200_000, 5_000), (MAX_KEYS, 1_000_000)]):
        g = torch.Generator(device=dev).manual_seed(100 + call)
        keys = torch.randint(-hi, hi, (n,), generator=g, device=dev, dtype=torch.int64)
        unique = torch.full((n,), -7, dtype=torch.int64, device=dev)
        inverse = torch.full((n,), -7, dtype=torch.int32, device=dev)
        first = torch.full((n,), -7, dtype=torch.int64, device=dev)
        count = torch.full((1,), -7, dtype=torch.int32, device=dev)
        rc = fn(keys.data_ptr(), n, unique.data_ptr(), inverse.data_ptr(), first.data_ptr(), count.data_ptr(),
                stream.cuda_stream)
        assert rc == 0
        torch.cuda.synchronize(dev)
        ref_u, ref_inv, ref_first = unique_first_occurrence(keys)
        k = int(count.item())
        assert k == ref_u.numel()
        # integer outputs: the tolerance is exact equality
        assert torch.equal(unique[:k], ref_u)
        assert torch.equal(inverse, ref_inv)
        assert torch.equal(first[:k], ref_first)


def test_noalloc_dedup_rejects_too_many_keys():
    fn = _entry_point()
    dev = torch.device("cuda", 0)
    out = torch.zeros(4, dtype=torch.int64, device=dev)
    rc = fn(out.data_ptr(), MAX_KEYS + 1, out.data_ptr(), out.data_ptr(), out.data_ptr(), out.data_ptr(),
            torch.cuda.current_stream(dev).cuda_stream)
    assert rc == -1


def test_noalloc_dedup_keys_differing_only_in_high_bits():
    """Keys i << 32 (a table tag packed above bit 32) must spread over the hash table: the
    call finishes quickly and returns what the allocating entry point returns."""
    import time

    from flare_b200.ops.sparse import unique_first_occurrence

    fn = _entry_point()
    dev = torch.device("cuda", 0)
    stream = torch.cuda.current_stream(dev)
    n = 4096
    keys = (torch.arange(n, device=dev, dtype=torch.int64) % 1024) << 32
    unique = torch.empty(n, dtype=torch.int64, device=dev)
    inverse = torch.empty(n, dtype=torch.int32, device=dev)
    first = torch.empty(n, dtype=torch.int64, device=dev)
    count = torch.empty(1, dtype=torch.int32, device=dev)
    torch.cuda.synchronize(dev)
    t0 = time.perf_counter()
    rc = fn(keys.data_ptr(), n, unique.data_ptr(), inverse.data_ptr(), first.data_ptr(), count.data_ptr(),
            stream.cuda_stream)
    torch.cuda.synchronize(dev)
    assert rc == 0
    assert time.perf_counter() - t0 < 1.0
    ref_u, ref_inv, ref_first = unique_first_occurrence(keys)
    k = int(count.item())
    assert k == 1024 == ref_u.numel()
    assert torch.equal(unique[:k], ref_u) and torch.equal(inverse, ref_inv) and torch.equal(first[:k], ref_first)
