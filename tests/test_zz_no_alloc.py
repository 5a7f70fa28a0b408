"""The allocation-free paged decode entry point, called through its exported C symbol.

Callers that cannot allocate device memory when they run the kernel (hosts that reserve all device
memory up front and manage it themselves, or that run under a hard memory cap) use
``es_paged_decode_noalloc``, which keeps its split-KV scratch in a fixed array inside the library.
This test loads the symbol with ctypes from the built extension, runs it twice in a row on
different inputs, and checks each output against the regular entry point (the torch binding with
caller-provided scratch): both run the same kernels with the same split length, so the outputs
must be identical bit for bit. It also checks that a request too
large for the fixed scratch is refused with an error instead of being served.

The file name sorts last, so a run that stops at the first failure has run every other test first.
"""

import ctypes
import math

import pytest
import torch

from everserve_b200 import _ext
from everserve_b200.ops import KernelOps

pytestmark = pytest.mark.gpu

CUDA_ERROR_INVALID_VALUE = 1


@pytest.fixture(scope="module")
def lib():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    so = _ext.load().__file__
    L = ctypes.CDLL(so)
    L.es_paged_decode_noalloc.restype = ctypes.c_int
    L.es_paged_decode_noalloc.argtypes = [
        ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_int, ctypes.c_int,
        ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int,
        ctypes.c_int, ctypes.c_int, ctypes.c_float, ctypes.c_void_p,
    ]
    L.es_noalloc_setup.restype = ctypes.c_int
    L.es_noalloc_status.restype = ctypes.c_int
    L.es_noalloc_status.argtypes = [ctypes.c_void_p, ctypes.POINTER(ctypes.c_int)]
    L.es_noalloc_last_error.restype = ctypes.c_char_p
    return L


def _case(seed, B=9, hq=32, hkv=8, d=128, bs=16, max_len=1100):
    g = torch.Generator(device="cuda").manual_seed(seed)
    lens = torch.randint(1, max_len, (B,), generator=g, device="cuda").int()
    mb = (max_len + bs - 1) // bs
    nb = B * mb + 5
    cache = torch.randn(nb, 2, hkv, bs, d, device="cuda", generator=g).bfloat16()
    bt = torch.randperm(nb, device="cuda", generator=g)[: B * mb].view(B, mb).int().contiguous()
    q = torch.randn(B, hq, d, device="cuda", generator=g).bfloat16()
    return q, cache, bt, lens, max_len


def _call(lib, q, cache, bt, lens, max_len, out):
    B, hq, d = q.shape
    _, _, hkv, bs, _ = cache.shape
    stream = torch.cuda.current_stream().cuda_stream
    return lib.es_paged_decode_noalloc(
        q.data_ptr(), q.stride(0), cache.data_ptr(), cache.shape[0], hkv, bs, d, bt.data_ptr(), bt.stride(0),
        lens.data_ptr(), out.data_ptr(), out.stride(0), B, hq, max_len, 1.0 / math.sqrt(d), stream)


def test_noalloc_matches_regular_entry_point(lib):
    assert lib.es_noalloc_setup() == 0
    kops = KernelOps("cuda:0")
    # both decode kernels (the persistent one by its run-time switch, which both entry points
    # follow); two calls each, the second reusing the scratch the first left behind
    cases = [(persist, seed) for persist in (0, 1) for seed in (11, 12)]
    prev = kops.C.set_decode_persist(0)
    for persist, seed in cases:
        kops.C.set_decode_persist(persist)
        q, cache, bt, lens, max_len = _case(seed)
        out = torch.empty(q.shape[0], q.shape[1] * q.shape[2], device="cuda", dtype=torch.bfloat16)
        rc = _call(lib, q, cache, bt, lens, max_len, out)
        assert rc == 0, lib.es_noalloc_last_error()
        torch.cuda.synchronize()
        st = ctypes.c_int(-1)
        assert lib.es_noalloc_status(ctypes.c_void_p(torch.cuda.current_stream().cuda_stream), ctypes.byref(st)) == 0
        assert st.value == 0
        kops.PART_TOKENS = 256
        expect = kops.decode_attention(q, cache, bt, lens, 1.0 / math.sqrt(q.shape[2]), max_len)
        # the same kernels on the same split length: the outputs are identical bit for bit
        assert torch.equal(out.view_as(expect), expect)
    kops.C.set_decode_persist(prev)


def test_noalloc_on_a_second_device(lib):
    """Kernel attributes and the scratch address are set up per device: the first call on another
    device works and matches that device's regular entry point."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    with torch.cuda.device(1):
        assert lib.es_noalloc_setup() == 0
        kops = KernelOps("cuda:1")
        q, cache, bt, lens, max_len = _case(21)
        assert q.device.index == 1
        out = torch.empty(q.shape[0], q.shape[1] * q.shape[2], device="cuda", dtype=torch.bfloat16)
        rc = _call(lib, q, cache, bt, lens, max_len, out)
        assert rc == 0, lib.es_noalloc_last_error()
        torch.cuda.synchronize()
        kops.PART_TOKENS = 256
        expect = kops.decode_attention(q, cache, bt, lens, 1.0 / math.sqrt(q.shape[2]), max_len)
        assert torch.equal(out.view_as(expect), expect)


def test_noalloc_rejects_oversized(lib):
    q, cache, bt, lens, _ = _case(13, B=4)
    out = torch.empty(q.shape[0], q.shape[1] * q.shape[2], device="cuda", dtype=torch.bfloat16)
    # 4 sequences x 32 heads x ceil(1 << 20 / 256) splits x 128 > 2^21 floats
    rc = _call(lib, q, cache, bt, lens, 1 << 20, out)
    assert rc == CUDA_ERROR_INVALID_VALUE
    assert b"exceeds the fixed scratch" in lib.es_noalloc_last_error()
