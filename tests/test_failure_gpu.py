"""Failure detection on the device without a GPU fault.

Every wait of the tensor-core kernels on an mbarrier is bounded
(%globaltimer); when the limit runs out the kernel records GPT_DEVERR_TIMEOUT
in the library's device error word and returns instead of hanging, and
gpt_device_error() turns that into GPT_ERR_TIMEOUT on the host. Here the
limit is shortened to 1 ms and the library's own bounded-wait helper waits
on an mbarrier whose second arrival never comes; the kernel must return, the
host must see GPT_ERR_TIMEOUT, and the context must stay usable.
"""
import pytest
import torch

from cutilegpt_b200 import _lib as L
from cutilegpt_b200.kernels import ops

pytestmark = pytest.mark.gpu

DEFAULT_LIMIT_NS = 4_000_000_000


def _selftest(expected, arrivals):
    out = torch.full((1,), -1, dtype=torch.int32, device="cuda")
    L.check(L.lib().gpt_selftest_wait(expected, arrivals, out.data_ptr(), L.stream_ptr()), "gpt_selftest_wait")
    return out


def test_bounded_wait_runs_out_and_reports_timeout():
    lib = L.lib()
    L.device_error()                                  # start from a clear error word
    L.check(lib.gpt_set_wait_limit_ns(1_000_000), "gpt_set_wait_limit_ns")
    try:
        out = _selftest(expected=2, arrivals=1)       # one arrival missing: the wait must run out
        with pytest.raises(L.GptError) as e:
            L.device_error()
        assert e.value.status == L.GPT_ERR_TIMEOUT
        assert out.item() == 0
        assert L.device_error() == 0                  # reading the word cleared it
        out = _selftest(expected=2, arrivals=2)       # all arrivals: the phase completes
        assert L.device_error() == 0 and out.item() == 1
    finally:
        L.check(lib.gpt_set_wait_limit_ns(DEFAULT_LIMIT_NS), "gpt_set_wait_limit_ns")


def test_context_usable_after_timeout():
    """After a recorded timeout the same process still runs the tensor-core GEMM correctly."""
    lib = L.lib()
    L.check(lib.gpt_set_wait_limit_ns(1_000_000), "gpt_set_wait_limit_ns")
    try:
        _selftest(expected=3, arrivals=0)
        with pytest.raises(L.GptError):
            L.device_error()
    finally:
        L.check(lib.gpt_set_wait_limit_ns(DEFAULT_LIMIT_NS), "gpt_set_wait_limit_ns")
    g = torch.Generator().manual_seed(0)
    a = torch.randn(512, 256, generator=g).bfloat16().cuda()
    w = torch.randn(384, 256, generator=g).bfloat16().cuda()
    out = torch.empty(512, 384, dtype=torch.bfloat16, device="cuda")
    ops.gemm(a, w, out)
    ref = a.double() @ w.double().t()
    assert ((out.double() - ref).abs().max() / ref.abs().max()).item() < 2e-2
    assert L.device_error() == 0


def test_selftest_argument_checks():
    z = torch.zeros(1, dtype=torch.int32, device="cuda")
    lib = L.lib()
    assert lib.gpt_selftest_wait(0, 0, z.data_ptr(), None) == L.GPT_ERR_SHAPE
    assert lib.gpt_selftest_wait(2, 3, z.data_ptr(), None) == L.GPT_ERR_SHAPE
    assert lib.gpt_set_wait_limit_ns(0) == L.GPT_ERR_ARG
