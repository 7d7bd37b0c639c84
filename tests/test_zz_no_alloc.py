"""gpt_attention_decode_noalloc — decode attention for callers that cannot allocate.

Some embedders (fixed-arena runtimes, plugins not allowed to call cudaMalloc
after start-up, latency-critical loops that must never enter the driver's
allocator) cannot provide the workspace gpt_attention_decode wants. The
no-alloc entry point keeps its split-KV partials in a fixed array inside the
library instead. These tests call both entry points directly through the C
ABI and require the same output, twice in a row (the second call must not be
disturbed by what the first left in the shared array), and check that sizes
beyond the fixed array are refused with a clear error.

Kept in its own file, named to be collected last.
"""
import ctypes
import math

import pytest
import torch

from cutilegpt_b200 import _lib as L

pytestmark = pytest.mark.gpu

NOALLOC_MAX = 256 * 1024   # GPT_NOALLOC_DECODE_SCRATCH_BYTES in include/gpt_b200.h


def _call_both(dtype, B, H, D, Tmax, length, seed, device_len=False):
    lib = L.lib()
    g = torch.Generator(device="cpu").manual_seed(seed)
    C = H * D
    kc = torch.randn((B, H, Tmax, D), generator=g).to(dtype).cuda()
    vc = torch.randn((B, H, Tmax, D), generator=g).to(dtype).cuda()
    q = torch.randn((B, 3 * C), generator=g).to(dtype).cuda()
    # With a device-side length (the graph-captured decode step) the scratch is sized for Tmax and
    # the host length argument is 0.
    need = lib.gpt_attention_decode_workspace_size(B, H, D, Tmax if device_len else length)
    len_dev = torch.tensor([length], dtype=torch.int64, device="cuda") if device_len else None
    lp = len_dev.data_ptr() if device_len else None
    host_len = 0 if device_len else length
    ws = torch.empty(max(need, 16), dtype=torch.uint8, device="cuda")
    ref = torch.empty((B, C), dtype=dtype, device="cuda")
    got = torch.full((B, C), float("nan"), dtype=dtype, device="cuda")
    dt = L.dtype_code(dtype)
    st = torch.cuda.current_stream().cuda_stream
    scale = 1.0 / math.sqrt(D)
    L.check(lib.gpt_attention_decode(q.data_ptr(), 3 * C, kc.data_ptr(), vc.data_ptr(), ref.data_ptr(), C,
                                     B, H, D, Tmax, host_len, lp, scale, ws.data_ptr(), dt, st),
            "gpt_attention_decode")
    L.check(lib.gpt_attention_decode_noalloc(q.data_ptr(), 3 * C, kc.data_ptr(), vc.data_ptr(), got.data_ptr(),
                                             C, B, H, D, Tmax, host_len, lp, scale, dt, st),
            "gpt_attention_decode_noalloc")
    torch.cuda.synchronize()
    return need, ref, got


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_noalloc_matches_workspace_entry_point_twice(dtype):
    # B*H small and a long cache -> several KV splits, so the fixed scratch is really used.
    B, H, D, Tmax = 2, 12, 64, 1024
    for call, (length, seed) in enumerate([(1000, 1), (777, 2)]):
        need, ref, got = _call_both(dtype, B, H, D, Tmax, length, seed)
        assert 0 < need <= NOALLOC_MAX, need
        assert not torch.isnan(got.float()).any(), f"call {call}: output not written"
        if dtype == torch.float32:
            torch.testing.assert_close(got, ref, atol=1e-5, rtol=1e-5)
        else:
            err = ((got.double() - ref.double()).abs().max() / ref.double().abs().max()).item()
            assert err < 2e-2, (call, err)


def test_noalloc_without_splits_and_refusal_of_oversize():
    lib = L.lib()
    # One split: no scratch needed at all.
    need, ref, got = _call_both(torch.bfloat16, 64, 12, 64, 256, 200, 3)
    assert need == 0
    assert torch.equal(got, ref)
    # Find a size whose split-KV scratch exceeds the fixed array on this GPU and check the refusal.
    for bh in range(150, 600):
        if lib.gpt_attention_decode_workspace_size(bh, 1, 128, 1024) > NOALLOC_MAX:
            break
    else:
        pytest.skip("no size on this device needs more than the fixed scratch")
    z = torch.zeros(16, device="cuda")
    st = lib.gpt_attention_decode_noalloc(z.data_ptr(), 3 * 128, z.data_ptr(), z.data_ptr(), z.data_ptr(), 128,
                                          bh, 1, 128, 1024, 1024, None, 0.1, L.GPT_F32, None)
    assert st == L.GPT_ERR_SHAPE
    assert b"fixed" in lib.gpt_last_error_string()


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_noalloc_device_length_twice(dtype):
    """Length read on the device (as in a captured decode step): scratch sized for Tmax, attended length
    below it; two calls in a row against the workspace entry point given the same device length."""
    B, H, D, Tmax = 2, 12, 64, 1024
    for call, (length, seed) in enumerate([(600, 4), (1023, 5)]):
        need, ref, got = _call_both(dtype, B, H, D, Tmax, length, seed, device_len=True)
        assert 0 < need <= NOALLOC_MAX, need
        assert not torch.isnan(got.float()).any(), f"call {call}: output not written"
        if dtype == torch.float32:
            torch.testing.assert_close(got, ref, atol=1e-5, rtol=1e-5)
        else:
            err = ((got.double() - ref.double()).abs().max() / ref.double().abs().max()).item()
            assert err < 2e-2, (call, err)
