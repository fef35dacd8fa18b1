"""The allocation-free global-scale entry point, checked against the regular one.

``ssw_global_scale_inv_noalloc`` exists for callers that own only their input
and output buffers and cannot hand the library a device workspace: a plugin in
an engine that plans all device memory up front, or a service that must keep
its device memory fixed after start-up.  Its scratch is a static array
inside the library, shared by every call.  This test calls it through the C
ABI twice in a row, on different inputs, and requires the same bits as
``ssw_global_scale_inv`` (which uses a caller workspace) every time.  It runs
the same whether it is the first test in a fresh process (the first call sets
the scratch address up for the device) or follows the rest of the suite.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def lib(built_library):
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from test_speed_scalesweep_b200 import _lib
    return _lib.lib()


def _p(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def _with_workspace(lib, x, fp8_max):
    ws = torch.zeros(2, dtype=torch.int32, device=x.device)
    scale = torch.empty(1, dtype=torch.float32, device=x.device)
    amax = torch.empty(1, dtype=torch.float32, device=x.device)
    st = lib.ssw_global_scale_inv(_p(x), 0 if x.dtype == torch.bfloat16 else 1, x.numel(),
                                  fp8_max, _p(scale), _p(amax), _p(ws),
                                  ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert st == 0, lib.ssw_last_error()
    return scale, amax


def _no_alloc(lib, x, fp8_max):
    scale = torch.empty(1, dtype=torch.float32, device=x.device)
    amax = torch.empty(1, dtype=torch.float32, device=x.device)
    st = lib.ssw_global_scale_inv_noalloc(_p(x), 0 if x.dtype == torch.bfloat16 else 1,
                                          x.numel(), fp8_max, _p(scale), _p(amax),
                                          ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert st == 0, lib.ssw_last_error()
    return scale, amax


def _bits(t):
    return t.view(torch.int32).item()


CASES = [((128, 4096), torch.bfloat16, 448.0, 0),
         ((4096, 14336), torch.bfloat16, 256.0, 0),
         ((333, 80), torch.float16, 448.0, 0),
         ((1, 16), torch.bfloat16, 448.0, 0),
         ((1000, 48), torch.bfloat16, 448.0, 1)]  # input starts 2 bytes past an aligned address


@pytest.mark.parametrize("shape,dtype,fp8_max,offset", CASES)
def test_no_alloc_matches_workspace_entry_on_two_calls_in_a_row(lib, shape, dtype, fp8_max,
                                                                offset):
    g = torch.Generator(device="cuda").manual_seed(shape[0] * 7 + shape[1])
    numel = shape[0] * shape[1]
    buf_a = (torch.randn(numel + offset, generator=g, device="cuda") * 3).to(dtype)
    buf_b = (torch.randn(numel + offset, generator=g, device="cuda") * 50).to(dtype)
    a = buf_a[offset:].view(shape)
    b = buf_b[offset:].view(shape)
    for x in (a, b):  # two calls in a row on different data share the static scratch
        s_ref, m_ref = _with_workspace(lib, x, fp8_max)
        s_got, m_got = _no_alloc(lib, x, fp8_max)
        torch.cuda.synchronize()
        assert _bits(s_got) == _bits(s_ref)
        assert _bits(m_got) == _bits(m_ref)
        assert m_got.item() == x.abs().max().float().item()


def _same(a, b):
    return _bits(a) == _bits(b)


def _check_pair(lib, x, fp8_max):
    s_ref, m_ref = _with_workspace(lib, x, fp8_max)
    s_got, m_got = _no_alloc(lib, x, fp8_max)
    torch.cuda.synchronize()
    assert _same(s_got, s_ref), (s_got.item(), s_ref.item())
    assert _same(m_got, m_ref), (m_got.item(), m_ref.item())
    return m_got.item()


def test_no_alloc_partial_tail_chunk_and_specials_in_a_late_chunk(lib):
    """3001 x 4096 elements end 0.1 of the way into a 32768-element chunk
    (the aligned path with a partial last CTA).  Then a NaN, an Inf and an
    all-zero tensor, each placed where only a late CTA sees it."""
    g = torch.Generator(device="cuda").manual_seed(3001)
    x = torch.randn(3001, 4096, generator=g, device="cuda").to(torch.bfloat16)
    assert x.numel() % 32768 != 0
    assert _check_pair(lib, x, 448.0) == x.abs().max().float().item()
    x_nan = x.clone()
    x_nan.view(-1)[x.numel() - 5] = float("nan")
    assert torch.isnan(torch.tensor(_check_pair(lib, x_nan, 448.0)))
    x_inf = x.clone()
    x_inf.view(-1)[x.numel() - 40000] = float("-inf")
    assert _check_pair(lib, x_inf, 256.0) == float("inf")
    zeros = torch.zeros(3001, 4096, dtype=torch.bfloat16, device="cuda")
    assert _check_pair(lib, zeros, 448.0) == 0.0   # the scale is then 1/0 = inf in both


def test_no_alloc_at_its_size_limit(lib):
    """Exactly the largest size the static scratch allows, and one chunk less."""
    limit = lib.ssw_global_scale_inv_noalloc_max_numel()
    g = torch.Generator(device="cuda").manual_seed(28)
    x = torch.empty(limit, dtype=torch.bfloat16, device="cuda")
    for i in range(0, limit, 1 << 26):
        x[i:i + (1 << 26)] = torch.randn(1 << 26, generator=g, device="cuda")
    x[limit - 3] = 1000.0  # the maximum sits in the very last CTA
    assert _check_pair(lib, x, 448.0) == 1000.0
    assert _check_pair(lib, x[: limit - 32768], 448.0) == x[: limit - 32768].abs().max().item()
    del x
    torch.cuda.empty_cache()


def test_no_alloc_rejects_tensors_beyond_its_static_scratch(lib):
    limit = lib.ssw_global_scale_inv_noalloc_max_numel()
    assert limit == 1 << 28
    out = torch.empty(1, dtype=torch.float32, device="cuda")
    x = torch.empty(16, dtype=torch.bfloat16, device="cuda")
    # the size check runs before anything is read, so a small buffer is enough
    st = lib.ssw_global_scale_inv_noalloc(_p(x), 0, limit + 1, 448.0, _p(out), None,
                                          ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert st == 1
    assert "268435456" in lib.ssw_last_error().decode()
