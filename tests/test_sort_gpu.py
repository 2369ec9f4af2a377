"""Binning primitives: the single-pass (decoupled look-back) scan and the onesweep stable
radix sort against torch on the same data, including ragged sizes and heavy duplicates."""
import ctypes

import pytest
import torch

from complex_valued_holographic_radiance_fields_b200 import _lib

pytestmark = pytest.mark.gpu


def _st(dev):
    return ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)


def _sort(keys, vals, b0, b1):
    L = _lib.lib()
    n = keys.numel()
    ws = torch.empty(max(1, L.cvhrf_sort_pairs_workspace_bytes(n)), dtype=torch.uint8, device=keys.device)
    _lib.check(L.cvhrf_sort_pairs_u32(ctypes.c_void_p(keys.data_ptr()), ctypes.c_void_p(vals.data_ptr()), n, b0, b1,
                                      ctypes.c_void_p(ws.data_ptr()), ws.numel(), _st(keys.device)), "sort")


@pytest.mark.parametrize("n", [1, 2, 1000, 2047, 2048, 2049, 300000, 5000000])
@pytest.mark.parametrize("bits", [(0, 32), (0, 12), (4, 20)])
def test_sort_pairs_stable(cuda, n, bits):
    g = torch.Generator(device=cuda).manual_seed(n + bits[1])
    keys64 = torch.randint(0, 2 ** 32, (n,), generator=g, device=cuda, dtype=torch.int64)
    if n > 1000:
        keys64[::3] = keys64[::3] & 0xFF  # many duplicates
    keys = keys64.to(torch.int32)  # same bits as uint32
    vals = torch.arange(n, dtype=torch.int32, device=cuda)
    b0, b1 = bits
    field = (keys64 >> b0) & ((1 << (b1 - b0)) - 1)
    order = torch.sort(field, stable=True).indices
    k, v = keys.clone(), vals.clone()
    _sort(k, v, b0, b1)
    assert torch.equal(v, vals[order].to(torch.int32))
    assert torch.equal(k, keys[order])


@pytest.mark.parametrize("n", [1, 100, 4095, 4096, 4097, 1000000, 3000000])
def test_inclusive_scan(cuda, n):
    L = _lib.lib()
    g = torch.Generator(device=cuda).manual_seed(n)
    x = torch.randint(0, 50, (n,), generator=g, device=cuda, dtype=torch.int32)
    out = torch.empty_like(x)
    ws = torch.empty(L.cvhrf_inclusive_scan_workspace_bytes(n), dtype=torch.uint8, device=cuda)
    _lib.check(L.cvhrf_inclusive_scan_u32(ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(out.data_ptr()), n,
                                          ctypes.c_void_p(ws.data_ptr()), ws.numel(), _st(cuda)), "scan")
    assert torch.equal(out.to(torch.int64), torch.cumsum(x.to(torch.int64), 0))
    # in place
    _lib.check(L.cvhrf_inclusive_scan_u32(ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(x.data_ptr()), n,
                                          ctypes.c_void_p(ws.data_ptr()), ws.numel(), _st(cuda)), "scan")
    assert torch.equal(x, out)


def test_no_lookback_timeouts(cuda):
    assert _lib.lib().cvhrf_lookback_timeouts() == 0
