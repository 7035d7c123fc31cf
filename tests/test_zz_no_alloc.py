"""armai_dev_int4_gemv_q4_x_q8_noalloc: the static-scratch variant gives the
same bits as armai_dev_int4_gemv_q4_x_q8 on two calls in a row (the second
reusing the scratch the first wrote), and refuses K beyond its scratch.

Named to be collected last, so it also runs after every other test has used
the device.
"""
import ctypes

import numpy as np
import pytest

from arm_ai_b200 import prims
from arm_ai_b200._lib import ArmaiError, check, load_cuda

pytestmark = pytest.mark.gpu

RNG = np.random.default_rng(2024)


def _dev(torch, arr):
    return torch.from_numpy(np.ascontiguousarray(arr)).cuda()


def _call(fn, torch, a, wp, ws, n, k):
    out = torch.empty(n, dtype=torch.float32, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    check(fn(ctypes.c_void_p(a.data_ptr()), ctypes.c_void_p(wp.data_ptr()), ctypes.c_void_p(ws.data_ptr()),
             ctypes.c_void_p(out.data_ptr()), n, k, ctypes.c_void_p(stream)))
    return out


@pytest.mark.parametrize("n,k", [(4096, 4096), (300, 16384)])
def test_noalloc_matches_allocating_entry(built, n, k):
    torch = pytest.importorskip("torch")
    lib = load_cuda()
    results = []
    for _ in range(2):  # two calls in a row, different inputs
        w = RNG.uniform(-1, 1, (n, k)).astype(np.float32)
        packed, scales = prims.quantize_int4_q4_0_op(w, n, k)
        a = RNG.uniform(-1, 1, k).astype(np.float32)
        da, dwp, dws = _dev(torch, a), _dev(torch, packed), _dev(torch, scales)
        want = _call(lib.armai_dev_int4_gemv_q4_x_q8, torch, da, dwp, dws, n, k)
        got = _call(lib.armai_dev_int4_gemv_q4_x_q8_noalloc, torch, da, dwp, dws, n, k)
        torch.cuda.synchronize()
        results.append((got.cpu().numpy(), want.cpu().numpy()))
    for got, want in results:
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    assert not np.array_equal(results[0][0], results[1][0])


def test_noalloc_rejects_k_beyond_scratch(built):
    torch = pytest.importorskip("torch")
    lib = load_cuda()
    k, n = 16384 + 32, 4
    dummy = torch.zeros(1, dtype=torch.float32, device="cuda")
    with pytest.raises(ArmaiError, match="exceeds the static scratch"):
        _call(lib.armai_dev_int4_gemv_q4_x_q8_noalloc, torch, dummy, dummy, dummy, n, k)
