"""l3m_gemv_splitk_dev, the exact quantised matvec that allocates nothing: on a B200 it must give
the same y as l3m_gemv_dev's exact table (tolerance: bit-identical, since both follow the
reference's block order), on two calls in a row through the same static scratch, and it must
refuse calls larger than its scratch or of f32/bf16 without launching anything.

Collected last on purpose, and it must also pass alone in a fresh process."""
import ctypes as C

import numpy as np
import pytest

from conftest import P, Vec
from test_gpu_kernels import Cuda, setup_case

pytestmark = pytest.mark.gpu

MAX_PAIRS = 1 << 19


@pytest.fixture(scope="module")
def cuda(gpu):
    c = Cuda()
    yield c
    c.free()


def device_case(gpu, oracle, cuda, rng, dtype, k, ntiles, missing=0, edge=False):
    tiles, x, v, vo, want, keep = setup_case(gpu, oracle, rng, dtype, k, ntiles, missing, edge)
    nb = k // 32
    q8 = np.frombuffer(keep[0], np.int8, k).copy()
    sc = np.frombuffer(keep[0][k:], np.float32, nb).copy()
    su = np.frombuffer(keep[0][k + 4 * nb:], np.int32, nb).copy()
    dv = Vec(q8=cuda.put(q8).value, scale=cuda.put(sc).value, sum=cuda.put(su).value)
    return cuda.put(tiles), dv, want


CASES = [(d, k, n) for d in (2, 3, 4) for k, n in ((288, 1), (288, 18), (1376, 9), (3072, 5), (768, 128))] + \
        [(2, 4096, 256), (4, 4096, 256)]          # 256 * 16 * 128 = the scratch's full 524,288 results


@pytest.mark.parametrize("dtype,k,ntiles", CASES)
def test_splitk_equals_exact_gemv_twice(gpu, oracle, cuda, dtype, k, ntiles):
    rng = np.random.default_rng(1000 + 10 * dtype + ntiles)
    dt, dv, want = device_case(gpu, oracle, cuda, rng, dtype, k, ntiles, missing=5 if ntiles > 1 else 0, edge=ntiles == 9)
    m = ntiles * 16
    y_ref, y1, y2 = cuda.empty(4 * m), cuda.empty(4 * m), cuda.empty(4 * m)
    assert gpu.l3m_gemv_dev(1, dtype, y_ref, dt, ntiles, k, C.byref(dv), None) == 0, gpu.l3m_cuda_error()
    assert gpu.l3m_gemv_splitk_dev(dtype, y1, dt, ntiles, k, C.byref(dv), None) == 0, gpu.l3m_cuda_error()
    assert gpu.l3m_gemv_splitk_dev(dtype, y2, dt, ntiles, k, C.byref(dv), None) == 0, gpu.l3m_cuda_error()
    r = cuda.get(y_ref, np.zeros(m, np.float32))
    a, b = cuda.get(y1, np.zeros(m, np.float32)), cuda.get(y2, np.zeros(m, np.float32))
    assert np.array_equal(r.view(np.uint32), want.view(np.uint32)), "l3m_gemv_dev differs from the oracle"
    assert np.array_equal(a.view(np.uint32), r.view(np.uint32)), ("first call", np.abs(a - r).max())
    assert np.array_equal(b.view(np.uint32), r.view(np.uint32)), ("second call", np.abs(b - r).max())
    cuda.free()


@pytest.mark.parametrize("dtype,k,ntiles", [(2, 768, 2000), (3, 4096, 256), (4, 288, 18)])
def test_const_tiles_flag_gives_the_same_y(gpu, oracle, cuda, dtype, k, ntiles):
    """l3m_gemv_dev with the tiles declared constant (bit 1 of exact: the kernel may read them before
    earlier work on the stream ends) computes the same y, on back-to-back calls."""
    rng = np.random.default_rng(77 + dtype)
    dt, dv, want = device_case(gpu, oracle, cuda, rng, dtype, k, ntiles)
    m = ntiles * 16
    y1, y2 = cuda.empty(4 * m), cuda.empty(4 * m)
    for y in (y1, y2, y1):
        assert gpu.l3m_gemv_dev(1 | 2, dtype, y, dt, ntiles, k, C.byref(dv), None) == 0, gpu.l3m_cuda_error()
    a, b = cuda.get(y1, np.zeros(m, np.float32)), cuda.get(y2, np.zeros(m, np.float32))
    assert np.array_equal(a.view(np.uint32), want.view(np.uint32)) and np.array_equal(b.view(np.uint32), want.view(np.uint32))
    cuda.free()


def test_splitk_rejects_what_it_cannot_hold(gpu, oracle, cuda):
    rng = np.random.default_rng(5)
    dt, dv, _ = device_case(gpu, oracle, cuda, rng, 2, 288, 1)
    y = cuda.empty(4 * 16)
    # one tile past the scratch: 3641 tiles * 16 * 9 blocks > 524,288 (arguments are checked before any access)
    assert gpu.l3m_gemv_splitk_dev(2, y, dt, MAX_PAIRS // (16 * 9) + 1, 288, C.byref(dv), None) == -1
    assert b"exceed the static scratch" in gpu.l3m_cuda_error()
    for dtype in (0, 1):
        assert gpu.l3m_gemv_splitk_dev(dtype, y, dt, 1, 288, C.byref(dv), None) == -1
        assert b"quantised dtypes only" in gpu.l3m_cuda_error()
    assert gpu.l3m_gemv_splitk_dev(2, y, dt, 1, 100, C.byref(dv), None) == -1
    assert gpu.l3m_gemv_splitk_dev(2, y, dt, 0, 288, C.byref(dv), None) == 0
    cuda.free()
