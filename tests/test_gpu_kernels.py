"""Parity of the kernel entry points (include/l3m_kernels.h) with the oracle, on a B200.

The sm100a table must equal the reference's scalar table bit for bit for every dtype (its own
test grid, tests/test_kernels.c:178-198, including the edge cases); the per-block int32 dots and
the unpacked weights are compared exactly; the sm100a-fast table's f32/bf16 entries are held to
the reference's own tolerance for its SIMD tables (1e-4 of the largest |y|, test_kernels.c:114).
The BASELINE.json matvec sweep shapes are checked at full size."""
import ctypes as C

import numpy as np
import pytest

from conftest import P, Vec
from test_oracle import random_rows

pytestmark = pytest.mark.gpu


class Cuda:
    """Just enough of the CUDA runtime (device buffers) to call the *_dev entry points."""

    def __init__(self):
        self.rt = C.CDLL("/usr/local/cuda/lib64/libcudart.so.12")
        self.rt.cudaMalloc.argtypes = [C.POINTER(C.c_void_p), C.c_size_t]
        self.rt.cudaMemcpy.argtypes = [C.c_void_p, C.c_void_p, C.c_size_t, C.c_int]
        self.rt.cudaFree.argtypes = [C.c_void_p]
        self.bufs = []

    def put(self, arr):
        p = C.c_void_p()
        assert self.rt.cudaMalloc(C.byref(p), max(arr.nbytes, 16)) == 0
        assert self.rt.cudaMemcpy(p, P(arr), arr.nbytes, 1) == 0
        self.bufs.append(p)
        return p

    def empty(self, nbytes):
        p = C.c_void_p()
        assert self.rt.cudaMalloc(C.byref(p), max(nbytes, 16)) == 0
        self.bufs.append(p)
        return p

    def get(self, p, arr):
        assert self.rt.cudaDeviceSynchronize() == 0
        assert self.rt.cudaMemcpy(P(arr), p, arr.nbytes, 2) == 0
        return arr

    def free(self):
        for p in self.bufs:
            self.rt.cudaFree(p)
        self.bufs = []


@pytest.fixture(scope="module")
def cuda(gpu):
    c = Cuda()
    yield c
    c.free()


def setup_case(gpu, oracle, rng, dtype, k, ntiles, missing, edge):
    rb, tb = gpu.l3m_row_bytes(dtype, k), gpu.l3m_tile_bytes(dtype, k)
    assert rb == oracle.o_row_bytes(dtype, k) and tb == oracle.o_tile_bytes(dtype, k)
    rows = random_rows(rng, dtype, ntiles * 16, k, rb, edge)
    tiles, tiles_o = np.zeros(ntiles * tb, np.uint8), np.zeros(ntiles * tb, np.uint8)
    for t in range(ntiles):
        ptrs = (C.c_void_p * 16)(*[rows[t * 16 + c].ctypes.data if t * 16 + c < ntiles * 16 - missing else None for c in range(16)])
        gpu.l3m_pack_tile(C.c_void_p(tiles.ctypes.data + t * tb), dtype, ptrs, k)
        oracle.o_pack_tile(C.c_void_p(tiles_o.ctypes.data + t * tb), dtype, ptrs, k)
    assert np.array_equal(tiles, tiles_o), "host packing differs from the reference layout"
    x = (rng.standard_normal(k) * 4).astype(np.float32)
    if edge:
        x[:min(32, k)] = 0
    s1, s2 = np.zeros(4 * k + 64, np.uint8), np.zeros(4 * k + 64, np.uint8)
    v, vo = Vec(), Vec()
    gpu.l3m_vec_prepare(C.byref(v), dtype, P(x), k, P(s1))
    oracle.o_vec_prepare(C.byref(vo), dtype, P(x), k, P(s2))
    assert np.array_equal(s1, s2), "host vec_prepare differs"
    want = np.zeros(ntiles * 16, np.float32)
    oracle.o_gemv(dtype, P(want), P(tiles), ntiles, k, C.byref(vo))
    return tiles, x, v, vo, want, (s1, s2)


GRID = [(d, k) for d in range(5) for k in ([2, 18, 34, 288, 1376] if d <= 1 else [288, 1376, 3072])]


@pytest.mark.parametrize("dtype,k", GRID)
def test_exact_table_matches_scalar(gpu, oracle, dtype, k):
    import l3m_b200
    table = l3m_b200.kernels("sm100a")
    assert gpu.l3m_kernels_usable(C.byref(table)) == 1
    rng = np.random.default_rng(100 + dtype * 10 + k % 7)
    for ntiles in (1, 2, 5, 9):
        for missing in (0, 5, 10, 15):
            for edge in ((False, True) if dtype >= 2 and missing == 5 else (False,)):
                tiles, x, v, vo, want, keep = setup_case(gpu, oracle, rng, dtype, k, ntiles, missing, edge)
                y = np.full(ntiles * 16, np.nan, np.float32)
                table.gemv[dtype](P(y), P(tiles), ntiles, k, C.byref(v))
                assert np.array_equal(y.view(np.uint32), want.view(np.uint32)), (ntiles, missing, edge, np.abs(y - want).max())


@pytest.mark.parametrize("dtype,k", GRID)
def test_fast_table_within_tolerance(gpu, oracle, dtype, k):
    import l3m_b200
    table = l3m_b200.kernels("sm100a-fast")
    rng = np.random.default_rng(7 + dtype)
    for ntiles in (1, 9):
        tiles, x, v, vo, want, keep = setup_case(gpu, oracle, rng, dtype, k, ntiles, 5, False)
        y = np.zeros(ntiles * 16, np.float32)
        table.gemv[dtype](P(y), P(tiles), ntiles, k, C.byref(v))
        if dtype >= 2:
            assert np.array_equal(y.view(np.uint32), want.view(np.uint32))
        else:
            assert np.abs(y - want).max() <= 1e-4 * max(np.abs(want).max(), 1e-30)


@pytest.mark.parametrize("dtype", [2, 3, 4])
def test_block_dots_and_unpack_exact(gpu, oracle, cuda, dtype):
    """The integer path of each quantised kernel: per-(output, block) int32 dots and the unpacked
    integer weights and scales, exactly as the oracle computes them."""
    rng = np.random.default_rng(dtype)
    for k, ntiles in ((288, 3), (1376, 5), (3072, 2)):
        for edge in (False, True):
            tiles, x, v, vo, want, keep = setup_case(gpu, oracle, rng, dtype, k, ntiles, 5, edge)
            nb = k // 32
            dt = cuda.put(tiles)
            q8 = np.frombuffer(keep[0], np.int8, k).copy()
            sc = np.frombuffer(keep[0][k:], np.float32, nb).copy()
            su = np.frombuffer(keep[0][k + 4 * nb:], np.int32, nb).copy()
            dv = Vec(q8=cuda.put(q8).value, scale=cuda.put(sc).value, sum=cuda.put(su).value)
            dd = cuda.empty(ntiles * 16 * nb * 4)
            assert gpu.l3m_block_dots_dev(dtype, dd, dt, ntiles, k, C.byref(dv), None) == 0, gpu.l3m_cuda_error()
            got = cuda.get(dd, np.zeros(ntiles * 16 * nb, np.int32))
            wantd = np.zeros(ntiles * 16 * nb, np.int32)
            oracle.o_block_dots(dtype, P(wantd), P(tiles), ntiles, k, C.byref(vo))
            assert np.array_equal(got, wantd)
            dq, ds = cuda.empty(ntiles * 16 * k), cuda.empty(ntiles * 16 * nb * 4)
            assert gpu.l3m_unpack_dev(dtype, dq, ds, dt, ntiles, k, None) == 0
            gq, gs = cuda.get(dq, np.zeros(ntiles * 16 * k, np.int8)), cuda.get(ds, np.zeros(ntiles * 16 * nb, np.float32))
            wq, ws = np.zeros_like(gq), np.zeros_like(gs)
            oracle.o_unpack(dtype, P(wq), P(ws), P(tiles), ntiles, k)
            assert np.array_equal(gq, wq) and np.array_equal(gs.view(np.uint32), ws.view(np.uint32))
            cuda.free()


def test_f16_scales_every_bit_pattern(gpu, oracle, cuda):
    """The device's binary16 -> binary32 scale conversion on all 65536 bit patterns (subnormals,
    infinities and NaN payloads included), through the q8_0 unpack entry: equal to the oracle's."""
    k, nb = 8192, 256
    tb = gpu.l3m_tile_bytes(2, k)
    ntiles = 65536 // (16 * nb)
    tiles = np.random.default_rng(5).integers(0, 256, ntiles * tb, dtype=np.uint8)
    h = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    for t in range(ntiles):
        for b in range(nb):
            o = t * tb + b * 544
            tiles[o:o + 32] = h[(t * nb + b) * 16:(t * nb + b + 1) * 16].view(np.uint8)
    dt = cuda.put(tiles)
    dq, ds = cuda.empty(ntiles * 16 * k), cuda.empty(ntiles * 16 * nb * 4)
    assert gpu.l3m_unpack_dev(2, dq, ds, dt, ntiles, k, None) == 0, gpu.l3m_cuda_error()
    gs = cuda.get(ds, np.zeros(ntiles * 16 * nb, np.float32))
    wq, ws = np.zeros(ntiles * 16 * k, np.int8), np.zeros(ntiles * 16 * nb, np.float32)
    oracle.o_unpack(2, P(wq), P(ws), P(tiles), ntiles, k)
    assert np.array_equal(gs.view(np.uint32), ws.view(np.uint32))
    cuda.free()


def test_device_prepare_exact(gpu, oracle, cuda):
    rng = np.random.default_rng(3)
    for dtype in (1, 2):
        for n in (288, 1376, 3072):
            x = (rng.standard_normal(n) * rng.uniform(0.01, 10)).astype(np.float32)
            x[32:64] = 0
            want = np.zeros(4 * n + 64, np.uint8)
            vo = Vec()
            oracle.o_vec_prepare(C.byref(vo), dtype, P(x), n, P(want))
            dx, ds = cuda.put(x), cuda.empty(4 * n + 64)
            v = Vec()
            assert gpu.l3m_vec_prepare_dev(dtype, C.byref(v), dx, n, ds, None) == 0
            got = cuda.get(ds, np.zeros(4 * n + 64, np.uint8))
            used = 2 * n if dtype == 1 else n + n // 4
            assert np.array_equal(got[:used], want[:used]), (dtype, n)
            cuda.free()


def test_attend_exact(gpu, oracle):
    """One head of attention, bit for bit (reference tests/test_kernels.c:124-149, 195-197)."""
    import l3m_b200
    table = l3m_b200.kernels("sm100a")
    rng = np.random.default_rng(11)
    from l3m_b200 import synth
    for hd in (16, 32, 40, 48, 64):
        for pos in (0, 1, 37, 255):
            for qscale in ((2.0, 40.0) if (hd, pos) == (64, 255) else (2.0,)):
                stride = 3 * hd
                q = (rng.uniform(-1, 1, hd) * qscale).astype(np.float32)
                k = synth.to_bf16(rng.uniform(-1, 1, (pos + 1) * stride).astype(np.float32))
                v = synth.to_bf16(rng.uniform(-1, 1, (pos + 1) * stride).astype(np.float32))
                a, b = np.full(hd, np.nan, np.float32), np.zeros(hd, np.float32)
                table.attend(P(a), P(q), P(k), P(v), pos, hd, stride)
                oracle.o_attend(P(b), P(q), P(k), P(v), pos, hd, stride)
                assert np.array_equal(a.view(np.uint32), b.view(np.uint32)), (hd, pos, qscale)


def test_expf_matches_c_library(gpu, oracle, cuda):
    """The device expf (softmax, SiLU gate, sampler weights) equals the host C library's expf, which
    the reference calls (src/ops.c:45, 50), bit for bit: one float in every 509 bit patterns over the
    whole 32-bit space (NaNs, infinities, subnormals and the over/underflow edges among them), and
    every 97th float in [-1, 1] plus the edges of the range where expf is finite and
    nonzero. The build already checks the same arithmetic on the host for all 2^32 inputs."""
    import l3m_b200
    lib = l3m_b200.lib()
    sweep = np.arange(0, 2**32, 509, dtype=np.uint64).astype(np.uint32)
    near = np.arange(0, 0x3F800001, 97, dtype=np.uint32)
    edges = np.array([0x42B17217, 0x42B17218, 0x42B17219, 0xC2CFF1B4, 0xC2CFF1B5, 0xC2CFF1B3, 0xC2AEAC4F, 0xC2AEAC50, 0x7F800000,
                      0xFF800000, 0x7FC00000, 0x00000001, 0x80000001, 0x33800000, 0xB3800000], np.uint32)
    x = np.concatenate([sweep, near, near | 0x80000000, edges]).view(np.float32)
    want = np.empty_like(x)
    oracle.o_expf_n(P(x), P(want), x.size)
    dx, dy = cuda.put(x), cuda.empty(x.nbytes)
    assert lib.l3m_expf_dev(dx, dy, x.size, None) == 0
    got = cuda.get(dy, np.empty_like(x))
    same = (got.view(np.uint32) == want.view(np.uint32)) | (np.isnan(got) & np.isnan(want))
    bad = np.nonzero(~same)[0]
    assert bad.size == 0, f"{bad.size} differ, first x bits 0x{x.view(np.uint32)[bad[0]]:08x}"


SWEEP = [(288, 288), (768, 288), (2048, 768), (4096, 4096), (32000, 768)]


@pytest.mark.parametrize("dtype", [1, 2, 3, 4])
def test_sweep_shapes_full_size(gpu, oracle, dtype):
    """The BASELINE.json matvec sweep at full size: exact table equals the scalar oracle."""
    import l3m_b200
    table = l3m_b200.kernels("sm100a")
    rng = np.random.default_rng(dtype)
    for m, k in SWEEP:
        ntiles = m // 16
        tiles, x, v, vo, want, keep = setup_case(gpu, oracle, rng, dtype, k, ntiles, 0, False)
        y = np.zeros(m, np.float32)
        table.gemv[dtype](P(y), P(tiles), ntiles, k, C.byref(v))
        assert np.array_equal(y.view(np.uint32), want.view(np.uint32)), (m, k)
