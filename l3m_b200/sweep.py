"""Standalone matvec sweep, batch 1: bandwidth of the device matvec over the reference's sweep shapes.

    python -m l3m_b200.sweep [--dtypes bf16,q8_0,q4_0,mxfp4] [--shapes 288x288,...] [--iters 200]
                             [--exact 1] [--json out.jsonl]

Shapes M x K: 288x288, 768x288, 2048x768, 4096x4096, 32000x768. Tiles are written straight into the
tile layout with the sweep's value distributions: q8_0 int8 uniform in [-127, 127] with fp16 scales
|N(0,1)|*0.01; q4_0 nibbles uniform in [0, 15] (value - 8) with the same scales; mxfp4 e2m1 codes
uniform with e8m0 scales uniform in [118, 130]; bf16 weights N(0, 0.02). x ~ N(0,1) is prepared on
the device (l3m_vec_prepare_dev). Each case runs l3m_gemv_dev (the C ABI, device pointers) in two
regimes; `iters` launches are captured into a CUDA graph, which is replayed once warm and once
timed with CUDA events (so the GPU time per launch is measured, not the host's launch rate). The
tiles are declared constant (L3M_GEMV_CONST_TILES, as model weights are), so a launch may start
streaming them while the previous one finishes; --ordered measures without that:

  hbm  R copies of the matrix, at least 2.5x the L2 in total, used round robin: every launch reads
       its tiles from HBM;
  l2   the same copy every launch (every sweep matrix fits in L2).

GB/s = tile bytes of one matrix / mean launch time (the activation and output are a few KB). The
HBM denominator is MEASURED_PEAKS.json's copy bandwidth; the L2 reference is a plain copy of a
32 MiB buffer (read + write bytes) measured here in the same process.
"""
import argparse
import ctypes as C
import json
import sys
from pathlib import Path

import numpy as np

SHAPES = [(288, 288), (768, 288), (2048, 768), (4096, 4096), (32000, 768)]
DTYPES = {"bf16": 1, "q8_0": 2, "q4_0": 3, "mxfp4": 4}
ROOT = Path(__file__).resolve().parent.parent


def make_tiles(rng, dtype, m, k):
    """The packed tiles (uint8) of an m x k matrix of `dtype` with the sweep's distributions."""
    nt, nb = m // 16, k // 32
    if dtype == "bf16":
        from .synth import to_bf16
        return to_bf16(rng.standard_normal(m * k, dtype=np.float32) * np.float32(0.02)).view(np.uint8)
    bb = {"q8_0": 544, "q4_0": 288, "mxfp4": 272}[dtype]
    t = np.empty((nt, nb, bb), np.uint8)
    if dtype == "q8_0":
        t[:, :, 32:] = rng.integers(1, 256, (nt, nb, 512), dtype=np.uint8)             # v + 128, v in [-127, 127]
    elif dtype == "q4_0":
        t[:, :, 32:] = rng.integers(0, 256, (nt, nb, 256), dtype=np.uint8)             # two uniform nibbles per byte
    else:
        t[:, :, 16:] = rng.integers(0, 256, (nt, nb, 256), dtype=np.uint8)             # two uniform e2m1 codes per byte
    if dtype == "mxfp4":
        t[:, :, :16] = rng.integers(118, 131, (nt, nb, 16), dtype=np.uint8)
    else:
        d = (np.abs(rng.standard_normal((nt, nb, 16))) * 0.01).astype(np.float16)
        t[:, :, :32] = d.view(np.uint8).reshape(nt, nb, 32)
    return t.reshape(-1)


def l2_copy_gbs(torch, iters=200):
    a = torch.empty(8 << 20, dtype=torch.float32, device="cuda")
    b = torch.empty_like(a)
    for _ in range(10):
        b.copy_(a)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(iters):
        b.copy_(a)
    e1.record()
    torch.cuda.synchronize()
    return 2 * a.numel() * 4 * iters / (e0.elapsed_time(e1) * 1e-3) / 1e9


CONST_TILES = 2   # l3m_gemv_dev flag: the tiles are constant (include/l3m_kernels.h, L3M_GEMV_CONST_TILES)


def run(dtypes, shapes, iters, exact, out, echo=True, const_tiles=True):
    import torch
    from . import Vec, lib
    L = lib()
    torch.cuda.init()
    stream = torch.cuda.current_stream()
    sp = C.c_void_p(stream.cuda_stream)
    l2 = torch.cuda.get_device_properties(0).L2_cache_size
    peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) if (ROOT / "MEASURED_PEAKS.json").exists() else {}
    hbm_peak, peak_kind = (peaks["hbm_gbs"], "measured") if "hbm_gbs" in peaks else (6650.0, "fallback")
    l2_ref = l2_copy_gbs(torch)
    rng = np.random.default_rng(2)
    rows = []
    for name in dtypes:
        dt = DTYPES[name]
        for m, k in shapes:
            host = make_tiles(rng, name, m, k)
            nbytes = host.size
            assert nbytes == L.l3m_tile_bytes(dt, k) * (m // 16)
            reps = max(1, -(-int(2.5 * l2) // nbytes))
            stride = -(-nbytes // 256) * 256
            buf = torch.empty(reps * stride, dtype=torch.uint8, device="cuda")
            one = torch.from_numpy(host).cuda()
            for r in range(reps):
                buf[r * stride:r * stride + nbytes].copy_(one)
            x = torch.from_numpy(rng.standard_normal(k).astype(np.float32)).cuda()
            scratch = torch.empty(4 * k + 64, dtype=torch.uint8, device="cuda")
            v = Vec()
            assert L.l3m_vec_prepare_dev(dt, C.byref(v), C.c_void_p(x.data_ptr()), k, C.c_void_p(scratch.data_ptr()), sp) == 0
            y = torch.empty(m, dtype=torch.float32, device="cuda")
            base = buf.data_ptr()
            for regime in ("hbm", "l2"):
                def launch(i, st):
                    p = base + (i % reps) * stride if regime == "hbm" else base
                    if L.l3m_gemv_dev(exact | (CONST_TILES if const_tiles else 0), dt, C.c_void_p(y.data_ptr()), C.c_void_p(p), m // 16,
                                      k, C.byref(v), st):
                        raise RuntimeError(L.l3m_cuda_error().decode())
                for i in range(min(20, reps) if regime == "hbm" else 20):
                    launch(i, sp)
                torch.cuda.synchronize()
                # The launches are captured into a CUDA graph and replayed, so the GPU runs them back to
                # back (a Python loop of single launches cannot issue faster than about one per 6 us).
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, capture_error_mode="relaxed"):
                    cs = C.c_void_p(torch.cuda.current_stream().cuda_stream)
                    for i in range(iters):
                        launch(i, cs)
                g.replay()
                torch.cuda.synchronize()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(stream)
                g.replay()
                e1.record(stream)
                torch.cuda.synchronize()
                us = e0.elapsed_time(e1) * 1e3 / iters
                del g
                gbs = nbytes / (us * 1e-6) / 1e9
                row = {"dtype": name, "m": m, "k": k, "regime": regime, "table": "exact" if exact else "fast", "const_tiles": bool(const_tiles),
                       "bytes": nbytes, "us_per_launch": round(us, 3), "gbs": round(gbs, 1),
                       "frac_hbm": round(gbs / hbm_peak, 4), "frac_l2_copy": round(gbs / l2_ref, 4),
                       "hbm_peak": hbm_peak, "hbm_peak_kind": peak_kind, "l2_copy_gbs": round(l2_ref, 1), "copies": reps}
                rows.append(row)
                if echo:
                    print(json.dumps(row), flush=True)
                if out:
                    out.write(json.dumps(row) + "\n")
            del buf, one
            torch.cuda.empty_cache()
    return rows


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--dtypes", default="bf16,q8_0,q4_0,mxfp4")
    ap.add_argument("--shapes", default=",".join(f"{m}x{k}" for m, k in SHAPES))
    ap.add_argument("--iters", type=int, default=200)
    ap.add_argument("--exact", type=int, default=1)
    ap.add_argument("--json", default="")
    ap.add_argument("--ordered", action="store_true",
                    help="do not declare the tiles constant: each launch reads its tiles only after the previous one ends")
    a = ap.parse_args()
    shapes = [tuple(int(v) for v in s.split("x")) for s in a.shapes.split(",")]
    with open(a.json, "w") if a.json else open("/dev/null", "w") as out:
        rows = run(a.dtypes.split(","), shapes, a.iters, a.exact, out, const_tiles=not a.ordered)
    print("\n| dtype | M x K | MB | HBM: us | GB/s | of HBM peak | L2: us | GB/s |")
    print("|---|---|---|---|---|---|---|---|")
    by = {(r["dtype"], r["m"], r["k"], r["regime"]): r for r in rows}
    for name in a.dtypes.split(","):
        for m, k in shapes:
            h, l = by[(name, m, k, "hbm")], by[(name, m, k, "l2")]
            print(f"| {name} | {m}x{k} | {h['bytes'] / 1e6:.2f} | {h['us_per_launch']:.2f} | {h['gbs']:.0f} | {h['frac_hbm']:.1%} "
                  f"| {l['us_per_launch']:.2f} | {l['gbs']:.0f} |")
    return 0


if __name__ == "__main__":
    sys.exit(main())
