#!/usr/bin/env python3
"""Batch-1 greedy decode throughput on B200 (BASELINE.json metric), one JSON line on stdout.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--config NAME]

Workload (default): SmolLM2-135M-shaped GQA Llama in q8_0 (the largest
decode configuration; seeded synthetic N(0, 0.02) weights), KV ctx 256, the 4 seeded benchmark
prompt ids, greedy until the context is full: 256 forward passes per step, which is one
l3m_generate call. tok/s counts forward passes, prompt included, as the reference's `l3m bench`.

  value      forward passes / device time of the decode kernel (CUDA events around each launch,
             inputs resident in HBM), max over ranks. With --gpus N (torchrun) one model is split over
             N GPUs and rank 0 drives them all: one batch-1 stream, so scaling is strong
  e2e        the same through the public API (l3m_generate: host prompt in, host tokens out via
             on_token), host wall clock around each call
  roofline   HBM: algorithmic bytes per launch (weights once per token + KV reads and writes) over
             the kernel's duration, against MEASURED_PEAKS.json
  chain_bound  the second bound of this latency-bound kernel: the launch's dependent fp32 chain steps
             (the reference's sequential sums, kept exact) x the measured cycles of one such step
  cpu_baseline  the reference itself (oracle/_ref/l3m bench, built from its sources) on this host's cores

The L2 is flushed (a 256 MiB write) between timed steps. --impl reference times the reference's
own CPU engine on the same model and context instead (rank 0 only).

    python bench.py --sweep [--dtypes bf16,q8_0,q4_0,mxfp4] [--no-cpu]

The matvec half of the metric: one JSON line per sweep case (M x K x dtype, BASELINE.json's sweep
shapes): the device matvec's GB/s with its tiles in HBM and in L2 (l3m_b200.sweep, when a GPU is
present), and as cpu_baseline the reference's own kernel table on the same tiles at 1 core and at
every core of this host (oracle/_ref/libsweep_ref.so: tiles split over an l3m_pool, one l3m_sync
per matvec, as the reference engine runs a sharded matvec).
"""
import argparse
import ctypes as C
import json
import os
import re
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))
from l3m_b200 import synth  # noqa: E402

REF_CLI = ROOT / "oracle" / "_ref" / "l3m"
PUBLISHED = {"SmolLM2-135M-q8_0": 530.0, "stories15M-bf16": 15300.0, "stories42M-q8_0": 10700.0, "stories110M-q4_0": 5800.0}
MODEL_DIR = Path(os.environ.get("L3M_BENCH_DIR", "/tmp/l3m_bench"))


def rank_env():
    return int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)), int(os.environ.get("LOCAL_RANK", 0))


class Clocks:
    """nvidia-smi sampled every 200 ms while the timed region runs."""
    Q = "clocks.sm,clocks.max.sm,clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown," \
        "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap"

    def __init__(self, gpu):
        self.gpu, self.rows, self.proc = gpu, [], None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                          "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=lambda: self.rows.extend(self.proc.stdout), daemon=True)
            self.t.start()
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *a):
        if self.proc:
            time.sleep(0.25)
            self.proc.terminate()
            self.proc.wait()

    def summary(self):
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in self.rows:
            f = [v.strip() for v in r.split(",")]
            if len(f) < 6 or not f[0].replace(".", "").isdigit():
                continue
            sm.append(float(f[0]))
            mx = max(mx, float(f[1]))
            reasons |= {n for n, v in zip(names, f[2:6]) if v.lower() == "active"}
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx or None, "reasons": sorted(reasons),
                "samples": len(sm)}


class L2Flush:
    """A 256 MiB device buffer written between steps (larger than the 126 MB L2)."""

    def __init__(self):
        self.rt = C.CDLL("/usr/local/cuda/lib64/libcudart.so.12")
        self.rt.cudaMalloc.argtypes = [C.POINTER(C.c_void_p), C.c_size_t]
        self.rt.cudaMemset.argtypes = [C.c_void_p, C.c_int, C.c_size_t]
        self.p, self.n = C.c_void_p(), 256 << 20
        assert self.rt.cudaMalloc(C.byref(self.p), self.n) == 0

    def __call__(self, v=0):
        self.rt.cudaMemset(self.p, v & 0xFF, self.n)
        self.rt.cudaDeviceSynchronize()


def algorithmic_bytes(name, positions):
    """Weights once per forward pass plus KV traffic: 2*L*(pos+1)*kv*2 bytes read and 2*L*kv*2 written per position."""
    shape = synth.CONFIGS[name][0]
    L, kvd = shape["n_layers"], shape["dim"] // shape["n_heads"] * shape["n_kv_heads"]
    w = synth.weight_bytes(name)
    kv = sum(2 * L * (p + 1) * kvd * 2 + 2 * L * kvd * 2 for p in range(positions))
    return positions * w + kv, positions


def chain_steps(name, positions, n_prompt):
    """Dependent fp32 steps on one launch's critical path (Llama family, the kernels' exact chains),
    summed over its forward passes: per layer the attention norm's sum of squares (dim steps), the
    qkv, wo, up/gate and down matvecs' chains over blocks (k/32 steps for quantised matrices, k for
    bf16/f32), one score's chain (head_dim), the softmax's sequential sum and the V mix (pos + 1 each),
    the ffn norm (dim); on every sampled position the final norm and the head's chain. Exchanges,
    barriers and loads come on top: this is a floor, not a model of the kernel."""
    shape, dtype, head_dtype, _ = synth.CONFIGS[name]
    dim, ffn, L, hd = shape["dim"], shape["ffn_dim"], shape["n_layers"], shape["dim"] // shape["n_heads"]
    mv = lambda dt, k: k if dt in ("bf16", "f32") else k // 32
    per_layer = 2 * dim + 2 * mv(dtype, dim) + mv(dtype, dim) + mv(dtype, ffn) + hd
    total = 0
    for pos in range(positions):
        total += L * (per_layer + 2 * (pos + 1))
        if pos >= n_prompt - 1:
            total += dim + mv(head_dtype, dim)
    return total


def chain_line(lib, name, positions, n_prompt, launch_s, clocks):
    """The chain-latency bound beside the HBM roofline: chain_steps x the measured cycles of one
    dependent fp32 step (l3m_chain_cycles_dev, timed here) at the median SM clock sampled during the
    timed region; frac = that time / the launch's device time."""
    cyc = C.c_double()
    if lib.l3m_chain_cycles_dev(65536, C.byref(cyc)) != 0:
        return {"unavailable": lib.l3m_cuda_error().decode()}
    steps = chain_steps(name, positions, n_prompt)
    mhz = clocks.get("sm_mhz") or clocks.get("sm_max_mhz") or 1965.0
    bound_s = steps * cyc.value / (mhz * 1e6)
    return {"steps_per_launch": steps, "cycles_per_step": round(cyc.value, 3), "sm_mhz": mhz, "bound_ms": round(bound_s * 1e3, 3),
            "launch_ms": round(launch_s * 1e3, 3), "frac": round(bound_s / launch_s, 4),
            "note": "dependent fp32 chain steps of one launch (norms, matvec block chains, attention score, softmax sum and V mix, "
                    "head) x the measured latency of one step; exchanges and loads not counted"}


def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d["hbm_gbs"], "measured"
    return 6650.0, "fallback"


def reference_cpu(path, ctx, n_tokens):
    """The reference's own CLI bench on this host (all its default cores), median of 3."""
    if not REF_CLI.exists():
        return None
    vals, desc = [], ""
    for _ in range(3):
        out = subprocess.run([str(REF_CLI), "bench", str(path), "--ctx", str(ctx), "-n", str(n_tokens), "--force", "--md"],
                             capture_output=True, text=True, timeout=900)
        if out.returncode:
            return {"unavailable": out.stderr.strip()[:200]}
        row = out.stdout.splitlines()[2].split("|")
        desc = row[1].strip()
        vals.append(float(row[2]))
    m = re.search(r"on (\d+) cores? \((\w+)\)", desc)
    return {"value": statistics.median(vals), "unit": "tok/s", "cores": int(m.group(1)) if m else None,
            "kind": "reference", "table": m.group(2) if m else None,
            "sample": f"reference `l3m bench --ctx {ctx} -n {n_tokens} --force`, median of 3 (16 warm-up tokens each)"}


SWEEP_REF = ROOT / "oracle" / "_ref" / "libsweep_ref.so"


def reference_sweep_cpu(lib, dtype, tiles, ntiles, k, x, cpus, seconds=0.25):
    """GB/s of the reference's kernel table on `tiles` over cores `cpus` (tile bytes per matvec over
    the mean time of a calibrated number of matvecs, about `seconds` in all), and the table's name."""
    y = np.zeros(ntiles * 16, np.float32)
    arr = (C.c_int * len(cpus))(*cpus)
    name = C.c_char_p()
    args = (dtype, C.c_void_p(tiles.ctypes.data), ntiles, k, C.c_void_p(x.ctypes.data), C.c_void_p(y.ctypes.data), arr, len(cpus))
    ns = lib.sweep_ref_gemv(*args, 3, C.byref(name))
    if ns <= 0:
        return None, None
    ns = lib.sweep_ref_gemv(*args, max(3, int(seconds * 1e9 / ns)), C.byref(name))
    return tiles.size / ns, name.value.decode()


def bench_sweep(a):
    from l3m_b200 import sweep
    dtypes = a.dtypes.split(",")
    gpu = {}
    try:
        import torch
        have_gpu = torch.cuda.is_available()
    except ImportError:
        have_gpu = False
    clocks = None
    if have_gpu:
        with Clocks(int(os.environ.get("LOCAL_RANK", 0))) as clk:
            for r in sweep.run(dtypes, sweep.SHAPES, 200, 1, None, echo=False):
                gpu[(r["dtype"], r["m"], r["k"], r["regime"])] = r
        clocks = clk.summary()
    lib = None
    if not a.no_cpu and SWEEP_REF.exists():
        lib = C.CDLL(str(SWEEP_REF))
        lib.sweep_ref_gemv.restype = C.c_double
        lib.sweep_ref_gemv.argtypes = [C.c_int, C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.POINTER(C.c_int), C.c_int,
                                       C.c_int, C.POINTER(C.c_char_p)]
    every = sorted(os.sched_getaffinity(0))
    peak, peak_kind = measured_peaks()
    for name in dtypes:
        for m, k in sweep.SHAPES:
            rng = np.random.default_rng([m, k, sweep.DTYPES[name]])
            tiles = sweep.make_tiles(rng, name, m, k)
            line = {"metric": "matvec GB/s", "dtype": name, "m": m, "k": k, "bytes": int(tiles.size), "unit": "GB/s",
                    "higher_is_better": True, "data": "synthetic", "peak_hbm_gbs": peak, "peak_kind": peak_kind}
            h, l2 = gpu.get((name, m, k, "hbm")), gpu.get((name, m, k, "l2"))
            if h:
                line.update(value=h["gbs"], frac_hbm=h["frac_hbm"], us_hbm=h["us_per_launch"], value_l2=l2["gbs"],
                            us_l2=l2["us_per_launch"], l2_copy_gbs=l2["l2_copy_gbs"], clocks=clocks)
            if lib is not None:
                x = rng.standard_normal(k).astype(np.float32)
                g1, table = reference_sweep_cpu(lib, sweep.DTYPES[name], tiles, m // 16, k, x, every[:1])
                gn, _ = reference_sweep_cpu(lib, sweep.DTYPES[name], tiles, m // 16, k, x, every)
                line["cpu_baseline"] = {"value_1core": g1, "value": gn, "unit": "GB/s", "cores": len(every), "kind": "reference",
                                        "table": table, "sample": "reference kernel table, tiles split over an l3m_pool, "
                                        "one l3m_sync per matvec, about 0.25 s of matvecs per core count"}
            print(json.dumps(line), flush=True)


# DRAM traffic of one decode launch per forward pass, from an ncu capture of a short case of the same
# kernel and model (dram__bytes_read.sum + dram__bytes_write.sum over the launch, divided by its
# forward passes), scaled by the bench's forward passes per launch.
DECODE_TRAFFIC = {
    "SmolLM2-135M-q8_0": {"dram_bytes_per_position": 138925084,
                          "note": "ncu dram__bytes_read.sum + dram__bytes_write.sum of one 64-position decode_kernel launch of this "
                                  "model (8,853,367,552 + 37,837,824 B; the 4 prompt positions skip the head), divided by 64 and "
                                  "scaled to this launch's positions"},
}


def matvec_line():
    """The matvec half of the metric on this GPU: q8_0 32000x768 (BASELINE's largest sweep shape) through
    l3m_gemv_dev, tiles read from HBM (copies cycled, 2.5x the L2) and from L2 (one copy), with the
    SM clocks sampled while it runs."""
    from l3m_b200 import sweep
    with Clocks(int(os.environ.get("LOCAL_RANK", 0))) as clk:
        rows = sweep.run(["q8_0"], [(32000, 768)], 400, 1, None, echo=False)
        ordered = sweep.run(["q8_0"], [(32000, 768)], 400, 1, None, echo=False, const_tiles=False)
    by = {r["regime"]: r for r in rows}
    h, l2 = by["hbm"], by["l2"]
    ho = {r["regime"]: r for r in ordered}["hbm"]
    return {"case": "q8_0 32000x768 l3m_gemv_dev (exact, tiles declared constant)", "bytes": h["bytes"], "unit": "GB/s",
            "hbm": {"value": h["gbs"], "us": h["us_per_launch"], "frac": h["frac_hbm"]},
            "l2": {"value": l2["gbs"], "us": l2["us_per_launch"], "frac_of_hbm_peak": round(l2["gbs"] / h["hbm_peak"], 4),
                   "l2_copy_gbs": l2["l2_copy_gbs"]},
            "hbm_ordered": {"value": ho["gbs"], "us": ho["us_per_launch"], "frac": ho["frac_hbm"],
                            "note": "tiles not declared constant: each launch reads them only after the previous launch ends"},
            "peak": h["hbm_peak"], "peak_kind": h["hbm_peak_kind"], "timing": "400 launches in a CUDA graph, CUDA events",
            "clocks": clk.summary()}


def combine_ranks(dist, t_dev, t_wall, positions):
    """The whole job's (device time, wall time, positions): the times as the maximum over ranks, the
    positions summed (a rank that drives no model reports zeros)."""
    if not dist:
        return t_dev, t_wall, positions
    import torch
    t = torch.tensor([t_dev, t_wall, positions], dtype=torch.float64)
    tmax = t.clone()
    dist.all_reduce(tmax, op=dist.ReduceOp.MAX)
    tsum = t.clone()
    dist.all_reduce(tsum, op=dist.ReduceOp.SUM)
    return tmax[0].item(), tmax[1].item(), tsum[2].item()


def residency_line(path, ctx, prompt, max_new, warm_value, steps=2):
    """The same decode with the weights evicted from L2 before every position (the reference's --cold,
    src/engine.c:330-338: the flush is not token time), device-timed, beside the warm number."""
    import l3m_b200
    m = l3m_b200.Model(str(path), ctx=ctx, force=True, cold=True)
    m.generate(prompt, max_new, temperature=0)
    m.perf()
    dev, pos = 0.0, 0
    for _ in range(steps):
        m.generate(prompt, max_new, temperature=0)
        dev += m.device_ns()
        pos += int(m.perf()["tokens"])
    m.close()
    cold = pos / (dev * 1e-9)
    return {"warm_tok_s": warm_value, "cold_tok_s": round(cold, 1), "cold_over_warm": round(cold / warm_value, 3),
            "cold": "weights evicted from L2 before every position by streaming 1.5 x L2 of scratch through the layer "
                    "cluster's shared memory; the flush time is excluded, as the reference's --cold"}


def bench_ours(a):
    rank, world, local = rank_env()
    import l3m_b200
    name = a.config
    _, dtype, _, ctx = synth.CONFIGS[name]
    path = synth.make(name, MODEL_DIR)
    prompt = synth.prompt(4, seed=1, vocab=32000)
    positions_per_step = min(a.positions or ctx, ctx)
    max_new = positions_per_step - len(prompt)
    dist = None
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("gloo", timeout=__import__("datetime").timedelta(seconds=600))
    # One batch-1 stream on all `world` GPUs: rank 0 loads the model split over GPUs 0..world-1 and
    # drives every GPU (one host thread per model, as the reference's one process per model); the
    # other ranks only join the barriers and report no work.
    dev_ns, wall_ns, positions, toks, waits = [], [], 0, [], []
    if rank == 0:
        m = l3m_b200.Model(path, cpus=list(range(world)), ctx=ctx, force=True)
        flush = L2Flush()
        sink = []
        for _ in range(a.warmup):
            m.generate(prompt, max_new, temperature=0, on_token=sink.append)
        m.perf()
    if dist:
        dist.barrier()
    with Clocks(local) as clk:
        for _ in range(a.steps if rank == 0 else 0):
            flush()
            t0 = time.perf_counter_ns()
            toks = m.generate(prompt, max_new, temperature=0, on_token=sink.append)
            wall_ns.append(time.perf_counter_ns() - t0)
            dev_ns.append(m.device_ns())
            p = m.perf()
            positions += int(p["tokens"])
            waits.append(p["ns_wait"])
    n_gen = len(toks)
    t_dev, t_wall, total = combine_ranks(dist, sum(dev_ns), sum(wall_ns), positions)
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    if rank:
        return
    value = total / (t_dev * 1e-9)
    e2e = total / (t_wall * 1e-9)
    alg, per_launch_pos = algorithmic_bytes(name, positions_per_step)
    launch_s = (t_dev / a.steps) * 1e-9
    peak, peak_kind = measured_peaks()
    achieved = alg / launch_s / 1e9
    traffic = DECODE_TRAFFIC.get(name)
    out = {
        "metric": "batch-1 decode tok/s", "value": round(value, 1), "unit": "tok/s", "n_gpus": world, "steps": a.steps,
        "warmup": a.warmup, "ms_per_step": round(t_dev / a.steps * 1e-6, 4), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": round(value / PUBLISHED[name], 3) if name in PUBLISHED else None,
        "dtype": {"q8_0": "int8 dot / fp32", "q4_0": "int4 dot / fp32", "mxfp4": "e2m1 dot / fp32", "bf16": "bf16 x bf16 / fp32"}[dtype],
        "data": "synthetic (seeded N(0,0.02) weights, 4 seeded prompt ids)",
        "config": {"workload": f"{name} batch-1 greedy decode, ctx {ctx}, {per_launch_pos} forward passes per step "
                               f"({len(prompt)}-token prompt, {n_gen} generated)", "ctx": ctx, "l2_flush_between_steps": True,
                   "parallelism": (f"one batch-1 stream, output channels split over {world} GPUs (activations exchanged "
                                   "over NVLink 4 times per layer)") if world > 1 else "1 GPU",
                   "table": "sm100a (bit-exact with the reference's scalar path)"},
        "e2e": {"value": round(e2e, 1), "unit": "tok/s", "h2d_bytes_per_step": 4 * len(prompt), "d2h_bytes_per_step": 4 * n_gen,
                "timing": "host wall clock around l3m_generate"},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s", "frac": round(achieved / peak, 4),
                     "traffic": traffic and round(traffic["dram_bytes_per_position"] * per_launch_pos),
                     "traffic_note": traffic["note"] if traffic else "not measured for this config",
                     "peak_kind": peak_kind,
                     "algorithmic_bytes_per_launch": alg},
        "chain_bound": chain_line(l3m_b200.lib(), name, per_launch_pos, len(prompt), launch_s, clk.summary()),
        "gpu_launches": a.steps,
        "clocks": clk.summary(),
        "ns_wait_per_token": round(float(np.mean(waits)), 1) if waits else None,
    }
    if not a.no_cold and world == 1:
        out["residency"] = residency_line(path, ctx, prompt, max_new, out["value"])
    if not a.no_matvec and world == 1:
        out["matvec"] = matvec_line()
    if not a.no_cpu and world == 1:
        out["cpu_baseline"] = reference_cpu(path, ctx, max_new)
    print(json.dumps(out), flush=True)


def bench_reference(a):
    rank, world, _ = rank_env()
    if rank:
        return
    name = a.config
    _, dtype, _, ctx = synth.CONFIGS[name]
    path = synth.make(name, MODEL_DIR)
    if not REF_CLI.exists():
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/l3m was not built (needs the reference sources)"}))
        return
    vals = []
    desc = ""
    for i in range(a.warmup + a.steps):
        out = subprocess.run([str(REF_CLI), "bench", str(path), "--ctx", str(ctx), "-n", "256", "--force", "--md"],
                             capture_output=True, text=True, timeout=900)
        if out.returncode:
            print(json.dumps({"impl": "reference", "unavailable": out.stderr.strip()[:200]}))
            return
        row = out.stdout.splitlines()[2].split("|")
        desc = row[1].strip()
        if i >= a.warmup:
            vals.append(float(row[2]))
    m = re.search(r"on (\d+) cores? \((\w+)\)", desc)
    value = statistics.median(vals)
    print(json.dumps({
        "impl": "reference", "metric": "batch-1 decode tok/s", "value": round(value, 1), "unit": "tok/s", "n_gpus": world,
        "steps": a.steps, "warmup": a.warmup, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": round(value / PUBLISHED[name], 3) if name in PUBLISHED else None, "dtype": dtype, "data": "synthetic",
        "config": {"workload": f"{name} batch-1 greedy decode, ctx {ctx}", "ctx": ctx},
        "cpu_baseline": {"value": round(value, 1), "unit": "tok/s", "cores": int(m.group(1)) if m else None, "kind": "reference",
                         "sample": f"reference `l3m bench --ctx {ctx} -n 256 --force` ({m.group(2) if m else '?'} table), median over steps"},
        "e2e": {"value": round(value, 1), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", default="SmolLM2-135M-q8_0", choices=list(synth.CONFIGS))
    ap.add_argument("--no-cpu", action="store_true", help="skip the cpu_baseline leg")
    ap.add_argument("--no-matvec", action="store_true", help="skip the matvec line of the decode bench")
    ap.add_argument("--no-cold", action="store_true", help="skip the cold-residency measurement of the decode bench")
    ap.add_argument("--positions", type=int, default=0,
                    help="forward passes per step (default: the whole context); small values make a profiling case")
    ap.add_argument("--sweep", action="store_true", help="the matvec sweep instead of decode (one JSON line per case)")
    ap.add_argument("--dtypes", default="bf16,q8_0,q4_0,mxfp4", help="--sweep: the dtypes")
    a = ap.parse_args()
    if a.warmup < 3:
        ap.error("--warmup must be at least 3")
    if a.sweep:
        bench_sweep(a)
        return
    (bench_reference if a.impl == "reference" else bench_ours)(a)


if __name__ == "__main__":
    main()
