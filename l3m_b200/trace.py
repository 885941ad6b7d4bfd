"""Per-phase timing of the decode kernel, from the cycle stamps it writes when L3M_TRACE is set.

    python -m l3m_b200.trace [--config SmolLM2-135M-q8_0] [--out /tmp/l3m_trace.bin] [--ctas 0-15]

Runs one greedy generation (the bench workload: the config's context, a 4-token prompt, the rest
generated) of a synthetic model through ``l3m_b200.Model`` with tracing on, then prints for the two
traced CTAs (CTA 0 of the layer cluster, and the first helper CTA, or the last CTA of the layer
cluster when the launch has no helpers) the median time, over layers and over the positions from 50
on, of every traced event after the layer's start, the layer and token periods, and the head step. Times are SM cycles converted at the clock the header records (the
maximum SM clock; the bench's clock samples show the part runs there under this load).

With ``--ctas`` (a range of the layer cluster's CTAs) it traces each of those CTAs in turn
(``L3M_TRACE_CTA``, one load and two generations per CTA) and prints one column per CTA: the median
time of every layer event after that CTA's own layer start. The SM cycle counters of different SMs
are not aligned, so columns compare durations, not instants: every CTA passes an exchange barrier
when the last bytes land, so the CTA with the shortest barrier wait is the one the others wait for.
"""
import argparse
import os
import sys

import numpy as np

# Event ids as stamped in csrc/decode.cu (per position and layer; the head uses layer index n_layers).
LAYER_EVENTS = {
    16: "Q   rmsnorm (head CTAs: K/V copies issued meanwhile)", 17: "Q   prepare", 18: "Q   weight copy waited", 19: "Q   matvec",
    27: "Q   bias", 1: "Q   exchanged", 2: "    barrier 1, wo copy issued",
    14: "A   RoPE + K/V row", 15: "A   attention", 3: "A   exchanged", 4: "    barrier 2",
    20: "B   prepare", 21: "B   weight copy waited", 22: "B   matvec", 28: "B   bias", 5: "B   exchanged", 6: "    barrier 3, up/gate copy issued",
    7: "C   x += proj, rmsnorm", 26: "C   prepare", 12: "C   weight copy waited", 13: "C   up/gate matvec", 29: "C   next copy issued",
    8: "C   SiLU gate exchanged", 9: "    barrier 4",
    23: "D   prepare", 24: "D   weight copy waited", 25: "D   matvec", 30: "D   bias", 10: "D   exchanged, next qkv copy issued",
    11: "    barrier 5, x += down (layer end)",
}
HEAD_EVENTS = {3: "rmsnorm + prepare", 4: "-", 5: "matvec", 1: "argmax slot", 2: "token agreed"}


def summarize(path, first=50):
    raw = open(path, "rb").read()
    hdr = np.frombuffer(raw[:32], np.int32)
    ctx, L, _, last, cta0, cta1, E, khz = (int(v) for v in hdr)
    t = np.frombuffer(raw[32:], np.uint64).reshape(2, ctx, L + 1, E).astype(np.float64) / (khz / 1e6)   # ns
    lines = [f"clock {khz / 1000:.0f} MHz; positions {first}..{last - 1}; medians in ns after the layer start"]
    for slot, cta in enumerate((cta0, cta1)):
        tt = t[slot, first:last]
        lines.append(f"-- CTA {cta}")
        rows = []
        for ev, name in LAYER_EVENTS.items():
            ok = (tt[:, :L, ev] > 0) & (tt[:, :L, 0] > 0)
            if ok.any():
                rows.append((np.median((tt[:, :L, ev] - tt[:, :L, 0])[ok]), name))
        for v, name in sorted(rows):
            lines.append(f"   {v:8.0f}  {name}")
        h = tt[:, L]
        if (tt[:, :L, 0] > 0).any():                                    # a CTA of the layer cluster
            lay = tt[:, 1:L, 0] - tt[:, :L - 1, 0]
            tok = np.diff(tt[:, 0, 0])
            lines.append(f"   layer period {np.median(lay):.0f} ns, token period {np.median(tok):.0f} ns")
            lines.append(f"   head (ns): x published to token agreed {np.median(h[:, 2] - h[:, 0]):.0f}")
            if (h[:, 6] > 0).any():                                     # several clusters: where CTA 0 waits
                parts = [f"{name} {np.median(h[:, e] - h[:, p]):.0f}" for p, e, name in
                         ((0, 1, "own slot"), (1, 6, "every arrival seen"), (6, 7, "slots reduced"), (7, 2, "token agreed"))]
                lines.append("   head steps (ns): " + ", ".join(parts))
        else:                                                           # a helper: its head step from the published x
            parts = [f"{HEAD_EVENTS[e]} {np.median(h[:, e] - h[:, p]):.0f}" for p, e in ((0, 3), (3, 4), (4, 5), (5, 1))]
            lines.append("   head step (ns): " + ", ".join(parts))
    return "\n".join(lines)


def medians(path, first=50):
    """{event: median ns after the layer start} of the traced layer CTA (slot 0)."""
    raw = open(path, "rb").read()
    ctx, L, _, last, _, _, E, khz = (int(v) for v in np.frombuffer(raw[:32], np.int32))
    tt = (np.frombuffer(raw[32:], np.uint64).reshape(2, ctx, L + 1, E).astype(np.float64) / (khz / 1e6))[0, first:last]
    out = {}
    for ev in LAYER_EVENTS:
        ok = (tt[:, :L, ev] > 0) & (tt[:, :L, 0] > 0)
        if ok.any():
            out[ev] = float(np.median((tt[:, :L, ev] - tt[:, :L, 0])[ok]))
    out["period"] = float(np.median(tt[:, 1:L, 0] - tt[:, :L - 1, 0]))
    return out


def per_cta(config, ctas, out, models):
    """One column per layer CTA (see the module docstring)."""
    import l3m_b200
    from l3m_b200 import synth
    _, _, _, ctx = synth.CONFIGS[config]
    path = synth.make(config, models)
    prompt = synth.prompt(4, seed=1, vocab=32000)
    cols = {}
    for c in ctas:
        os.environ["L3M_TRACE_CTA"] = str(c)
        m = l3m_b200.Model(str(path), ctx=ctx, force=True)
        for _ in range(2):
            m.generate(prompt, ctx - len(prompt), temperature=0)
        m.close()
        cols[c] = medians(out)
    order = sorted(LAYER_EVENTS, key=lambda e: cols[ctas[0]].get(e, 1e18))
    lines = [f"{config}: median ns after each CTA's layer start", "event".ljust(44) + "".join(f"{c:>7d}" for c in ctas)]
    for ev in order:
        lines.append(LAYER_EVENTS[ev][:43].ljust(44) + "".join(f"{cols[c][ev]:7.0f}" if ev in cols[c] else "      -" for c in ctas))
    lines.append("layer period".ljust(44) + "".join(f"{cols[c]['period']:7.0f}" for c in ctas))
    return "\n".join(lines)


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--config", default="SmolLM2-135M-q8_0")
    ap.add_argument("--out", default="/tmp/l3m_trace.bin")
    ap.add_argument("--models", default="/tmp/l3m_bench")
    ap.add_argument("--ctas", default=None, help="a range of layer CTAs, e.g. 0-15: one column each")
    a = ap.parse_args()
    os.environ["L3M_TRACE"] = a.out
    if a.ctas:
        lo, _, hi = a.ctas.partition("-")
        print(per_cta(a.config, list(range(int(lo), int(hi or lo) + 1)), a.out, a.models))
        return 0
    import l3m_b200
    from l3m_b200 import synth
    _, _, _, ctx = synth.CONFIGS[a.config]
    path = synth.make(a.config, a.models)
    m = l3m_b200.Model(str(path), ctx=ctx, force=True)
    prompt = synth.prompt(4, seed=1, vocab=32000)
    for _ in range(2):                                   # the second run is the one summarized
        m.perf()
        m.generate(prompt, ctx - len(prompt), temperature=0)
    dev = m.device_ns()
    p = m.perf()
    print(f"{a.config}: {p['tokens'] * 1e9 / dev:.1f} tok/s (device), {1e9 / p['ns_token']:.1f} tok/s (wall), "
          f"ns_wait {p['ns_wait']:.0f} per token")
    print(summarize(a.out))
    return 0


if __name__ == "__main__":
    sys.exit(main())
