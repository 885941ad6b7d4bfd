"""bench.py --sweep on the CPU: one JSON line per sweep case with the reference's kernels timed on
this host (1 core and every core) as cpu_baseline; without a GPU the device fields are absent."""
import json
import subprocess
import sys
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parent.parent


def test_sweep_lines_carry_the_reference_cpu_baseline():
    if not (ROOT / "oracle" / "_ref" / "libsweep_ref.so").exists():
        pytest.skip("oracle/_ref/libsweep_ref.so not built")
    out = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--sweep", "--dtypes", "q4_0"], capture_output=True, text=True,
                         timeout=600, cwd=ROOT)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [json.loads(l) for l in out.stdout.splitlines() if l.startswith("{")]
    assert [(d["m"], d["k"]) for d in lines] == [(288, 288), (768, 288), (2048, 768), (4096, 4096), (32000, 768)]
    for d in lines:
        assert d["metric"] == "matvec GB/s" and d["dtype"] == "q4_0" and d["unit"] == "GB/s" and d["higher_is_better"]
        assert d["bytes"] == d["m"] // 16 * (d["k"] // 32) * 288           # q4_0 tile bytes per 32 inputs
        c = d["cpu_baseline"]
        assert c["kind"] == "reference" and c["cores"] >= 1 and c["value"] > 0 and c["value_1core"] > 0 and c["table"]
        if not torch.cuda.is_available():
            assert "value" not in d
