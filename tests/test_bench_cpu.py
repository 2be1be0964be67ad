"""bench.py's reference arm runs on the host cores (no GPU) and prints one JSON
line with the keys the benchmark contract names.  With the reference installed
in baseline/_ref it times the reference's own code: the whole forward at a
small S, and above S=10 its pieces on bounded samples, composed (an
extrapolation, labelled as one; ms_per_step is then the sample's own time)."""
import json
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def _run(frames, steps):
    out = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--frames",
                          str(frames), "--steps", str(steps), "--warmup", "0"], capture_output=True,
                         text=True, timeout=900, cwd=ROOT)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [ln for ln in out.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "impl", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["impl"] == "reference" and d["n_gpus"] == 1 and d["higher_is_better"] is False
    assert d["value"] > 0 and d["unit"] == "ms" and d["dtype"] == "fp32"
    assert d["config"]["workload"] == f"gpa_vggt_forward_S{frames}"
    assert d["cpu_baseline"]["kind"] in ("reference", "port") and d["cpu_baseline"]["cores"] >= 1
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["value"] == d["value"]
    return d


def test_reference_arm_direct_forward_at_small_s():
    d = _run(2, 1)
    if d["cpu_baseline"]["kind"] == "reference":
        assert d["extrapolated"] is False
        assert abs(d["ms_per_step"] - d["value"]) <= 0.2 * d["value"]


def test_reference_arm_composes_above_s10():
    d = _run(12, 2)
    assert d["extrapolated"] is True
    assert d["ms_per_step"] < d["value"]      # a sample step is cheaper than the forward it stands for
    assert d["steps_values_ms"]["min"] <= d["value"] <= d["steps_values_ms"]["max"]


@pytest.mark.skipif(not (ROOT / "baseline" / "_ref" / "merging" / "merge.py").exists(),
                    reason="the reference is not installed in baseline/_ref")
def test_composition_tracks_the_direct_forward():
    """The composed estimate at S=4 is within 35% of the reference's whole S=4
    forward (the check that the schedule and the pieces cover the forward)."""
    import torch
    sys.path.insert(0, str(ROOT))
    from oracle import reference_runs as RR
    torch.set_num_threads(torch.get_num_threads())
    model = RR.build_cpu_model()
    RR.forward_ms(model, 4)
    direct = min(RR.forward_ms(model, 4) for _ in range(2))
    comp = RR.Composer(4)
    composed = min(comp.compose_ms(comp.parts(reps=1)) for _ in range(2))
    print(f"S=4: direct {direct:.0f} ms, composed {composed:.0f} ms")
    assert abs(composed - direct) <= 0.35 * direct
