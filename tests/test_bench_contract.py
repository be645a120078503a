"""bench.py's JSON-line contract, checked on the CPU through the reference
arm (`--impl reference`, the reference's own CPU loops): one JSON line with
the metric, unit and config the GPU arm reports, `impl`, a `cpu_baseline`
describing the run and an `e2e` object with zero transfer bytes."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_reference_arm_prints_one_contract_line():
    proc = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "2",
                           "--warmup", "1"], cwd=ROOT, capture_output=True, text=True,
                          timeout=600)
    assert proc.returncode == 0, proc.stderr[-2000:]
    lines = [ln for ln in proc.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, proc.stdout
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    assert d["metric"].startswith("row-op HBM GB/s")
    assert d["unit"] == "GB/s" and d["higher_is_better"] is True
    assert d["n_gpus"] == 1 and d["steps"] == 2 and d["warmup"] == 1
    assert d["value"] > 0 and d["ms_per_step"] > 0
    assert d["cpu_baseline"]["kind"] in ("reference", "port")
    assert d["cpu_baseline"]["cores"] >= 1 and d["cpu_baseline"]["value"] == d["value"]
    assert d["e2e"] == {"value": d["value"], "unit": "GB/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}
    import bench

    assert d["config"]["workload"] == bench.WORKLOAD  # same config as the GPU arm


def test_rotation_sets_exceed_twice_l2():
    """Timed inputs rotate over sets that together exceed 2x L2 (plus one set),
    within 2 GiB; sets larger than L2 need no rotation beyond that rule."""
    import bench

    for set_bytes in [1 << 20, 8_388_608, 16_764_924, 33_554_432, 67_108_864,
                      134_217_728, 1 << 30, 3 << 30]:
        sets = bench._rotations(set_bytes)
        assert sets >= 1
        assert sets * set_bytes <= max(2 << 30, set_bytes)
        if (2 << 30) // set_bytes > -(-2 * bench.L2_BYTES // set_bytes):
            assert (sets - 1) * set_bytes >= 2 * bench.L2_BYTES
