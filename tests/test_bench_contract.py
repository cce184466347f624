"""bench.py's contract, checked on the CPU: the default run covers the five
BASELINE configurations with the mapreduce headline last, and the reference
arm prints the same `config` object as this library's arm for the same N (so
a run pair compares like with like)."""
import json
import subprocess
import sys

from conftest import ROOT

sys.path.insert(0, str(ROOT))
import bench  # noqa: E402


def test_default_kinds_cover_the_five_configs_with_the_headline_last():
    assert sorted(bench.BASELINE_KINDS) == ["gather", "histogram", "matmul", "reduce", "vadd"]
    assert bench.BASELINE_KINDS[-1] == "reduce"


def test_config_objects_name_the_workload_and_the_parallelism():
    for kind in bench.BASELINE_KINDS:
        one, two = bench.config_of(kind, 1), bench.config_of(kind, 2)
        assert one["workload"] == two["workload"] and "configs[" in one["workload"]
        assert one["parallelism"] == "single GPU" and two["parallelism"].startswith("dp2")
        assert "l2" in one
    assert "REDUCED SIZE" in bench.config_of("reduce", 1, 1 << 20)["workload"]


def test_reference_arm_prints_the_same_config():
    r = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--kernel", "vadd",
                        "--steps", "2", "--warmup", "1"], capture_output=True, text=True, timeout=300, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    line = json.loads([ln for ln in r.stdout.splitlines() if ln.startswith("{")][-1])
    assert line["impl"] == "reference"
    assert line["config"] == bench.config_of("vadd", 1)
    assert line["metric"] == "vadd HBM GB/s" and line["unit"] == "GB/s" and line["higher_is_better"]
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["d2h_bytes_per_step"] == 0
    assert line["cpu_baseline"]["kind"] == "port" and line["cpu_baseline"]["cores"] >= 1


def test_clock_sampler_reports_a_sample_for_a_short_region(tmp_path, monkeypatch):
    # a fake nvidia-smi that prints one CSV row every 50 ms after a slow start,
    # like the real one; a region shorter than one period still gets a sample
    fake = tmp_path / "nvidia-smi"
    fake.write_text("#!/bin/sh\nsleep 0.3\nwhile true; do echo '0, 1965, 1965, 700.0, 0x0, Not Active, "
                    "Not Active, Not Active, Active'; sleep 0.05; done\n")
    fake.chmod(0o755)
    monkeypatch.setenv("PATH", f"{tmp_path}:" + __import__("os").environ["PATH"])
    c = bench.ClockSampler(0).start()
    info = c.stop()
    assert info is not None and info["samples"] >= 1
    assert info["sm_mhz"] == 1965.0 and info["reasons"] == ["sw_power_cap"]
