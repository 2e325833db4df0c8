"""The benchmark's reference arm runs on the host alone: `bench.py --impl
reference` times the reference's CPU path (decode primitives + FP32 loop) on
a row sample of the format sweep and prints one JSON line with the fields the
benchmark contract names.  Checked here without a GPU."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_reference_arm_prints_contract_line():
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--steps", "1",
                        "--warmup", "3"], capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    line = json.loads(r.stdout.strip().splitlines()[-1])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "impl", "cpu_baseline", "e2e"):
        assert key in line, key
    assert line["impl"] == "reference"
    assert line["value"] > 0 and line["unit"] == "TFLOP/s"
    assert line["steps"] == 1 and line["warmup"] >= 3
    cb = line["cpu_baseline"]
    assert cb["kind"] in ("reference", "port") and cb["cores"] >= 1 and cb["value"] == line["value"]
    assert line["e2e"] == {"value": line["value"], "unit": line["unit"], "h2d_bytes_per_step": 0,
                           "d2h_bytes_per_step": 0}
    assert "workload" in line["config"]


def _bench_module():
    import importlib.util
    spec = importlib.util.spec_from_file_location("bench_mod", os.path.join(ROOT, "bench.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_reference_arm_config_matches_ours():
    """Both arms name the same workload object, so the two lines compare."""
    bench = _bench_module()
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--steps", "1",
                        "--warmup", "3"], capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    line = json.loads(r.stdout.strip().splitlines()[-1])
    assert line["config"] == bench.sweep_config(4096, 4096, 4096, 1)


def test_targets_object_is_compact():
    """The target figures close the line in a few hundred characters, so they
    survive in the tail of the output that is kept."""
    bench = _bench_module()
    sq = {"pct_f16_dense_peak_nominal": 75.0}
    mlp = [{"W": w, "fmt": f, "tokens": t, "fused_pct_hbm": 50.0 + t}
           for w in ("14336x4096", "4096x14336") for f in ("e4m3", "e2m1") for t in (1, 16, 128, 2048)]
    formats = {k: {"fused_tflops": 1.0, "unfused_tflops": 2.0} for k in bench.FORMATS}
    formats.update({f"native_{k}": {"pct_fp8_dense_peak": 50.0} for k in ("e4m3", "e2m1")})
    line = {"fp4_8192_fused": sq, "fp4_8192_fused_after_load": sq, "e4m3_8192_fused": sq, "weight_only_mlp": mlp,
            "formats": formats, "int8_4096": {"pct_i8_dense_peak": 40.0},
            "sharded_weight_gemm": {"world": 1, "ms": 9.9, "check": {"pass": True, "rel_frob_max_vs_fp64": 1e-6}},
            "config_256_e4m3": {"us": 5.0, "rel_frob_vs_unquantized_fp32": 0.025},
            "cpu_baseline": {"naive_single_thread": {"256^3": {"ms": 15.0}, "512^3": {"ms": 120.0}}},
            "native_8192": {"e4m3_pct_fp8_dense_peak": 60.04, "i8_pct_i8_dense_peak": 55.55}}
    t = bench.targets(line)
    assert t["skinny_pct_hbm_min_max"]["14336x4096_e4m3"] == [51.0, 66.0]
    assert t["native_8192_pct_dense"] == {"e4m3": 60.0, "i8": 55.5}
    assert t["sharded"]["check_pass"] is True
    assert len(json.dumps(t)) < 1200


def test_targets_sharded_two_paths():
    """On N GPUs the sharded section reports the peer-store path and, beside
    it, the NCCL path; both reach the targets object with their checks."""
    bench = _bench_module()
    sq = {"pct_f16_dense_peak_nominal": 75.0}
    formats = {k: {"fused_tflops": 1.0, "unfused_tflops": 2.0} for k in bench.FORMATS}
    formats.update({f"native_{k}": {"pct_fp8_dense_peak": 50.0} for k in ("e4m3", "e2m1")})
    check = {"pass": True, "rel_frob_max_vs_fp64": 2.08e-4}
    line = {"fp4_8192_fused": sq, "fp4_8192_fused_after_load": sq, "e4m3_8192_fused": sq, "weight_only_mlp": [],
            "formats": formats, "int8_4096": {"pct_i8_dense_peak": 40.0},
            "sharded_weight_gemm": {"world": 8, "ms": 1.796, "gemm_only_ms": 1.166, "check": check,
                                    "nccl": {"chunks": 4, "ms": 2.40, "allgather_only_ms": 1.34, "check": check}},
            "config_256_e4m3": {"us": 12.3, "rel_frob_vs_unquantized_fp32": 0.0254}}
    t = bench.targets(line)
    assert t["sharded"]["world"] == 8 and t["sharded"]["ms"] == 1.796 and t["sharded"]["check_pass"] is True
    assert t["sharded"]["nccl"] == {"ms": 2.4, "allgather_only_ms": 1.34, "check_pass": True}
    assert len(json.dumps(t)) < 1200
