"""CPU: the bench's host-side bookkeeping (algorithmic bytes, clock summary, workload defaults)."""
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))


def test_qgemm_algorithmic_bytes_config1():
    import bench
    total, n = bench.qgemm_algorithmic_bytes("gq8")
    assert n == 97   # 4 quantized linears x 24 layers + output_proj
    # one fused QKV launch: W_packed + 4MK + 4MN + 4N with M=257, K=768, N=2304
    M, K, N = 257, 768, 2304
    qkv = N * K * 34 / 32 + 4 * M * K + 4 * M * N + 4 * N
    assert qkv < total / 24
    # Q4_K packs tighter than Q8_0
    assert bench.qgemm_algorithmic_bytes("gq4")[0] < total


def test_clock_summary_flags_throttle_reasons():
    import bench
    c = bench.ClockSampler(0)
    c.rows = [["0", "1965", "1965", "700", "0x0", "Not Active", "Not Active", "Not Active", "Not Active"],
              ["0", "1800", "1965", "990", "0x4", "Not Active", "Not Active", "Not Active", "Active"]]
    s = c.summary()
    assert s["sm_max_mhz"] == 1965.0
    assert s["samples"] == 2
    assert s["reasons"] == ["sw_power_cap"]
    assert bench.ClockSampler(0).summary()["reasons"] == ["unsampled"]


def test_bench_cli_lists_the_workloads():
    out = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--help"], capture_output=True, text=True,
                         timeout=120).stdout
    for w in ("c1", "c4", "c5", "sweep"):
        assert w in out
    assert "--impl" in out


def test_reference_arm_models_do_not_load_the_cuda_library(tmp_path):
    """The reference arm builds its models with the oracle's packers: libmgcuda.so stays unmapped."""
    code = f"""
import os, sys
sys.path.insert(0, {str(ROOT)!r})
os.environ["MGC_BENCH_DIR"] = {str(tmp_path)!r}
import bench
bench.MODEL_DIR = bench.Path({str(tmp_path)!r})
p, t = bench.ensure_model("gq8", 1, twin=True, packers=bench._oracle_packers())
assert p.exists() and t.exists()
maps = open("/proc/self/maps").read()
assert "libmgcuda" not in maps, "the CUDA library was loaded"
print("ok")
"""
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and "ok" in r.stdout, r.stderr[-2000:]
