"""bench.py's output contract, checked on the CPU through its reference arm.

The driver reads exactly one JSON line from bench.py's standard output; C libraries
that print banners (NCCL's version line) must not get onto that stream. The reference
arm needs no GPU, so it shows the contract here: one line, the keys the driver reads,
and the reference-arm fields.
"""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


# Runs bench.py's main() in this interpreter, then reports whether the CUDA library was
# mapped into the process (it must not be on the reference arm).
_RUN = (
    "import runpy, sys; sys.argv = ['bench.py'] + sys.argv[1:]; "
    "runpy.run_path('bench.py', run_name='__main__'); "
    "loaded = 'libdiskmule_cuda' in open('/proc/self/maps').read(); "
    "sys.stderr.write('CUDA_LIBRARY_LOADED=%d\\n' % loaded)"
)


def test_reference_arm_prints_one_json_line():
    # one token per step keeps the host weights it generates small (its 8 experts)
    r = subprocess.run([sys.executable, "-c", _RUN, "--impl", "reference", "--steps", "1",
                        "--warmup", "0", "--sample", "1"], cwd=ROOT, capture_output=True,
                       text=True, timeout=900)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [l for l in r.stdout.splitlines() if l.strip()]
    assert len(lines) == 1, r.stdout
    d = json.loads(lines[0])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
                "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config",
                "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["impl"] == "reference" and d["value"] > 0
    assert d["cpu_baseline"]["kind"] in ("port", "reference") and d["cpu_baseline"]["cores"] >= 1
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["d2h_bytes_per_step"] == 0
    # the same metric string as the GPU arm's default line (configuration 4)
    sys.path.insert(0, ROOT)
    import bench
    assert d["metric"] == bench.metric_name("glm52", 8192)
    # the reference arm generates its inputs with the oracle library only
    assert "CUDA_LIBRARY_LOADED=0" in r.stderr, r.stderr[-2000:]


def test_roofline_follows_the_arithmetic_intensity():
    sys.path.insert(0, ROOT)
    import bench
    hbm, tensor = (6456.8, "measured"), (1666.2, "measured")
    # Qwen T=512 gate/up: 36.5 FLOP/byte, under the ridge (258) -> HBM
    r = bench.choose_roofline("expert_up", 2.2e10, 6.2e8, 0.228, hbm, tensor, None)
    assert r["bound"] == "hbm" and r["unit"] == "GB/s"
    assert abs(r["achieved"] - 6.2e8 / 0.228e-3 / 1e9) < 1e-6 and abs(r["frac"] - r["achieved"] / 6456.8) < 1e-12
    # Gemma T=4096 gate/up: 613 FLOP/byte -> tensor peak, TFLOP/s
    r = bench.choose_roofline("expert_up", 2.598e11, 4.239e8, 0.718, hbm, tensor, 1.0)
    assert r["bound"] == "tensor" and r["unit"] == "TFLOP/s" and r["traffic"] == 1.0
    assert abs(r["achieved"] - 2.598e11 / 0.718e-3 / 1e12) < 1e-9 and r["flop_per_byte"] > 258
