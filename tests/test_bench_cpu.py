"""CPU: bench.py's reference arm (the reference's exact PyTorch path on the host cores) prints
one JSON line with the keys the bench contract names, on the same metric and workload as the
device arm."""
import json
import os
import subprocess
import sys

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_reference_arm_json_line():
    out = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "1", "--warmup", "0"],
                         cwd=REPO, capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [ln for ln in out.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    for key in ("impl", "metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["impl"] == "reference" and d["steps"] == 1 and d["higher_is_better"] is False
    assert d["value"] > 0 and d["cpu_baseline"]["cores"] >= 1 and d["cpu_baseline"]["kind"] == "port"
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["d2h_bytes_per_step"] == 0
    assert "workload" in d["config"]


def test_native_stdout_kept_off_the_json_line():
    """What a native library writes on file descriptor 1 while the process group is created
    (NCCL prints its version banner there) goes to stderr: rank 0's stdout stays one JSON line."""
    code = ("import os, sys; sys.path.insert(0, %r); import bench\n"
            "with bench._stdout_to_stderr():\n"
            "    os.write(1, b'banner from a native library\\n')\n"
            "    print('python print inside')\n"
            "print('{\"after\": 1}')\n") % REPO
    out = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=300)
    assert out.returncode == 0, out.stderr[-2000:]
    assert out.stdout.splitlines() == ['{"after": 1}']
    assert "banner from a native library" in out.stderr and "python print inside" in out.stderr
