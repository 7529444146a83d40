"""CPU checks of bench.py's output contract: the result line is the only
thing on stdout, whatever else the process writes to file descriptor 1; the
storage-ceiling reader reads whole files; peaks come from the measured file."""
import importlib.util
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
BENCH = os.path.join(ROOT, "bench.py")


def _bench_module():
    spec = importlib.util.spec_from_file_location("bench_under_test", BENCH)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_result_line_alone_on_stdout():
    code = f"""
import importlib.util, os, sys
spec = importlib.util.spec_from_file_location("b", {BENCH!r})
b = importlib.util.module_from_spec(spec); spec.loader.exec_module(b)
print("before")
b.keep_stdout_for_result()
print("a library print")
os.write(1, b"NCCL version 0.0.0+cuda0.0\\n")
b.emit({{"metric": "m", "value": 1.5}})
print("after")
"""
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stderr
    lines = r.stdout.splitlines()
    assert lines[-1] == json.dumps({"metric": "m", "value": 1.5})
    assert "NCCL" not in r.stdout and "library" not in r.stdout and "after" not in r.stdout
    assert "NCCL version" in r.stderr and "a library print" in r.stderr


def test_plain_read_reads_the_whole_file(tmp_path):
    b = _bench_module()
    p = tmp_path / "f.bin"
    data = os.urandom((3 << 20) + 12345)
    p.write_bytes(data)
    t = b.plain_read_seconds(str(p), len(data), drop=False, lanes=3, piece=1 << 20)
    assert t > 0
    t2 = b.plain_read_seconds(str(p), len(data), drop=True, lanes=8, piece=8 << 20)
    assert t2 > 0


def test_peaks_from_measured_file():
    b = _bench_module()
    peaks, src = b.measured_peaks()
    if os.path.exists(os.path.join(ROOT, "MEASURED_PEAKS.json")):
        assert src == "measured"
        assert peaks["bf16_tflops"] > 1000 and peaks["hbm_gbs"] > 4000
    else:
        assert src == "fallback" and peaks["bf16_tflops"] == 1590.0
