"""bench.py's contract that needs no GPU: the reference arm prints one JSON line and exits 0, and the model
description follows the preset it ran."""
import importlib.util
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_reference_arm_prints_one_json_line():
    out = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--gpus", "1", "--steps", "2",
                          "--warmup", "3"], capture_output=True, text=True, timeout=120, cwd=ROOT)
    assert out.returncode == 0, out.stderr[-1000:]
    lines = [ln for ln in out.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["unavailable"]


def test_model_description_follows_the_preset():
    spec = importlib.util.spec_from_file_location("bench", os.path.join(ROOT, "bench.py"))
    bench = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(bench)
    from bitresearch_b200.config import preset
    assert bench.model_desc(preset("d512").model).startswith("autoresearch GPT d512 depth-8 (4x128 heads, vocab 8192")
    assert "d1280 depth-20 (10x128 heads, vocab 65536" in bench.model_desc(preset("d1280").model)
