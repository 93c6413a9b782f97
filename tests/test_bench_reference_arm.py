"""The bench's reference arm (the reference's own CPU kernels, or the C
restatement when they are not built) runs here without a GPU and prints one
JSON line with the keys the driver reads."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_reference_arm_json_line():
    out = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "1",
                          "--warmup", "1"], cwd=ROOT, capture_output=True, text=True,
                         timeout=600, env=dict(os.environ, INFERC_THREADS="4"))
    assert out.returncode == 0, out.stderr[-2000:]
    line = json.loads(out.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference"
    assert line["metric"] == "encoder seqs/s (DistilBERT-arch seq128)"
    assert line["value"] > 0 and line["unit"] == "seq/s"
    assert line["e2e"]["value"] == line["value"]
    assert line["cpu_baseline"]["kind"] in ("reference", "port")
