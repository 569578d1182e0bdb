"""bench.py's reference arm (the CPU restatement of the reference's ggml
numerics, timed on the host) prints one JSON line with the contract's keys
and honours --steps / --warmup.  No GPU."""
import json
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent


def test_reference_arm_json_line():
    r = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--steps", "1",
                        "--warmup", "3"], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    line = json.loads(r.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference" and line["metric"] == "qwen2_decode_tokens_per_s"
    assert line["unit"] == "tokens/s" and line["higher_is_better"] is True
    assert line["steps"] == 1 and line["warmup"] == 3 and line["value"] > 0
    for k in ("cpu_baseline", "e2e", "config"):
        assert k in line
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["cpu_baseline"]["kind"] == "port"
