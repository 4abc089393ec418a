"""bench.py's reference arm runs on the host: its stdout is exactly one JSON line
with the contract's keys (the GPU arm shares the emitter)."""
from __future__ import annotations

import json
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def test_reference_arm_prints_one_json_line():
    r = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--steps", "1",
                        "--warmup", "0"], capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [l for l in r.stdout.splitlines() if l.strip()]
    assert len(lines) == 1, r.stdout
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "config", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["value"] > 0 and d["warmup"] >= 3
    cb = d["cpu_baseline"]
    assert cb["kind"] in ("port", "reference") and cb["cores"] >= 1 and cb["sample"] and cb["value"] == d["value"]
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["d2h_bytes_per_step"] == 0
    assert d["e2e"]["value"] == d["value"] and d["e2e"]["unit"] == d["unit"]


def test_reference_arm_never_loads_the_cuda_library():
    """The reference arm times the reference's algorithm only: the package (and
    with it libsa_b200.so) is never imported in that process."""
    code = (
        "import runpy, sys\n"
        "sys.argv = ['bench.py', '--impl', 'reference', '--steps', '1', '--warmup', '3']\n"
        "runpy.run_path('bench.py', run_name='__main__')\n"
        "maps = open('/proc/self/maps').read()\n"
        "bad = 'libsa_b200' in maps or any(m.startswith('sparseattentioninfer_b200') for m in sys.modules)\n"
        "sys.stderr.write('LOADED\\n' if bad else 'CLEAN\\n')\n"
    )
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    assert "CLEAN" in r.stderr and "LOADED" not in r.stderr


def test_lpt_assignment_balances_and_is_deterministic():
    # bench.py redirects fd 1 when imported: run the pure function from its source instead
    src = (ROOT / "bench.py").read_text()
    start = src.index("def lpt_assign(")
    end = src.index("\ndef ", start + 10)
    ns: dict = {}
    exec(src[start:end], ns)
    lpt = ns["lpt_assign"]
    loads = [9, 1, 7, 3, 5, 5, 2, 8]
    for world in (1, 2, 4, 8):
        bins = lpt(loads, world)
        assert sorted(i for b in bins for i in b) == list(range(8))
        assert bins == lpt(loads, world)
    b2 = lpt(loads, 2)
    assert abs(sum(loads[i] for i in b2[0]) - sum(loads[i] for i in b2[1])) <= 1
