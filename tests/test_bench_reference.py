"""bench.py's reference arm on the CPU: the JSON line it prints, and that it
never loads this library (the arm must time the reference's CPU code, or the
pinned port where the reference's function cannot be called). CPU only."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _run(*args):
    out = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", *args],
                         cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [l for l in out.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1, out.stdout
    return json.loads(lines[0])


def test_attnres_reference_line():
    d = _run("--config", "attnres", "--steps", "1", "--warmup", "0")
    assert d["impl"] == "reference" and d["metric"] == "attention-residual positions/s"
    assert d["unit"] == "positions/s" and d["value"] > 0 and d["higher_is_better"] is True
    assert d["config"]["positions"] == 576 and d["config"]["sources"] == 8 and d["config"]["hidden"] == 7168
    assert d["cpu_baseline"]["kind"] == "port" and d["cpu_baseline"]["value"] == d["value"]
    assert d["e2e"] == {"value": d["value"], "unit": "positions/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


def test_configs_without_cpu_path_are_unavailable():
    for cfg in ("c3", "tc"):
        d = _run("--config", cfg)
        assert d["impl"] == "reference" and "unavailable" in d


def test_reference_arm_does_not_load_the_library():
    code = ("import runpy, sys\n"
            "sys.argv = ['bench.py', '--impl', 'reference', '--config', 'attnres', '--steps', '1', '--warmup', '0']\n"
            "runpy.run_path('bench.py', run_name='__main__')\n"
            "mods = [m for m in sys.modules if m == 'k3xb' or m.startswith('k3xb.')]\n"
            "maps = open('/proc/self/maps').read()\n"
            "assert not mods, mods\n"
            "assert 'libk3xb' not in maps, 'libk3xb loaded'\n")
    out = subprocess.run([sys.executable, "-c", code], cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stderr[-2000:]
