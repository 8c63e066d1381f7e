"""The JSON line bench.py prints for its reference arm (CpuBackend semantics
on the host cores), checked on the CPU: one line, the keys and types the
benchmark driver reads, and the same metric and unit as the device arm."""

import json
import os
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent


def _run(*args):
    env = dict(os.environ, PYTHONPATH=os.pathsep.join(
        [str(ROOT), str(ROOT / "paged-kv-cache_b200"), os.environ.get("PYTHONPATH", "")]))
    out = subprocess.run([sys.executable, str(ROOT / "bench.py"), *args], cwd=ROOT, env=env,
                         capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [l for l in out.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1, out.stdout[-2000:]
    return json.loads(lines[0])


def test_reference_arm_line():
    d = _run("--impl", "reference", "--steps", "1", "--warmup", "1")
    for key, typ in (("metric", str), ("value", float), ("unit", str), ("n_gpus", int),
                     ("steps", int), ("warmup", int), ("ms_per_step", float),
                     ("higher_is_better", bool), ("scaling", str), ("dtype", str),
                     ("data", str), ("config", dict), ("cpu_baseline", dict), ("e2e", dict)):
        assert isinstance(d[key], typ), key
    assert d["impl"] == "reference"
    assert d["vs_baseline"] is None
    assert (d["steps"], d["warmup"], d["n_gpus"]) == (1, 1, 1)
    assert d["unit"] == "tokens/s" and d["higher_is_better"] is True
    assert "reshape_and_cache" in d["metric"]
    assert d["value"] > 0 and d["ms_per_step"] > 0
    cb = d["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and cb["value"] == d["value"]
    assert isinstance(cb["sample"], str) and cb["sample"]
    e2e = d["e2e"]
    assert e2e["value"] == d["value"] and e2e["unit"] == d["unit"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0
    assert "workload" in d["config"]
    # The same config as the device arm's line, plus the thread count; the
    # single-threaded figure of CpuBackend (which is single-threaded) beside it.
    assert d["config"]["host_threads"] == cb["cores"]
    assert d["config"]["tokens_per_step"] == 65536 and d["config"]["layers"] == 28
    assert d["config"]["workload"].startswith("ragged prefill chunk x1")
    st = d["single_thread"]
    assert st["cores"] == 1 and st["value"] > 0 and st["unit"] == "tokens/s"


def test_reference_arm_maps_no_device_library():
    """The reference arm runs only CpuBackend semantics (the oracle): it must
    not map the device library, which `import pagedkv` no longer loads."""
    code = (
        "import sys; sys.argv = ['bench.py', '--impl', 'reference', '--steps', '1', '--warmup', '1']\n"
        "import bench; bench.main()\n"
        "maps = [l.split()[-1] for l in open('/proc/self/maps') if '.so' in l]\n"
        "print('LIBS', sorted(set(m for m in maps if 'pagedkv_b200' in m or 'liboracle' in m)))\n")
    env = dict(os.environ, PYTHONPATH=os.pathsep.join(
        [str(ROOT), str(ROOT / "paged-kv-cache_b200"), os.environ.get("PYTHONPATH", "")]))
    out = subprocess.run([sys.executable, "-c", code], cwd=ROOT, env=env, capture_output=True,
                         text=True, timeout=600)
    assert out.returncode == 0, out.stderr[-2000:]
    libs = [l for l in out.stdout.splitlines() if l.startswith("LIBS")][0]
    assert "liboracle.so" in libs and "pagedkv_b200" not in libs
