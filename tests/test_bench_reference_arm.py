"""The bench's reference arm on the CPU: the line the driver reads, single and 2-rank.

``bench.py --impl reference`` times the CPU port of the reference's naive decode on
the host cores (rank 0 only) and prints one JSON line with the headline metric's
name and unit, a cpu_baseline object and an e2e object with no host<->device bytes.
"""

from __future__ import annotations

import json
import os
import socket
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _check_line(line: dict, n_gpus: int) -> None:
    import bench

    assert line["impl"] == "reference"
    assert line["metric"] == bench.METRIC and line["unit"] == bench.UNIT
    assert line["n_gpus"] == n_gpus and line["higher_is_better"] is True
    assert line["value"] > 0 and line["ms_per_step"] > 0
    cb = line["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and cb["value"] == line["value"]
    assert line["e2e"] == {"value": line["value"], "unit": line["unit"], "h2d_bytes_per_step": 0,
                           "d2h_bytes_per_step": 0}


def test_reference_arm_prints_one_contract_line():
    out = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--steps", "1",
                          "--warmup", "0"], capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [l for l in out.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1
    _check_line(json.loads(lines[0]), 1)


def test_reference_arm_under_two_ranks_prints_once():
    env = dict(os.environ, OMP_NUM_THREADS="2")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
           "--master-addr", "127.0.0.1", "--master-port", str(_free_port()), str(ROOT / "bench.py"),
           "--impl", "reference", "--gpus", "2", "--steps", "1", "--warmup", "0"]
    out = subprocess.run(cmd, capture_output=True, text=True, timeout=900, cwd=ROOT, env=env)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [l for l in out.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1  # rank 0 alone runs and prints; rank 1 exits without work
    _check_line(json.loads(lines[0]), 2)


def test_reference_arm_never_loads_the_product_library():
    """The reference arm times the CPU port only: the minisgl_b200 package (whose import
    loads libb200attn.so) is never imported, and the library is not mapped."""
    code = (
        "import runpy, sys\n"
        "sys.argv = ['bench.py', '--impl', 'reference', '--steps', '1', '--warmup', '0']\n"
        "runpy.run_path('bench.py', run_name='__main__')\n"
        "maps = open('/proc/self/maps').read()\n"
        "print('PKG', any(m == 'minisgl_b200' or m.startswith('minisgl_b200.') for m in sys.modules))\n"
        "print('LIB', 'libb200attn' in maps)\n"
    )
    out = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert out.returncode == 0, out.stderr[-2000:]
    assert "PKG False" in out.stdout and "LIB False" in out.stdout, out.stdout[-500:]
    line = json.loads([l for l in out.stdout.splitlines() if l.startswith("{")][0])
    assert line["warmup"] >= 3  # the same warm-up rule as the GPU arm
