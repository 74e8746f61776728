"""The drop-in claim for the control plane, shown with the reference's own tests.

The reference's unit tests of its block manager and scheduler (``tests/unit/test_block_manager.py``
and ``tests/unit/test_scheduler.py`` of yurun00/mini-infra-qwen3 v0.7.0: FIFO block reuse, the null
block, atomic allocation failure, admission, pool sizing, the counters, the arrival / waiting /
running queues, the prefill-first, token-budget and chunked-prefill policies, decode protection and
the loud failure on block exhaustion) run unmodified, from the reference checkout, with
``mini_infra.core`` aliased to ``mini_infra_b200.core`` (``tests/reference_alias.py``).  Their
``conftest.py`` is not loaded: its fixtures build the reference's CPU model, which these two files
do not use.

The checkout is taken from ``MINI_INFRA_REFERENCE`` or, by default, a ``reference`` directory next
to this repository; without it (as on a GPU box) the test is skipped.  CPU only.
"""

import os
import re
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
REFERENCE = Path(os.environ.get("MINI_INFRA_REFERENCE", ROOT.parent / "reference"))
FILES = [REFERENCE / "tests" / "unit" / name for name in ("test_block_manager.py", "test_scheduler.py")]


@pytest.mark.skipif(not all(f.exists() for f in FILES), reason="no reference checkout next to this repository")
def test_reference_control_plane_tests_pass_unchanged(tmp_path):
    env = dict(os.environ)
    env["PYTHONPATH"] = os.pathsep.join([str(ROOT / "tests"), str(ROOT / "mini-infra-qwen3_b200")])
    run = subprocess.run(
        [sys.executable, "-m", "pytest", "-q", "--noconftest", "-p", "reference_alias", "-p", "no:cacheprovider",
         "-c", os.devnull, "--rootdir", str(tmp_path), *map(str, FILES)],
        capture_output=True, text=True, timeout=300, cwd=tmp_path, env=env)
    tail = run.stdout[-3000:] + run.stderr[-2000:]
    assert run.returncode == 0, tail
    passed = re.search(r"(\d+) passed", run.stdout)
    assert passed and int(passed.group(1)) >= 40 and "failed" not in run.stdout.splitlines()[-1], tail
