"""The C ABI from a plain C host: include/*.h compile as pedantic C99 (what cgo, JNI or any FFI
generator reads), and a C program linked against libmi_paged.so gets the host-side results the
ctypes binding gets (tests/abi/consumer.c; no GPU needed)."""

import shutil
import subprocess
from pathlib import Path

import pytest

from mini_infra_b200.build import LIB_PATH

ROOT = Path(__file__).resolve().parents[1]
SOURCE = ROOT / "tests" / "abi" / "consumer.c"
C_FLAGS = ["-std=c99", "-pedantic", "-Wall", "-Wextra", "-Werror"]


@pytest.fixture(scope="module")
def gcc():
    path = shutil.which("gcc")
    if path is None:
        pytest.skip("no C compiler")
    if not LIB_PATH.exists():
        pytest.fail(f"{LIB_PATH} is missing: build it with `python -m mini_infra_b200.build`")
    return path


def test_headers_compile_as_c99(gcc, tmp_path):
    for header in sorted((ROOT / "include").glob("*.h")):
        src = tmp_path / f"only_{header.stem}.c"
        src.write_text(f'#include "{header.name}"\nint main(void) {{ return 0; }}\n')
        run = subprocess.run([gcc, *C_FLAGS, "-I", str(ROOT / "include"), "-c", str(src), "-o", str(tmp_path / "x.o")],
                             capture_output=True, text=True)
        assert run.returncode == 0, f"{header.name} is not plain C99:\n{run.stderr}"


def test_c_program_links_and_gets_host_side_results(gcc, tmp_path):
    exe = tmp_path / "consumer"
    lib_dir = str(LIB_PATH.parent)
    build = subprocess.run([gcc, *C_FLAGS, "-I", str(ROOT / "include"), str(SOURCE), "-L", lib_dir, "-lmi_paged",
                            f"-Wl,-rpath,{lib_dir}", "-o", str(exe)], capture_output=True, text=True)
    assert build.returncode == 0, build.stderr
    run = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    lines = run.stdout.splitlines()
    assert run.returncode == 0, run.stdout + run.stderr
    assert lines and all(line.startswith("ok ") for line in lines), run.stdout
    assert len(lines) == 9
