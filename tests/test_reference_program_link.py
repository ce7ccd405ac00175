"""The reference's own test program (advanced/neural_layer/src/npl_test.cpp),
built by `make -C oracle reftest` where it lies, against this repository's
include/neural_primitives.h and linked to libnpl_b200.so: every npl_* symbol it
calls resolves in this library. Running it needs a B200 (`npl_test_b200 -q`).
Skipped where the reference tree was not there to build it."""
import shutil
import subprocess
from pathlib import Path

import pytest

import support as S

BIN = S.REPO / "oracle" / "_ref" / "npl_test_b200"
LIB = S.REPO / "project-jcore_b200" / "lib" / "libnpl_b200.so"


def _symbols(path, *flags):
    out = subprocess.run(["nm", "-D", *flags, str(path)], capture_output=True, text=True,
                         check=True).stdout
    return {line.split()[-1] for line in out.splitlines() if line.strip()}


def test_reference_test_program_links_against_the_library():
    if not BIN.exists():
        pytest.skip("reference test program not built (no reference tree)")
    if not (shutil.which("ldd") and shutil.which("nm")):
        pytest.skip("binutils / ldd unavailable")
    text = subprocess.run(["ldd", "-r", str(BIN)], capture_output=True, text=True)
    text = text.stdout + text.stderr
    assert "undefined symbol" not in text
    lines = [ln for ln in text.splitlines() if "libnpl_b200.so" in ln]
    assert lines and "not found" not in lines[0]
    assert "=>" in lines[0]
    resolved = lines[0].split("=>")[1].split("(")[0].strip()
    assert S.REPO.resolve() in Path(resolved).resolve().parents
    imported = {s for s in _symbols(BIN, "--undefined-only") if s.startswith("npl_")}
    exported = _symbols(LIB, "--defined-only")
    assert len(imported) >= 15  # init, tensors, matmul, add/mul, conv, activations, norms, pools
    assert imported <= exported
