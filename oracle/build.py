"""Build recipe for the C oracle: ``oracle/_build/libkv_oracle.so``.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``). Plain gcc on the one
source file; no reference source is compiled (the reference is Python).
"""
from __future__ import annotations

import os
import shutil
import subprocess
from pathlib import Path

ORACLE_DIR = Path(__file__).resolve().parent
SOURCE = ORACLE_DIR / "kv_oracle.c"
OUTPUT = ORACLE_DIR / "_build" / "libkv_oracle.so"


def build(force: bool = False) -> Path:
    if not force and OUTPUT.exists() and OUTPUT.stat().st_mtime >= SOURCE.stat().st_mtime:
        return OUTPUT
    cc = os.environ.get("CC") or shutil.which("gcc") or shutil.which("cc")
    if not cc:
        raise RuntimeError("no C compiler found for the oracle")
    OUTPUT.parent.mkdir(parents=True, exist_ok=True)
    tmp = OUTPUT.with_suffix(".so.tmp")
    cmd = [cc, "-O3", "-march=x86-64-v2", "-std=c11", "-shared", "-fPIC", "-pthread", "-o", str(tmp), str(SOURCE)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"oracle build failed:\n{res.stdout}\n{res.stderr}")
    os.replace(tmp, OUTPUT)
    return OUTPUT


if __name__ == "__main__":
    print(build(force=True))
