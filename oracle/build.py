"""Builds the oracle's C restatements with gcc into oracle/_build/ (test infrastructure)."""
from __future__ import annotations

import subprocess
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_build"


def build_ngram(force: bool = False) -> Path:
    src = HERE / "ngram.c"
    lib = OUT / "libngram_oracle.so"
    if force or not lib.exists() or lib.stat().st_mtime < src.stat().st_mtime:
        OUT.mkdir(exist_ok=True)
        subprocess.run(["gcc", "-O2", "-shared", "-fPIC", "-o", str(lib), str(src)], check=True)
    return lib


def build_all(force: bool = False) -> None:
    build_ngram(force)


if __name__ == "__main__":
    build_all(force=True)
    print(OUT)
