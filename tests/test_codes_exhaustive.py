"""Exhaustive host check of the encode arithmetic the kernels run.

tests/native/check_codes.cpp compiles the kernels' own glint_codec.cuh and the
build-generated lookup table with g++ and compares, against the CPU oracle's
restatement of the reference scan (cuda/glint_encode.cu:67-102):
  codes    every f32 in [-1, 1] and every quiet NaN (2.1e9 values)
  bf16div  every BF16 (w, s) pair with |w| <= s: Markstein quotient == IEEE w/s
  f32div   2^26 random f32 pairs
"""
import os
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent


@pytest.fixture(scope="module")
def checker(tmp_path_factory):
    from glint_b200 import build
    import glint_oracle
    build.build()
    glint_oracle.build()
    exe = tmp_path_factory.mktemp("chk") / "check_codes"
    subprocess.run(["g++", "-O2", "-fopenmp", "-std=c++17", "-I", str(ROOT / "glint_b200" / "_build"),
                    "-o", str(exe), str(ROOT / "tests" / "native" / "check_codes.cpp"),
                    "-L", str(ROOT / "oracle"), "-lglint_oracle", f"-Wl,-rpath,{ROOT / 'oracle'}"], check=True)
    return exe


@pytest.mark.parametrize("mode", ["codes", "bf16div", "f32div"])
def test_exhaustive(checker, mode):
    env = dict(os.environ, OMP_NUM_THREADS=str(os.cpu_count() or 1))
    r = subprocess.run([str(checker), mode], capture_output=True, text=True, env=env, timeout=900)
    assert r.returncode == 0 and r.stdout.startswith("OK"), r.stdout + r.stderr
