"""The FP8 quantizer's division-free quotient (csrc/fp8_product.h:
Markstein's correction of x * RN(1 / s)), checked on the CPU against IEEE
division and through the C restatement's encoder.  At the reference's
default backoff 1 the check is exhaustive: every bf16 weight against every
per-channel scale the reference can form (all positive finite bf16 absmax
values, E4M3 and E5M2 maxima); other backoffs are strided samples.  The
harness compiles the same header the CUDA kernel includes."""
import os
import shutil
import subprocess

import pytest

from conftest import ROOT

HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.fixture(scope="module")
def checker(tmp_path_factory):
    if shutil.which("g++") is None or shutil.which("gcc") is None:
        pytest.skip("no C/C++ compiler")
    d = tmp_path_factory.mktemp("fp8p")
    obj = str(d / "fp8_oracle.o")
    subprocess.run(["gcc", "-O2", "-fopenmp", "-c", os.path.join(ROOT, "oracle", "fp8_oracle.c"), "-o", obj],
                   check=True)
    flags = ["-O2", "-std=c++17", "-fopenmp", "-ffp-contract=off"]
    with open("/proc/cpuinfo") as f:
        if " fma " in f.read():
            flags.append("-mfma")   # the same fmaf results, in hardware
    exe = str(d / "check")
    subprocess.run(["g++"] + flags + ["-I", os.path.join(ROOT, "reciprocating-engine_b200", "csrc"),
                                      os.path.join(HERE, "fp8_product_check.cc"), obj, "-o", exe, "-lm"],
                   check=True)
    return exe


def run(exe, *args):
    r = subprocess.run([exe] + [str(a) for a in args], capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, r.stdout + r.stderr
    lines = r.stdout.strip().splitlines()
    assert len(lines) == 2 and all("bits_mismatch 0 code_mismatch 0" in l for l in lines), r.stdout
    return lines


def test_every_weight_against_every_default_scale(checker):
    lines = run(checker, 1, 1.0)
    # 32639 positive finite bf16 absmax values per format's scale set
    assert all(" rows 32639 " in l for l in lines), lines


def test_other_backoffs_sampled(checker):
    run(checker, 7, 0.5, 0.25, 0.75, 1.5, 2.0, 3.0e-3, 1.0e3)
