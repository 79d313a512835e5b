"""The device exp (jero-arch-llama_b200/csrc/libm_expf.h) against the host
libm expf that the reference's f32::exp and the oracle call.

The header is plain C++ for host and device; here its host build is compared
with expf bit for bit on every 97th float with |x| <= 110 and on special
values (the full range, 2,243,428,356 floats, was checked the same way).
"""
import os
import subprocess

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_expf_ref_equals_host_libm(tmp_path):
    exe = tmp_path / "expf_sample"
    cc = subprocess.run(["g++", "-O2", "-ffp-contract=off", "-std=c++17",
                         "-I", os.path.join(REPO, "jero-arch-llama_b200", "csrc"),
                         os.path.join(REPO, "tests", "expf_sample.cpp"), "-o", str(exe), "-lm"],
                        capture_output=True, text=True)
    if cc.returncode != 0:
        pytest.fail(cc.stderr)
    r = subprocess.run([str(exe), "97"], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "mismatched 0" in r.stdout
