"""verify_full (csrc/bench/verify_full.cpp) against the reference checker's
reports (ring/attention/verify_full.c, recorded in tests/golden/
verify_full_golden.txt) on deterministic dump sets: the same PASS/FAIL lines,
element and NaN/Inf counts, overall result and exit code, and the same error
figures and worst index (to the last printed digit where the reference values
are exact, within one fp32 ulp of the ~6.6e4 outputs otherwise)."""
import os
import re
import subprocess

import pytest

from verify_full_cases import CASES, write_case

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def verify_bin(tmp_path_factory):
    exe = os.path.join(ROOT, "build", "bin", "verify_full")
    if not os.path.exists(exe):
        exe = str(tmp_path_factory.mktemp("vf") / "verify_full")
        src = [os.path.join(ROOT, "csrc/bench/verify_full.cpp")] + [
            os.path.join(ROOT, "csrc/sched", f)
            for f in ("scheduler.cpp", "workload.cpp", "shard_plan.cpp")]
        subprocess.check_call(["g++", "-O2", "-std=c++17", "-pthread", "-o", exe] + src)
    return exe


def _golden():
    text = open(os.path.join(ROOT, "tests/golden/verify_full_golden.txt")).read()
    out = {}
    for block in text.split("CASE ")[1:]:
        name, rest = block.split("\n", 1)
        body, rc = rest.rsplit("RC ", 1)
        out[name] = (body, int(rc.strip()))
    return out


GOLDEN = _golden()
_NUM = re.compile(r"-?\d+\.\d+|-?\d+|nan|inf", re.I)


def _compare(got, exp):
    gl, el = got.strip().splitlines(), exp.strip().splitlines()
    assert len(gl) == len(el), f"line count {len(gl)} vs {len(el)}\n{got}"
    for g, e in zip(gl, el):
        assert _NUM.sub("#", g) == _NUM.sub("#", e), f"{g!r} vs {e!r}"
        for a, b in zip(_NUM.findall(g), _NUM.findall(e)):
            if "." in b:
                fa, fb = float(a), float(b)
                assert abs(fa - fb) <= max(0.0079, 1e-7 * abs(fb)), f"{g!r} vs {e!r}"
            else:
                assert a == b, f"{g!r} vs {e!r}"


@pytest.mark.parametrize("name", list(CASES))
def test_report_matches_reference(tmp_path, verify_bin, name):
    P, kv = write_case(name, str(tmp_path))
    p = subprocess.run([verify_bin, str(tmp_path), str(P), str(kv)], capture_output=True,
                       text=True, timeout=120)
    body, rc = GOLDEN[name]
    assert p.returncode == rc
    _compare(p.stdout.replace(str(tmp_path), "<DIR>"), body)


def test_bad_size_is_rejected(verify_bin):
    p = subprocess.run([verify_bin, "/nonexistent", "2", "1000"], capture_output=True, text=True,
                       timeout=60)
    assert p.returncode == GOLDEN["bad_size"][1] == 1
    assert "Usage:" in p.stderr
