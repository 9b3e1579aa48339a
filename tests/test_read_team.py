"""The source-read team (kadan_b200/csrc/read_team.hpp), the reference's
PackedReadTeam (services/hikari/inference_worker/include/kadan/
packed_read_team.hpp:22-275), as a C++ unit test built with the host compiler:
row runs, exactly-once items over rounds and lane counts, failure reporting.
No GPU."""
from __future__ import annotations

import shutil
import subprocess

import pytest

from conftest import ROOT


def test_read_team(tmp_path):
    cxx = shutil.which("g++")
    if cxx is None:
        pytest.skip("no host C++ compiler")
    exe = tmp_path / "read_team_test"
    subprocess.run([cxx, "-std=c++17", "-O1", "-pthread", f"-I{ROOT / 'include'}", f"-I{ROOT / 'kadan_b200' / 'csrc'}",
                    str(ROOT / "tests" / "cpp" / "read_team_test.cpp"), "-o", str(exe)], check=True)
    run = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert run.returncode == 0, run.stderr
    assert run.stdout.strip() == "ok"
