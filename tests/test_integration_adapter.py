"""The worker-side adapter include/kadan_b200_dense_compute.hpp compiles
against the reference's own kadan/dense_compute.hpp (its overrides match the
reference's virtual signatures) and links against libkadan_b200.so with no
undefined symbol. Needs the reference tree; no GPU."""
from __future__ import annotations

import shutil
import subprocess
from pathlib import Path

import pytest

from conftest import ROOT
from oracle.pyoracle import REFERENCE_TREE

IW = REFERENCE_TREE / "services" / "hikari" / "inference_worker"


def test_adapter_compiles_against_reference_interface(kb, tmp_path):
    cxx = shutil.which("g++")
    if cxx is None or not (IW / "include" / "kadan" / "dense_compute.hpp").exists():
        pytest.skip("needs the reference headers and a host C++ compiler")
    tu = tmp_path / "adapter.cpp"
    tu.write_text(
        '#include "kadan_b200_dense_compute.hpp"\n'
        "std::unique_ptr<kadan::DenseCompute> make(std::shared_ptr<kadan::DenseCompute> f) {\n"
        "    return std::make_unique<kadan::b200::Compute>(std::move(f), std::vector<int>{0, 1}, 1ull << 30,\n"
        "                                                  1ull << 30);\n"
        "}\n")
    lib = Path(kb.LIB_PATH)
    cmd = [cxx, "-std=c++20", "-Wall", "-Wextra", "-Werror", "-shared", "-fPIC", f"-I{ROOT / 'include'}",
           f"-I{IW / 'include'}", f"-I{IW / 'third_party' / 'ggml' / 'include'}", str(tu), f"-L{lib.parent}",
           "-lkadan_b200", "-Wl,--no-undefined", "-o", str(tmp_path / "adapter.so")]
    run = subprocess.run(cmd, capture_output=True, text=True)
    assert run.returncode == 0, run.stderr


def test_adapter_overrides_every_virtual():
    """Every virtual of the reference's DenseCompute is overridden, so the
    adapter can take the place of the worker's compute object without turning
    any of its features off."""
    import re

    header = IW / "include" / "kadan" / "dense_compute.hpp"
    if not header.exists():
        pytest.skip("needs the reference headers")
    text = header.read_text()
    body = text[text.index("class DenseCompute {"):]
    names = set(re.findall(r"virtual\s+(?:[\w:<>,\s]+?\s+)?(\w+)\s*\(", body)) - {"~DenseCompute"}
    adapter = (ROOT / "include" / "kadan_b200_dense_compute.hpp").read_text()
    overridden = set(re.findall(r"(\w+)\s*\([^;{]*?\)\s*(?:const\s*)?override", adapter, re.S))
    assert len(names) >= 20
    assert names <= overridden, sorted(names - overridden)


def test_adapter_behaviour_over_fake_devices(kb, tmp_path):
    """tests/cpp/adapter_test.cpp: the adapter through the reference's own
    DenseCompute interface, its device entry points played by host fakes and
    the partition, support and status code the real library's. Covers the
    column split over two devices in proportion to the banks' envelopes
    (gguf_batch_partition, as h3_compute.cu:4020-4027 and the weighted split
    of :1697-1758 make it) and the scatter back, rows read once each through
    shifted sources, the bias slice, unsupported before any read or write,
    the reference's exception messages, a source's exception rethrown, and the
    residency virtuals over the wrapped compute plus the banks."""
    cxx = shutil.which("g++")
    if cxx is None or not (IW / "include" / "kadan" / "dense_compute.hpp").exists():
        pytest.skip("needs the reference headers and a host C++ compiler")
    lib = Path(kb.LIB_PATH)
    exe = tmp_path / "adapter_test"
    cmd = [cxx, "-std=c++20", "-O1", "-g", "-Wall", "-Wextra", "-Werror", "-pthread", f"-I{ROOT / 'include'}",
           f"-I{IW / 'include'}", f"-I{IW / 'third_party' / 'ggml' / 'include'}",
           str(ROOT / "tests" / "cpp" / "adapter_test.cpp"), f"-L{lib.parent}", "-lkadan_b200",
           f"-Wl,-rpath,{lib.parent}", "-o", str(exe)]
    run = subprocess.run(cmd, capture_output=True, text=True)
    assert run.returncode == 0, run.stderr
    run = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert run.returncode == 0 and run.stdout.strip() == "ok", run.stdout + run.stderr
