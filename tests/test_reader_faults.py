"""Read-fault injection for the checkpoint readers, as the reference tests its
GGUF reader (pread wrapped at link time, IW/CMakeLists.txt:439): the readers
are built as host C++ with -Wl,--wrap=pread around tests/cpp/
reader_faults_test.cpp, which checks short reads, an interrupted read and an
I/O error at every read position. No GPU."""
from __future__ import annotations

import shutil
import subprocess
from pathlib import Path

import numpy as np
import pytest

from conftest import ROOT


def test_reader_read_faults(tmp_path):
    cxx = shutil.which("g++")
    nvcc = shutil.which("nvcc")
    if cxx is None or nvcc is None:
        pytest.skip("needs a host C++ compiler and the CUDA headers")
    cuda_include = Path(nvcc).resolve().parent.parent / "include"
    import kadan_b200 as kb
    from kadan_b200 import gguf_write as gw
    from kadan_b200 import synth
    from test_shard import mxfp4_tensors, write_shard

    gdir, sdir = tmp_path / "gguf", tmp_path / "shard"
    gdir.mkdir()
    sdir.mkdir()
    w = synth.gguf(kb.Q4_K, 40, 512, seed=4)  # 40 rows of 288 bytes
    gw.write_arrays(gdir / "m.gguf", [("general.architecture", gw.STRING, "llama")],
                    [("w", [512, 40], 12, w), ("n", [16], 0, np.ones(16, np.float32))])
    (tmp_path / "gguf_rows.bin").write_bytes(w.tobytes())
    tensors, blocks, scales = mxfp4_tensors("e", 2, 33, 3, seed=5)
    write_shard(sdir / "s.safetensors", tensors)
    (tmp_path / "mxfp4_rows.bin").write_bytes(blocks[0].tobytes() + scales[0].tobytes())
    exe = tmp_path / "reader_faults_test"
    csrc = ROOT / "kadan_b200" / "csrc"
    cmd = [cxx, "-std=c++17", "-O1", f"-I{ROOT / 'include'}", f"-I{csrc}", f"-I{cuda_include}",
           str(ROOT / "tests" / "cpp" / "reader_faults_test.cpp"), str(csrc / "gguf_file.cpp"),
           str(csrc / "safetensors.cpp"), "-Wl,--wrap=pread", "-o", str(exe)]
    subprocess.run(cmd, check=True)
    run = subprocess.run([str(exe), str(gdir), "w", str(tmp_path / "gguf_rows.bin"), str(sdir), "s.safetensors", "e",
                          str(tmp_path / "mxfp4_rows.bin")], capture_output=True, text=True, timeout=120)
    assert run.returncode == 0, run.stderr
    assert run.stdout.strip() == "ok"
