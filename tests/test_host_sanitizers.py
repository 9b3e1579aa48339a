"""The host-only C++ of the library under AddressSanitizer and
UndefinedBehaviorSanitizer (the reference runs its host unit tests that way):
the source-read team, the weight bank over fake device operations, the
checkpoint readers with injected read faults, and the readers over 200 seeded
random mutations of valid GGUF and safetensors files. Any sanitizer report
fails the run. No GPU."""
from __future__ import annotations

import random
import shutil
import subprocess
from pathlib import Path

import numpy as np
import pytest

from conftest import ROOT

CSRC = ROOT / "kadan_b200" / "csrc"
FLAGS = ["-std=c++17", "-O1", "-g", "-fsanitize=address,undefined", "-fno-sanitize-recover=all",
         "-fno-omit-frame-pointer"]


def compiler():
    cxx, nvcc = shutil.which("g++"), shutil.which("nvcc")
    if cxx is None or nvcc is None:
        pytest.skip("needs a host C++ compiler and the CUDA headers")
    return cxx, Path(nvcc).resolve().parent.parent / "include"


def build(tmp_path, name, sources, extra=()):
    cxx, cuda_include = compiler()
    exe = tmp_path / name
    cmd = [cxx, *FLAGS, f"-I{ROOT / 'include'}", f"-I{CSRC}", f"-I{cuda_include}", *map(str, sources), *extra,
           "-pthread", "-o", str(exe)]
    subprocess.run(cmd, check=True)
    return exe


def run(exe, *args):
    env = {"ASAN_OPTIONS": "detect_leaks=1:abort_on_error=0", "UBSAN_OPTIONS": "print_stacktrace=1"}
    r = subprocess.run([str(exe), *map(str, args)], capture_output=True, text=True, timeout=300, env=env)
    assert r.returncode == 0, r.stderr[-4000:]
    assert "runtime error" not in r.stderr and "AddressSanitizer" not in r.stderr, r.stderr[-4000:]
    return r.stdout


def test_read_team_sanitized(tmp_path):
    exe = build(tmp_path, "read_team", [ROOT / "tests" / "cpp" / "read_team_test.cpp"])
    assert run(exe).strip() == "ok"


def test_weight_bank_sanitized(tmp_path):
    cuda_lib = compiler()[1].parent / "lib64"
    exe = build(tmp_path, "bank", [ROOT / "tests" / "cpp" / "bank_test.cpp", CSRC / "weight_bank.cpp"],
                [f"-L{cuda_lib}", f"-Wl,-rpath,{cuda_lib}", "-lcudart"])
    assert run(exe).strip() == "ok"


def test_reader_faults_sanitized(tmp_path):
    import kadan_b200 as kb
    from kadan_b200 import gguf_write as gw
    from kadan_b200 import synth
    from test_shard import mxfp4_tensors, write_shard

    exe = build(tmp_path, "faults", [ROOT / "tests" / "cpp" / "reader_faults_test.cpp", CSRC / "gguf_file.cpp",
                                     CSRC / "safetensors.cpp"], ["-Wl,--wrap=pread"])
    gdir, sdir = tmp_path / "gguf", tmp_path / "shard"
    gdir.mkdir()
    sdir.mkdir()
    w = synth.gguf(kb.Q4_K, 40, 512, seed=4)
    gw.write_arrays(gdir / "m.gguf", [("general.architecture", gw.STRING, "llama")],
                    [("w", [512, 40], 12, w), ("n", [16], 0, np.ones(16, np.float32))])
    (tmp_path / "g.bin").write_bytes(w.tobytes())
    tensors, blocks, scales = mxfp4_tensors("e", 2, 33, 3, seed=5)
    write_shard(sdir / "s.safetensors", tensors)
    (tmp_path / "s.bin").write_bytes(blocks[0].tobytes() + scales[0].tobytes())
    assert run(exe, gdir, "w", tmp_path / "g.bin", sdir, "s.safetensors", "e", tmp_path / "s.bin").strip() == "ok"


def test_readers_on_mutated_files_sanitized(tmp_path):
    from kadan_b200 import gguf_write as gw
    from test_gguf_file import KVS, TENSORS
    from test_reader_fuzz import mutate
    from test_shard import mxfp4_tensors, write_shard

    exe = build(tmp_path, "open_many", [ROOT / "tests" / "cpp" / "reader_open_many.cpp", CSRC / "gguf_file.cpp",
                                        CSRC / "safetensors.cpp"])
    gguf_base, _ = gw.build(KVS, TENSORS, alignment=64)
    seed_dir = tmp_path / "seed"
    seed_dir.mkdir()
    tensors, _, _ = mxfp4_tensors("p", 2, 4, 2, seed=1)
    write_shard(seed_dir / "s.safetensors", tensors, metadata={"format": "pt"})
    shard_base = (seed_dir / "s.safetensors").read_bytes()
    rng = random.Random(99)
    args = [f"gguf:{seed_dir.parent / 'none'}"]
    for i in range(200):
        d = tmp_path / f"g{i}"
        d.mkdir()
        (d / "m.gguf").write_bytes(bytes(mutate(rng, bytearray(gguf_base), 1200)))
        args.append(f"gguf:{d}")
        e = tmp_path / f"s{i}"
        e.mkdir()
        (e / "s.safetensors").write_bytes(bytes(mutate(rng, bytearray(shard_base), 400)))
        args.append(f"shard:{e}/s.safetensors")
    out = run(exe, *args)
    assert out.strip().endswith("ok") and int(out.split()[0]) > 0


def test_host_sources_build_warning_free(tmp_path):
    """The host-only sources compile with -Wall -Wextra -Wpedantic -Werror,
    the warning level the reference builds with."""
    cxx, cuda_include = compiler()
    for src in ("gguf_file.cpp", "safetensors.cpp", "weight_bank.cpp", "partition.cpp"):
        cmd = [cxx, "-std=c++17", "-Wall", "-Wextra", "-Wpedantic", "-Werror", "-fsyntax-only", f"-I{ROOT / 'include'}",
               f"-I{CSRC}", f"-I{cuda_include}", str(CSRC / src)]
        r = subprocess.run(cmd, capture_output=True, text=True)
        assert r.returncode == 0, (src, r.stderr[-2000:])
    for header in ("read_team.hpp", "gguf_geometry.hpp"):
        tu = tmp_path / "h.cpp"
        tu.write_text(f'#include "{header}"\nint main() {{ return 0; }}\n')
        r = subprocess.run([cxx, "-std=c++17", "-Wall", "-Wextra", "-Wpedantic", "-Werror", "-fsyntax-only",
                            f"-I{ROOT / 'include'}", f"-I{CSRC}", str(tu)], capture_output=True, text=True)
        assert r.returncode == 0, (header, r.stderr[-2000:])
