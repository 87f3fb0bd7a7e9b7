"""CPU: the contest packaging (flashinfer-mlsys_b200/pack_solution.py) writes
the harness's solution document with every source of the library, flat, and
the extracted tree compiles for sm_100a on its own include path."""
import importlib
import json
import os
import shutil
import subprocess

import pytest

pack = importlib.import_module("flashinfer-mlsys_b200.pack_solution")
build = importlib.import_module("flashinfer-mlsys_b200.build")


def test_solution_document_fields_and_sources(tmp_path):
    sol = json.loads(json.dumps(pack.pack("s1", "me")))          # JSON round trip
    assert sol["name"] == "s1" and sol["author"] == "me"
    assert sol["definition"] == "moe_fp8_block_scale_ds_routing_topk8_ng8_kg4_e32_h7168_i2048"
    spec = sol["spec"]
    assert spec["language"] == "cuda" and spec["entry_point"] == "kernel.cu::kernel"
    assert spec["binding"] == "torch" and spec["destination_passing_style"] is True
    assert spec["target_hardware"] == ["cuda"] and spec["dependencies"] == []
    paths = [s["path"] for s in sol["sources"]]
    assert paths[0] == "kernel.cu" and len(paths) == len(set(paths))
    assert set(build.SOURCES + build.HEADERS + ["moe_fp8_ds.h"]) <= set(paths)
    cu = pack.extract(sol, str(tmp_path))
    assert sorted(os.path.basename(c) for c in cu) == sorted(["kernel.cu"] + build.SOURCES)
    for path, disk in pack.source_files():
        with open(disk) as a, open(tmp_path / path) as b:
            assert a.read() == b.read()


def test_extract_rejects_paths_outside_the_directory(tmp_path):
    bad = {"sources": [{"path": "../escape.cu", "content": ""}]}
    with pytest.raises(ValueError):
        pack.extract(bad, str(tmp_path / "sol"))


def test_extracted_tree_compiles_flat(tmp_path):
    """The C-ABI sources find moe_fp8_ds.h beside them (no repository
    layout), for sm_100a; the arch guard rejects any other target."""
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(nvcc):
        pytest.skip("nvcc not available")
    pack.extract(pack.pack(), str(tmp_path))
    src = str(tmp_path / "moe_api.cu")
    ok = subprocess.run([nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-std=c++17", "-I", str(tmp_path),
                         "-c", src, "-o", str(tmp_path / "a.o")], capture_output=True, text=True)
    assert ok.returncode == 0, ok.stderr[-2000:]
    bad = subprocess.run([nvcc, "-gencode", "arch=compute_100,code=sm_100", "-std=c++17", "-I", str(tmp_path),
                          "-c", src, "-o", str(tmp_path / "b.o")], capture_output=True, text=True)
    assert bad.returncode != 0 and "sm_100a" in bad.stderr


def test_tvm_ffi_binding_entry(tmp_path):
    """binding "tvm-ffi": the entry kernel.cu is the TVM-FFI export of the
    same operator, and it compiles flat against tvm_ffi's headers."""
    sol = pack.pack(binding="tvm-ffi")
    assert sol["spec"]["binding"] == "tvm-ffi" and sol["spec"]["entry_point"] == "kernel.cu::kernel"
    entry = next(s["content"] for s in sol["sources"] if s["path"] == "kernel.cu")
    assert "TVM_FFI_DLL_EXPORT_TYPED_FUNC(kernel" in entry and "PYBIND11_MODULE" not in entry
    with pytest.raises(ValueError):
        pack.pack(binding="tvm")
    tvm_ffi = pytest.importorskip("tvm_ffi")
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(nvcc):
        pytest.skip("nvcc not available")
    pack.extract(sol, str(tmp_path))
    inc = os.path.join(os.path.dirname(tvm_ffi.__file__), "include")
    r = subprocess.run([nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-std=c++17", "-I", str(tmp_path),
                        "-I", inc, "-c", str(tmp_path / "kernel.cu"), "-o", str(tmp_path / "k.o")],
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stderr[-2000:]
