"""Contest CUDA-route package: solution.json schema and layout, the TVM-FFI
binding source compiles for sm_100a, and (GPU) the unpacked solution built by
tvm_ffi.cpp.load gives the library kernel()'s results bit for bit."""
from __future__ import annotations

import importlib.util
import json
import os
import shutil
import subprocess
import sys

import pytest

from flashinfer_repo_b200.contest import pack

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_solution_schema_and_sources(tmp_path):
    sol = pack.build_solution()
    assert set(sol) == {"name", "definition", "author", "spec", "sources", "description"}
    assert sol["definition"] == "dsa_sparse_attention_h16_ckv512_kpe64_topk2048_ps64"
    assert sol["spec"] == {"language": "cuda", "target_hardware": ["cuda"],
                           "entry_point": "binding.py::kernel", "dependencies": [],
                           "destination_passing_style": False, "binding": None}
    paths = [s["path"] for s in sol["sources"]]
    assert paths[:3] == ["binding.py", "binding.cu", "include/dsa_b200.h"]
    assert "flashinfer_repo_b200/csrc/attention.cu" in paths
    out = tmp_path / "solution.json"
    subprocess.run([sys.executable, "-m", "flashinfer_repo_b200.contest.pack", "-o", str(out)],
                   cwd=ROOT, check=True, capture_output=True)
    assert json.loads(out.read_text()) == sol
    pack.unpack(sol, str(tmp_path / "unpacked"))
    for s in sol["sources"]:
        assert (tmp_path / "unpacked" / s["path"]).read_text() == s["content"]


def test_binding_compiles_for_sm100a(tmp_path):
    import tvm_ffi
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    inc = os.path.join(os.path.dirname(tvm_ffi.__file__), "include")
    subprocess.run([nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-std=c++17", "-Xcompiler",
                    "-fPIC", "-I", ROOT, "-I", inc, "-c",
                    os.path.join(ROOT, "flashinfer_repo_b200", "contest", "binding.cu"),
                    "-o", str(tmp_path / "binding.o")], check=True, capture_output=True)


@pytest.mark.gpu
def test_unpacked_solution_matches_library(cuda_device, tmp_path):
    import torch

    from flashinfer_repo_b200 import kernel
    from flashinfer_repo_b200.bench_inputs import make_paged_batch
    sol = pack.build_solution()
    d = tmp_path / "solution"
    pack.unpack(sol, str(d))
    os.environ.setdefault("TVM_FFI_CACHE_DIR", str(tmp_path / "tvm_ffi_cache"))
    spec = importlib.util.spec_from_file_location("dsa_contest_binding", d / "binding.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    qn, qp, ckv, kpe, idx, sc = make_paged_batch([20000, 3000, 70000], 11, cuda_device)
    out, lse = mod.kernel(qn, qp, ckv, kpe, idx, sc)
    ref_out, ref_lse = kernel(qn, qp, ckv, kpe, idx, sc)
    torch.cuda.synchronize()
    assert torch.equal(out, ref_out) and torch.equal(lse, ref_lse)
