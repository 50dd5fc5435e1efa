"""The C ABI from a plain C program: a translation unit that includes
include/dsa_b200.h compiles with gcc, links libdsa_b200.so and gets the
documented status codes and messages for argument errors (no GPU needed)."""
from __future__ import annotations

import os
import shutil
import subprocess

import pytest

from flashinfer_repo_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

C_SOURCE = r"""
#include <stdio.h>
#include <string.h>
#include "dsa_b200.h"

int main(void) {
  size_t n = 0;
  int rc = dsa_sparse_attention_workspace_size(1, 20, 2048, &n);  /* heads not a multiple of 16 */
  printf("ws %d %s\n", rc, strstr(dsa_last_error_message(), "multiple of 16") ? "msg" : "nomsg");
  rc = dsa_sparse_attention(0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0,
                            1, 16, 64, 32 /* page_size */, 2048, 0.1f, 0, 0, 0, 0, 0, 0, 0, 0, 0);
  printf("page %d\n", rc);
  rc = dsa_sparse_attention(0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0,
                            0 /* tokens */, 16, 64, 64, 2048, 0.1f, 0, 0, 0, 0, 0, 0, 0, 0, 0);
  printf("empty %d\n", rc);
  rc = dsa_topk_select(0, 0, 0, 0, 0, 1, 4096 /* k > 2048 */, 0, 0, 0, 0);
  printf("topk %d\n", rc);
  return 0;
}
"""


def test_c_program_links_and_sees_the_abi(tmp_path):
    gcc = shutil.which("gcc")
    if gcc is None:
        pytest.skip("gcc not available")
    lib = _lib.load()  # builds the library if needed
    libdir = os.path.dirname(_lib.lib_path())
    src = tmp_path / "abi.c"
    src.write_text(C_SOURCE)
    exe = tmp_path / "abi"
    subprocess.run([gcc, "-std=c99", "-Wall", "-Werror", "-I", os.path.join(ROOT, "include"),
                    str(src), "-L", libdir, "-ldsa_b200", f"-Wl,-rpath,{libdir}", "-o", str(exe)],
                   check=True, capture_output=True)
    out = subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout.split("\n")
    assert out[0] == "ws 1 msg"        # DSA_ERR_INVALID_ARG with its message
    assert out[1] == "page 2"          # DSA_ERR_UNSUPPORTED: page_size must be 64
    assert out[2] == "empty 0"         # zero tokens: nothing to do
    assert out[3] == "topk 2"          # k above 2048 is unsupported
    del lib
