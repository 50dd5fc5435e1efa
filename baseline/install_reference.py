"""Place the unmodified reference checkout in baseline/_ref (git-ignored).

    python baseline/install_reference.py /path/to/reference

The reference (Starkdoorstep12/flashinfer-repo) has no setup.py or
pyproject.toml, so `pip install --target baseline/_ref <reference>` cannot
build it; its Python/Triton sources are importable as they stand once the
checkout's root is on sys.path (`import solution.triton.kernel`, a namespace
package).  This script therefore copies the checkout file for file, contents
unchanged, into baseline/_ref.  baseline/_ref is listed in .gitignore (it is
not part of this repository's history) but travels with a snapshot of the
working tree to a GPU machine, where the fixture generator
tests/golden/make_ref_gpu_golden.py and `bench.py --impl reference` import it.
"""
from __future__ import annotations

import os
import shutil
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
DEST = os.path.join(HERE, "_ref")
# large binary profiling captures and images are not needed to run the code
SKIP = {"profiling_results", "images", ".git"}


def install(src: str) -> str:
    if not os.path.isfile(os.path.join(src, "solution", "triton", "kernel.py")):
        raise SystemExit(f"{src} does not look like the reference checkout")
    if os.path.isdir(DEST):
        shutil.rmtree(DEST)
    shutil.copytree(src, DEST, ignore=lambda d, names: [n for n in names if n in SKIP])
    for root, dirs, files in os.walk(DEST):  # the source tree may be read-only
        for n in dirs + files:
            os.chmod(os.path.join(root, n), 0o755 if n in dirs else 0o644)
    return DEST


def available() -> bool:
    return os.path.isfile(os.path.join(DEST, "solution", "triton", "kernel.py"))


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit("usage: python baseline/install_reference.py /path/to/reference")
    print(install(sys.argv[1]))
