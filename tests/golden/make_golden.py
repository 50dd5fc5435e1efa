"""Generate tests/golden/*.npz from the reference's own golden function.

Runs the reference `run` (solution/triton/indexer_kernel.py:436-497) on CPU in
this build container, where the reference checkout is mounted, and saves its
outputs (bf16 output as uint16 bits, fp32 base-2 LSE) together with a digest
of the inputs.  The reference module only does `import torch, triton` and uses
`math` without importing it (indexer_kernel.py:490), so `math` is injected
into its namespace; the reference file itself is not modified.

Usage:  python tests/golden/make_golden.py /path/to/reference
The GPU box never runs this script; it only reads the committed .npz files.
"""
from __future__ import annotations

import importlib.util
import math
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from tests.golden.cases import CASES, digest  # noqa: E402


def load_reference_run(ref_root: str):
    path = os.path.join(ref_root, "solution", "triton", "indexer_kernel.py")
    spec = importlib.util.spec_from_file_location("_ref_indexer_kernel", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    mod.math = math  # the reference uses math.log without importing math
    return mod.run


def bf16(bits: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(bits.astype(np.int16)).view(torch.bfloat16)


def main(ref_root: str):
    run = load_reference_run(ref_root)
    for name, make in CASES.items():
        c = make()
        out, lse = run(bf16(c.q_nope), bf16(c.q_pe), bf16(c.ckv), bf16(c.kpe),
                       torch.from_numpy(c.idx), c.sm_scale)
        out_bits = out.view(torch.int16).numpy().astype(np.uint16)
        np.savez_compressed(os.path.join(HERE, f"attn_{name}.npz"), out=out_bits,
                            lse=lse.numpy().astype(np.float32), digest=np.array(digest(c)))
        print(f"{name}: T={c.T} pages={c.ckv.shape[0]} digest={digest(c)[:12]}")


if __name__ == "__main__":
    main(*sys.argv[1:])
