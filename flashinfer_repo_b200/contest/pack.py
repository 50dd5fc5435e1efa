"""Pack the CUDA-route solution into solution.json.

    python -m flashinfer_repo_b200.contest.pack [-o solution.json]

Replaces the reference's scripts/pack_solution.py (:34-84), which needs the
external flashinfer_bench package (absent here).  Writes the same Solution
document: name / definition / author from config.toml's [solution], a spec
{language, target_hardware ["cuda"], entry_point, dependencies [],
destination_passing_style, binding null} from [build], an empty description,
and `sources` as {path, content} entries -- binding.py and binding.cu at the
root, the header under include/ and the kernels under
flashinfer_repo_b200/csrc/, the relative layout their #include lines use.
"""
from __future__ import annotations

import argparse
import glob
import json
import os

try:
    import tomllib
except ImportError:  # Python < 3.11
    import tomli as tomllib

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))


def source_files() -> list[tuple[str, str]]:
    """(path inside the solution, file on disk) for every packed source."""
    files = [("binding.py", os.path.join(HERE, "binding.py")),
             ("binding.cu", os.path.join(HERE, "binding.cu")),
             ("include/dsa_b200.h", os.path.join(ROOT, "include", "dsa_b200.h"))]
    csrc = os.path.join(ROOT, "flashinfer_repo_b200", "csrc")
    for f in sorted(glob.glob(os.path.join(csrc, "*.cu")) + glob.glob(os.path.join(csrc, "*.cuh"))):
        files.append((f"flashinfer_repo_b200/csrc/{os.path.basename(f)}", f))
    return files


def build_solution(config_path: str | None = None) -> dict:
    with open(config_path or os.path.join(HERE, "config.toml"), "rb") as f:
        cfg = tomllib.load(f)
    sol, build = cfg["solution"], cfg["build"]
    if build["language"] != "cuda":
        raise ValueError("this package is the CUDA route")
    sources = []
    for path, disk in source_files():
        with open(disk, encoding="utf-8") as f:
            sources.append({"path": path, "content": f.read()})
    return {
        "name": sol["name"],
        "definition": sol["definition"],
        "author": sol["author"],
        "spec": {
            "language": build["language"],
            "target_hardware": ["cuda"],
            "entry_point": build["entry_point"],
            "dependencies": [],
            "destination_passing_style": bool(build.get("destination_passing_style", True)),
            "binding": None,
        },
        "sources": sources,
        "description": "",
    }


def unpack(solution: dict, directory: str) -> None:
    """Write a Solution document's sources into `directory` (the layout the
    entry point loads from)."""
    for src in solution["sources"]:
        dst = os.path.join(directory, src["path"])
        os.makedirs(os.path.dirname(dst), exist_ok=True)
        with open(dst, "w", encoding="utf-8") as f:
            f.write(src["content"])


def main():
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("-o", "--output", default=os.path.join(ROOT, "solution.json"))
    ap.add_argument("--config", default=None)
    args = ap.parse_args()
    solution = build_solution(args.config)
    with open(args.output, "w", encoding="utf-8") as f:
        json.dump(solution, f, indent=2)
    print(f"Solution packed: {args.output} ({len(solution['sources'])} sources, "
          f"entry point {solution['spec']['entry_point']})")


if __name__ == "__main__":
    main()
