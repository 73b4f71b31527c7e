"""Build recipes for the parity checker (test infrastructure only).

* ``build_oracle()`` compiles ``oracle/ebx_oracle.c`` with gcc into
  ``oracle/_build/libebx_oracle.so``.  ``-ffp-contract=off`` keeps float
  products and sums un-fused, matching the reference host analyzer.
* ``build_reference()`` compiles the reference's own ElasticBit runtime
  (``mlbricks/elasticbit/csrc/elasticbit_runtime.cu`` in the MLBricks tree) out
  of tree into ``oracle/_ref/_C.so`` with the same flags the reference's
  setup.py gives it (``--use_fast_math``), for sm_100a.  It is only used as a
  checker: its host analyzer produces the golden vectors in tests/golden, and
  on a GPU box its RuntimeMatrix is an A/B reference.  The reference sources are
  read in place and never copied.
"""
from __future__ import annotations

import hashlib
import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
BUILD_DIR = HERE / "_build"
REF_DIR = HERE / "_ref"
ORACLE_SO = BUILD_DIR / "libebx_oracle.so"
REFERENCE_CU_REL = Path("mlbricks") / "elasticbit" / "csrc" / "elasticbit_runtime.cu"


def reference_root(explicit: str | os.PathLike | None = None) -> Path | None:
    """The MLBricks source tree: `explicit`, else $EBX_REFERENCE_ROOT, else None."""
    root = explicit if explicit is not None else os.environ.get("EBX_REFERENCE_ROOT")
    return Path(root) if root else None


def build_oracle(force: bool = False) -> Path:
    src = HERE / "ebx_oracle.c"
    BUILD_DIR.mkdir(exist_ok=True)
    if not force and ORACLE_SO.exists() and ORACLE_SO.stat().st_mtime >= src.stat().st_mtime:
        return ORACLE_SO
    cmd = [
        "gcc", "-O2", "-std=c11", "-ffp-contract=off", "-fno-fast-math", "-fPIC", "-shared",
        str(src), "-o", str(ORACLE_SO), "-lm",
    ]
    subprocess.run(cmd, check=True)
    return ORACLE_SO


def build_reference(root: str | os.PathLike | None = None, force: bool = False,
                    verbose: bool = False) -> Path | None:
    """Compile the reference ElasticBit runtime into oracle/_ref/_C.so.

    `root` is the MLBricks source tree (default: $EBX_REFERENCE_ROOT).  Returns
    the path, or the previously built library (or None) when no tree is given
    or it is absent (as on a GPU box).  Skips the ~3 minute nvcc build when the
    output matches the source hash.
    """
    out = REF_DIR / "_C.so"
    tree = reference_root(root)
    reference_cu = tree / REFERENCE_CU_REL if tree else None
    if reference_cu is None or not reference_cu.exists():
        return out if out.exists() else None
    digest = hashlib.sha256(reference_cu.read_bytes()).hexdigest()
    stamp = REF_DIR / "source.sha256"
    if not force and out.exists() and stamp.exists() and stamp.read_text().strip() == digest:
        return out
    REF_DIR.mkdir(exist_ok=True)
    from torch.utils.cpp_extension import load

    load(
        name="_C",
        sources=[str(reference_cu)],
        build_directory=str(REF_DIR),
        extra_cflags=["-O3"],
        extra_cuda_cflags=["-O3", "--use_fast_math",
                           "-gencode", "arch=compute_100a,code=sm_100a"],
        verbose=verbose,
        is_python_module=True,
    )
    stamp.write_text(digest + "\n")
    return out


if __name__ == "__main__":
    # python oracle/build.py [--force] [--reference MLBRICKS_TREE]
    print(build_oracle(force="--force" in sys.argv))
    if "--reference" in sys.argv:
        i = sys.argv.index("--reference")
        tree = sys.argv[i + 1] if i + 1 < len(sys.argv) else None
        print(build_reference(tree, force="--force" in sys.argv, verbose=True))
