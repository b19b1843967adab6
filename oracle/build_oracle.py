"""Build recipes for the CPU checkers (test infrastructure only).

* ``build_oracle()`` compiles ``oracle/akv_oracle.c`` into
  ``oracle/_build/libakv_oracle.so`` with gcc.  ``-ffp-contract=off`` keeps
  every float operation rounded once, as the reference kernel's
  ``enable_fp_fusion=False`` does.
* ``build_reference()`` compiles the reference's own CPU event compiler, the
  C++ source that ``akv/system/sglang/kernels/ops/attention/context_plan.py``
  carries in its ``_SOURCE`` string (context_plan.py:48-540), into
  ``oracle/_ref/``.  The source is read where it lies in the reference tree
  (parsed with ``ast``, never executed) and built with tvm_ffi's own
  ``build_inline`` and the reference's flags (context_plan.py:41-45).
  Nothing of it is copied into this repository; ``oracle/_ref/`` is
  git-ignored and only travels to the GPU box as a built library.

Both are called by ``__graft_entry__.build()``; ``build_reference`` is a
no-op when the reference tree is absent (as on the GPU box).
"""

from __future__ import annotations

import ast
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "_build", "libakv_oracle.so")
REF_DIR = os.path.join(HERE, "_ref")
REF_NAME = "akv_ref_context_plan"
REF_SO = os.path.join(REF_DIR, REF_NAME + ".so")
# Root of a tree that holds akv/system/sglang: AKV_REFERENCE_ROOT when set,
# else the reference package installed into baseline/_ref (pip --target of
# the reference's akv/system project, which keeps that layout).
REFERENCE_ROOT = os.environ.get(
    "AKV_REFERENCE_ROOT", os.path.join(os.path.dirname(HERE), "baseline", "_ref")
)
REF_PLAN = os.path.join(
    REFERENCE_ROOT, "akv/system/sglang/kernels/ops/attention/context_plan.py"
)


def build_oracle(force: bool = False) -> str:
    src = os.path.join(HERE, "akv_oracle.c")
    os.makedirs(os.path.dirname(ORACLE_SO), exist_ok=True)
    if (
        not force
        and os.path.exists(ORACLE_SO)
        and os.path.getmtime(ORACLE_SO) >= os.path.getmtime(src)
    ):
        return ORACLE_SO
    cmd = [
        "gcc", "-O2", "-std=c11", "-fPIC", "-shared", "-ffp-contract=off",
        "-fno-fast-math", "-Wall", "-Wno-unused-function", src, "-o", ORACLE_SO,
    ]
    subprocess.run(cmd, check=True)
    return ORACLE_SO


def _reference_source() -> str:
    tree = ast.parse(open(REF_PLAN).read())
    for node in tree.body:
        if isinstance(node, ast.Assign) and any(
            getattr(t, "id", None) == "_SOURCE" for t in node.targets
        ):
            return ast.literal_eval(node.value)
    raise RuntimeError("reference context_plan.py has no _SOURCE string")


def build_reference(force: bool = False) -> str | None:
    """Build the reference C++ event compiler; None if the tree is absent."""
    if not os.path.exists(REF_PLAN):
        return REF_SO if os.path.exists(REF_SO) else None
    if os.path.exists(REF_SO) and not force:
        return REF_SO
    from tvm_ffi.cpp import build_inline

    os.makedirs(REF_DIR, exist_ok=True)
    path = build_inline(
        REF_NAME,
        cpp_sources=_reference_source(),
        extra_cflags=["-std=c++20", "-O3"],
        build_directory=REF_DIR,
    )
    return path


if __name__ == "__main__":
    print(build_oracle(force="--force" in sys.argv))
    print(build_reference(force="--force" in sys.argv))
