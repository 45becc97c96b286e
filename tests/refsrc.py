"""Locate the unmodified reference package (llm-cuda) for tests that run its own code.

The reference is installed, unmodified, into ``baseline/_ref`` (git-ignored; it travels
with the working tree to the GPU machine), or named by ``LLMCUDA_REF_SRC`` (its
``src/`` directory).  Tests that need it skip when neither is present.
"""

from __future__ import annotations

import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def reference_path() -> str | None:
    env = os.environ.get("LLMCUDA_REF_SRC")
    for cand in (env, os.path.join(ROOT, "baseline", "_ref")):
        if cand and os.path.isdir(os.path.join(cand, "llm_cuda")):
            return cand
    return None


def import_reference():
    """Return the reference's ``llm_cuda`` package (imported from its install), or None."""
    path = reference_path()
    if path is None:
        return None
    if path not in sys.path:
        sys.path.insert(0, path)
    import llm_cuda

    return llm_cuda
