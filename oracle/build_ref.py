"""TEST INFRASTRUCTURE ONLY: builds the reference's own device LSAP solver for the GPU-baseline leg.

The reference keeps its CUDA solver (``lsap_kernel`` / ``batch_lap_cuda``) as C++ source strings in
``kernels_lap.py`` (``_CUDA_SOURCE``, ``_CPP_SOURCE``; kernels_lap.py:69-310) and compiles them with
``torch.utils.cpp_extension.load_inline`` under the name ``rfdetr_lab_batch_lap`` with
``-O3 --use_fast_math`` (kernels_lap.py:315-329).  This recipe reads those strings from the
reference tree where they lie, compiles them with the same call and flags for sm_100 in a scratch
directory outside this repository, and copies only the resulting extension module to
``oracle/_ref/`` (git-ignored; it travels to the GPU box with the tree, where the reference tree
itself is absent).  ``bench.py`` loads it to time the reference's own GPU solver on the same
device and batches as ``rfm_lsap_dense``.

Run where the reference tree exists:  ``python -m oracle.build_ref``.
"""

from __future__ import annotations

import ast
import os
import shutil
import sys
import tempfile

HERE = os.path.dirname(os.path.abspath(__file__))
REF_DIR = os.path.join(HERE, "_ref")
REFERENCE = os.environ.get("RFM_REFERENCE_TREE", "/root/reference")
MODULE = "rfdetr_lab_batch_lap"
SO_PATH = os.path.join(REF_DIR, MODULE + ".so")


def _reference_sources(path: str) -> tuple[str, str]:
    """The two source strings of kernels_lap.py, read without importing the module."""
    tree = ast.parse(open(path).read())
    found: dict[str, str] = {}
    for node in tree.body:
        if isinstance(node, (ast.Assign, ast.AnnAssign)):
            targets = node.targets if isinstance(node, ast.Assign) else [node.target]
            for t in targets:
                if isinstance(t, ast.Name) and t.id in ("_CUDA_SOURCE", "_CPP_SOURCE"):
                    found[t.id] = ast.literal_eval(node.value)
    return found["_CUDA_SOURCE"], found["_CPP_SOURCE"]


def build(force: bool = False) -> str | None:
    """Build the module when the reference tree is present; returns its path (or None)."""
    src = os.path.join(REFERENCE, "kernels_lap.py")
    if not os.path.exists(src):
        return SO_PATH if os.path.exists(SO_PATH) else None
    if not force and os.path.exists(SO_PATH) and os.path.getmtime(SO_PATH) >= os.path.getmtime(src):
        return SO_PATH
    cuda_src, cpp_src = _reference_sources(src)
    os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0")
    from torch.utils.cpp_extension import load_inline

    scratch = tempfile.mkdtemp(prefix="rfm_ref_lap_")
    try:
        load_inline(name=MODULE, cpp_sources=cpp_src, cuda_sources=cuda_src, functions=["batch_lap_cuda"],
                    extra_cuda_cflags=["-O3", "--use_fast_math"], build_directory=scratch, verbose=False)
        os.makedirs(REF_DIR, exist_ok=True)
        shutil.copy2(os.path.join(scratch, MODULE + ".so"), SO_PATH + ".tmp")
        os.replace(SO_PATH + ".tmp", SO_PATH)
    finally:
        shutil.rmtree(scratch, ignore_errors=True)
    return SO_PATH


def load():
    """Import the built module (``batch_lap_cuda(cost [P, W, T] float32 CUDA) -> [P, W] int64``)."""
    import importlib.machinery
    import importlib.util

    import torch  # noqa: F401  (the extension links against torch's libraries)

    if not os.path.exists(SO_PATH):
        return None
    loader = importlib.machinery.ExtensionFileLoader(MODULE, SO_PATH)
    spec = importlib.util.spec_from_file_location(MODULE, SO_PATH, loader=loader)
    mod = importlib.util.module_from_spec(spec)
    loader.exec_module(mod)
    return mod


if __name__ == "__main__":
    print(build(force="--force" in sys.argv))
