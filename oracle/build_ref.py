"""Compile the reference's own C++ tree builders into oracle/_ref/ -- TEST INFRASTRUCTURE ONLY.

The reference keeps its C++ inside Python strings:
  - inference/hf/tree_build_ext.py `_CPP_SOURCE` (build_single / build_mixture / Tree.follow), and
  - the SGLang patch's ddtree_utils.py `_CPP_SOURCE` (batched build_trees), a new file inside
    inference/sglang/patches/sglang-v0.5.22-mfd.patch.
This recipe reads those strings from the mounted reference (never copied into this repository) and
compiles each with torch.utils.cpp_extension.load_inline into oracle/_ref/, exactly the way the
reference's own tests build them (tests/test_sglang_tree_builder.py:28-48).  The resulting .so files are
git-ignored but travel to the GPU box, where `load()` imports them without the reference mounted.

    python oracle/build_ref.py            # needs the reference checkout (MFD_REFERENCE_ROOT); no-op without it
"""

from __future__ import annotations

import importlib.machinery
import importlib.util
import os
import re
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
REF_DIR = os.path.join(HERE, "_ref")
REFERENCE = os.environ.get("MFD_REFERENCE_ROOT", "/root/reference")
HF_EXT = "inference/hf/tree_build_ext.py"
PATCH = "inference/sglang/patches/sglang-v0.5.22-mfd.patch"
SGL_FILE = "python/sglang/srt/speculative/ddtree_utils.py"

NAMES = {"hf": "mfd_ref_tree_build_ext", "sglang": "mfd_ref_sglang_build_trees"}


def _new_file_from_patch(patch_path: str, path: str) -> str:
    out, inside = [], False
    with open(patch_path, encoding="utf-8") as f:
        for line in f:
            if line.startswith("diff --git "):
                inside = line.strip().endswith(f"b/{path}")
                continue
            if inside and line.startswith("+") and not line.startswith("+++"):
                out.append(line[1:])
    if not out:
        raise FileNotFoundError(path)
    return "".join(out)


def _cpp_string(text: str) -> str:
    m = re.search(r'_CPP_SOURCE = r"""(.*?)"""', text, re.S)
    if m is None:
        raise RuntimeError("no _CPP_SOURCE string found")
    return m.group(1)


def sources() -> dict[str, str]:
    with open(os.path.join(REFERENCE, HF_EXT), encoding="utf-8") as f:
        hf = _cpp_string(f.read())
    sgl = _cpp_string(_new_file_from_patch(os.path.join(REFERENCE, PATCH), SGL_FILE))
    return {"hf": hf, "sglang": sgl}


def build(verbose: bool = False) -> bool:
    """Compile both builders; returns False when the reference is not mounted."""
    if not os.path.isdir(REFERENCE):
        return False
    from torch.utils.cpp_extension import load_inline

    os.makedirs(REF_DIR, exist_ok=True)
    for key, src in sources().items():
        name = NAMES[key]
        so = os.path.join(REF_DIR, f"{name}.so")
        if os.path.exists(so):
            continue
        load_inline(name=name, cpp_sources=[src], extra_cflags=["-O3"], build_directory=REF_DIR, verbose=verbose)
    # keep only the compiled modules: load_inline leaves the extracted source and objects beside them
    for f in os.listdir(REF_DIR):
        if not f.endswith(".so"):
            os.remove(os.path.join(REF_DIR, f))
    return True


def available() -> bool:
    return all(os.path.exists(os.path.join(REF_DIR, f"{n}.so")) for n in NAMES.values())


_LOADED = {}


def load(key: str):
    """Import a prebuilt reference builder ('hf' or 'sglang') from oracle/_ref/."""
    if key in _LOADED:
        return _LOADED[key]
    import torch  # noqa: F401  (the extension links against libtorch)

    name = NAMES[key]
    path = os.path.join(REF_DIR, f"{name}.so")
    if not os.path.exists(path):
        raise FileNotFoundError(f"{path} is not built (python oracle/build_ref.py with the reference mounted)")
    loader = importlib.machinery.ExtensionFileLoader(name, path)
    spec = importlib.util.spec_from_file_location(name, path, loader=loader)
    mod = importlib.util.module_from_spec(spec)
    loader.exec_module(mod)
    _LOADED[key] = mod
    return mod


if __name__ == "__main__":
    ok = build(verbose="-v" in sys.argv)
    print("built" if ok else f"reference not mounted at {REFERENCE}; nothing built")
