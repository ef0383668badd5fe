#!/usr/bin/env python
"""Build oracle/_ref/atflash_ref from the reference tree (test and baseline
infrastructure, never part of the product).

The reference's CPU path for windowed attention is its own torch code:
atflash/reference.py (ref_window_attn, the fp32 correctness baseline) and
atflash/window_table.py (the window rule it uses), plus the package's
__init__.py. This recipe byte-compiles those three files, where they lie in the
reference tree, into sourceless modules of a package named ``atflash_ref``
(renamed so that it never shadows this repository's own ``atflash`` package; the
reference imports its modules relatively, so the name does not matter to it).

    python oracle/build_ref.py [--reference <path of the reference tree>]

The reference tree is found through --reference, the ATFLASH_REFERENCE
environment variable or the default path. Output goes to oracle/_ref/ only,
which git ignores and which travels with the tree to the GPU box, like a built
library. Without the reference tree the recipe does nothing and says so;
bench.py then times the numpy restatement (oracle/attention.py) instead.

Used by bench.py --impl reference and by the cpu_baseline leg of bench.py.
"""
import argparse
import os
import py_compile
import shutil
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "_ref", "atflash_ref")
FILES = ("__init__.py", "reference.py", "window_table.py")
DEFAULT_REFERENCE = os.path.join(os.sep, "root", "reference")


def build(reference=None, quiet=False):
    ref = reference or os.environ.get("ATFLASH_REFERENCE") or DEFAULT_REFERENCE
    src_dir = os.path.join(ref, "atflash")
    if not all(os.path.exists(os.path.join(src_dir, f)) for f in FILES):
        if not quiet:
            print(f"reference package not found under {src_dir}; oracle/_ref not built")
        return None
    tmp = OUT + ".tmp"
    if os.path.exists(tmp):
        shutil.rmtree(tmp)
    os.makedirs(tmp)
    for f in FILES:
        py_compile.compile(os.path.join(src_dir, f), cfile=os.path.join(tmp, f[:-3] + ".pyc"),
                           doraise=True, invalidation_mode=py_compile.PycInvalidationMode.UNCHECKED_HASH)
    with open(os.path.join(tmp, "BUILT_FROM"), "w") as fh:
        fh.write(f"{src_dir} ({', '.join(FILES)}), python {sys.version.split()[0]}\n")
    if os.path.exists(OUT):
        shutil.rmtree(OUT)
    os.replace(tmp, OUT)
    if not quiet:
        print("built", OUT)
    return OUT


def load():
    """Import and return the compiled reference package, or None when it has not
    been built (or was built for another Python)."""
    base = os.path.dirname(OUT)
    if not os.path.exists(os.path.join(OUT, "reference.pyc")):
        return None
    if base not in sys.path:
        sys.path.insert(0, base)
    try:
        import atflash_ref
    except ImportError:
        return None
    return atflash_ref


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=None)
    a = ap.parse_args()
    build(a.reference)
