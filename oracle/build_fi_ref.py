#!/usr/bin/env python
"""Build the reference's windowed decode kernel as a benchmark competitor
(oracle/_ref/fi_atfwin.so; never part of the product).

The reference's decode is not its own source file: it is a diff against
FlashInfer 0.6.13's attention/decode.cuh and utils.cuh
(kernels/flashinfer_port/decode.cuh.diff, utils.cuh.diff), compiled through
FlashInfer's JIT as a customised single-request decode module that carries the
window table as an extra int32 tensor (kernels/flashinfer_port/fiwin_common.py:
66-92 builds it with gen_customize_single_decode_module). This recipe does the
same with the installed FlashInfer (0.6.11.post2, to which both diffs apply):

  1. copy FlashInfer's header tree to a temporary directory and apply the two
     diffs there (the reference tree and the installed package stay untouched);
  2. build the customised decode module for sm_100a with FlashInfer's JIT, its
     include directory pointed at the patched copy;
  3. keep only the built shared library, as oracle/_ref/fi_atfwin.so (git
     ignores oracle/_ref; the library travels with the tree like any build
     output). The patched headers are deleted.

    python oracle/build_fi_ref.py [--reference <path of the reference tree>]

bench.py loads the library with FlashInfer's module loader and times it beside
this repository's decode on the same single request. Without the reference
tree, FlashInfer or nvcc the recipe does nothing and says why.
"""
import argparse
import os
import shutil
import subprocess
import sys
import tempfile

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "_ref", "fi_atfwin.so")
DEFAULT_REFERENCE = os.path.join(os.sep, "root", "reference")
# the module signature of the reference's JIT glue (fiwin_common.py:76-90)
MODULE_NAME = "single_decode_atfwin_dtype_bfloat16_hd128"
ADDITIONAL_TENSORS = (["maybe_alibi_slopes", "maybe_zhi_slice"], ["float", "int32_t"])
ADDITIONAL_SCALARS = (["logits_soft_cap", "sm_scale", "rope_rcp_scale", "rope_rcp_theta"],
                      ["double", "double", "double", "double"])
VARIANT = ("DefaultAttention<false, false, false, false>", "#include<flashinfer/attention/variants.cuh>")


def module_spec(dtype=None):
    """FlashInfer JitSpec of the reference's customised decode module."""
    import torch
    from flashinfer.jit.attention import gen_customize_single_decode_module
    dtype = dtype or torch.bfloat16
    return gen_customize_single_decode_module(
        MODULE_NAME, dtype, dtype, dtype, 128, 128, ADDITIONAL_TENSORS[0], ADDITIONAL_TENSORS[1],
        ADDITIONAL_SCALARS[0], ADDITIONAL_SCALARS[1], VARIANT[0], VARIANT[1], pos_encoding_mode=0,
        use_sliding_window=False, use_logits_soft_cap=False)


def build(reference=None, quiet=False):
    ref = reference or os.environ.get("ATFLASH_REFERENCE") or DEFAULT_REFERENCE
    port = os.path.join(ref, "kernels", "flashinfer_port")
    diffs = [os.path.join(port, "decode.cuh.diff"), os.path.join(port, "utils.cuh.diff")]
    if not all(os.path.exists(d) for d in diffs):
        if not quiet:
            print(f"reference diffs not found under {port}; {OUT} not built")
        return None
    work = tempfile.mkdtemp(prefix="fi_atfwin_")
    # FlashInfer fixes its target architectures and workspace when first
    # imported: set them before that (no GPU is needed to compile)
    os.environ["FLASHINFER_CUDA_ARCH_LIST"] = "10.0a"
    os.environ["FLASHINFER_WORKSPACE_BASE"] = work
    try:
        import flashinfer.jit.env as jit_env
    except ImportError:
        shutil.rmtree(work, ignore_errors=True)
        if not quiet:
            print("flashinfer is not importable; not built")
        return None
    try:
        src_inc = str(jit_env.FLASHINFER_INCLUDE_DIR)
        inc = os.path.join(work, "include")
        shutil.copytree(src_inc, inc)
        for rel, diff in (("flashinfer/attention/decode.cuh", diffs[0]), ("flashinfer/utils.cuh", diffs[1])):
            subprocess.run(["patch", "-s", os.path.join(inc, rel), diff], check=True)
        import pathlib
        jit_env.FLASHINFER_INCLUDE_DIR = pathlib.Path(inc)
        spec = module_spec()
        spec.build(verbose=False)
        so = spec.get_library_path()
        os.makedirs(os.path.dirname(OUT), exist_ok=True)
        shutil.copyfile(str(so), OUT + ".tmp")
        os.replace(OUT + ".tmp", OUT)
    finally:
        shutil.rmtree(work, ignore_errors=True)
    if not quiet:
        print("built", OUT)
    return OUT


def load():
    """The competitor module, or None when it was not built."""
    if not os.path.exists(OUT):
        return None
    spec = module_spec()
    return spec.load(OUT)


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=None)
    a = ap.parse_args()
    build(a.reference)
    sys.exit(0)
