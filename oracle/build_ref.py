"""Compile the reference's own BA CUDA extension into ``oracle/_ref/`` (test infrastructure).

This is part of the oracle, not of the product.  It compiles the single reference
source ``src/blast3r/extensions/cujac/sfm_jacobian_rigs.cu`` (naver/blast3r), where it
lies in the reference checkout, into a torch extension named
``ba_with_rigs_cuda_kernels`` for sm_100a.  The reference's own ``setup.py`` is NOT
used: this recipe calls ``torch.utils.cpp_extension.load`` with our own flags, which
mirror the reference build (``-O3``, no ``--use_fast_math``; reference ``setup.py:22-27``).

The built ``.so`` is git-ignored but travels to the GPU box, where the GPU tests use it
to pin the oracle's residual/Jacobian restatement to the reference kernels' actual
outputs (``tests/test_ref_kernels_gpu.py``).  Nothing in the product imports it.

Usage:  python oracle/build_ref.py [--reference /path/to/blast3r]
"""
import argparse
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT_DIR = os.path.join(HERE, '_ref')
REL_SRC = os.path.join('src', 'blast3r', 'extensions', 'cujac', 'sfm_jacobian_rigs.cu')
NAME = 'ba_with_rigs_cuda_kernels'


def default_reference():
    """The reference checkout: $B3R_REFERENCE, else a ``reference`` directory beside this
    repository's own directory; None when neither exists (the GPU box has no checkout and
    uses the prebuilt extension)."""
    cands = [os.environ.get('B3R_REFERENCE'),
             os.path.join(os.path.dirname(os.path.dirname(HERE)), 'reference')]
    for c in cands:
        if c and os.path.isfile(os.path.join(c, REL_SRC)):
            return c
    return None


def built_path():
    """Path of the compiled reference extension, or None if it was never built."""
    if not os.path.isdir(OUT_DIR):
        return None
    for f in sorted(os.listdir(OUT_DIR)):
        if f.startswith(NAME) and f.endswith('.so'):
            return os.path.join(OUT_DIR, f)
    return None


def build(reference_root, verbose=False):
    src = os.path.join(reference_root, REL_SRC)
    if not os.path.isfile(src):
        raise FileNotFoundError(f'reference source not found: {src}')
    os.makedirs(OUT_DIR, exist_ok=True)
    from torch.utils.cpp_extension import load
    load(name=NAME, sources=[src], build_directory=OUT_DIR, verbose=verbose,
         extra_cflags=['-O3'],
         extra_cuda_cflags=['-O3', '-gencode', 'arch=compute_100a,code=sm_100a', '-lineinfo'],
         is_python_module=True)
    return built_path()


def load_built():
    """Import the prebuilt reference extension from ``oracle/_ref`` (no compilation)."""
    path = built_path()
    if path is None:
        return None
    import importlib.util
    spec = importlib.util.spec_from_file_location(NAME, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


if __name__ == '__main__':
    ap = argparse.ArgumentParser()
    ap.add_argument('--reference', default=default_reference())
    ap.add_argument('-v', '--verbose', action='store_true')
    a = ap.parse_args()
    if a.reference is None:
        sys.exit('no reference checkout found: pass --reference or set B3R_REFERENCE')
    p = build(a.reference, verbose=a.verbose)
    print(p)
    sys.exit(0 if p else 1)
