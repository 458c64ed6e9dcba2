"""Compile the reference's routed-MoE HIP sources for the CPU (test infrastructure).

The reference ships its routed path only as HIP C++ for gfx1151.  This recipe
builds those sources, where they lie in the reference checkout, into host
shared libraries under oracle/_ref/ so that their outputs pin the C oracle:

  1. copy each needed source and header into oracle/_ref/src/<library>/,
     rewriting only the CUDA/HIP launch syntax `kernel<<<grid,block,smem,stream>>>(args)`
     into `::hipshim::Launch(grid,block,smem,stream)(kernel,args)` because g++
     cannot parse triple chevrons; nothing else in the text changes; the
     copies are deleted once the library is compiled;
  2. compile with g++ against oracle/hipshim (a CPU SIMT shim written for this
     repository) using the reference's numerics flags (-O2 -ffp-contract=off,
     correctly rounded division, -DORNITH_PREFILL_OUTPUT32=1 as in
     scripts/build-native.sh:45-47).

Outputs (git-ignored, never committed):
  oracle/_ref/libref_routed_storage_n32.so   kernels/routed_storage/ (production library)
  oracle/_ref/libref_routed_direct_n16.so    kernels/routed/ (N16 checkpoint layout)
  oracle/_ref/libref_dense_n32.so            kernels/dense_n32/ (dense G256 projections)
  oracle/_ref/libref_head_i8.so              kernels/head/ (W8 LM head)

Usage: python oracle/build_ref.py [--reference DIR]   (default: ORNITH_REFERENCE, else
BASELINE.json's reference_path)
The reference checkout exists only in the build container; on other machines
the prebuilt libraries travel with the repository snapshot.
"""
import argparse
import os
import re
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / '_ref'
LIBS = {
    'routed_storage_n32': ('kernels/routed_storage',
                           ['routed_storage_n32_consumer.cpp', 'routed_storage_n32_prefill.h',
                            'routed_direct_api.h', 'portable_exp.h'],
                           'routed_storage_n32_consumer.cpp'),
    'routed_direct_n16': ('kernels/routed',
                          ['routed_direct_consumer.cpp', 'routed_direct_prefill.h',
                           'routed_direct_api.h', 'portable_exp.h'],
                          'routed_direct_consumer.cpp'),
    'dense_n32': ('kernels/dense_n32',
                  ['dense_g256_consumer.cpp', 'dense_g256_api.h'],
                  'dense_g256_consumer.cpp'),
    'head_i8': ('kernels/head',
                ['head_i8_tile_consumer.cpp', 'head_i8_tile_api.h'],
                'head_i8_tile_consumer.cpp'),
}
ROOT = HERE.parent


def reference_root():
    """The reference checkout: the ORNITH_REFERENCE environment variable, else
    the `reference_path` that BASELINE.json at the repository root records;
    None when neither names an existing checkout (as on the GPU boxes, where
    the prebuilt libraries travel with the repository instead)."""
    path = os.environ.get('ORNITH_REFERENCE')
    if not path:
        try:
            import json
            path = json.loads((ROOT / 'BASELINE.json').read_text()).get('reference_path')
        except (OSError, ValueError):
            path = None
    if path and Path(path, 'kernels').is_dir():
        return Path(path)
    return None


LAUNCH = re.compile(r'(\b[A-Za-z_]\w*(?:<[^<>;()]*>)?)\s*<<<(.*?)>>>\s*\(')


def rewrite(text):
    return LAUNCH.sub(lambda m: f'::hipshim::Launch({m.group(2)})({m.group(1)},', text)


def build(reference, names=None):
    reference = Path(reference)
    OUT.mkdir(exist_ok=True)
    built = []
    for name, (subdir, files, main) in LIBS.items():
        if names and name not in names:
            continue
        src_dir = OUT / 'src' / name
        src_dir.mkdir(parents=True, exist_ok=True)
        for f in files:
            text = (reference / subdir / f).read_text()
            (src_dir / f).write_text(rewrite(text))
        lib = OUT / f'libref_{name}.so'
        cmd = ['g++', '-std=c++20', '-O2', '-ffp-contract=off', '-fopenmp', '-fPIC', '-shared',
               '-w', '-Wno-psabi', '-DORNITH_PREFILL_OUTPUT32=1', f'-I{HERE / "hipshim"}', f'-I{src_dir}',
               str(src_dir / main), '-o', str(lib)]
        try:
            subprocess.run(cmd, check=True)
        finally:
            # only the compiled library stays: no copy of the reference's
            # sources remains in the repository tree
            shutil.rmtree(src_dir, ignore_errors=True)
        built.append(lib)
    shutil.rmtree(OUT / 'src', ignore_errors=True)
    return built


def main():
    parser = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    parser.add_argument('--reference', default=None,
                        help='reference checkout (default: ORNITH_REFERENCE, else BASELINE.json reference_path)')
    args = parser.parse_args()
    args.reference = args.reference or reference_root()
    if args.reference is None or not Path(args.reference, 'kernels').is_dir():
        print(f'reference checkout not found at {args.reference}; nothing built', file=sys.stderr)
        return 1
    for lib in build(args.reference):
        print(lib)
    return 0


if __name__ == '__main__':
    sys.exit(main())
