"""Build libornith_moe_b200.so in-tree with nvcc for sm_100a.

The library is pure CUDA C++ behind a C ABI (include/ornith_moe_b200.h): no
torch types cross the boundary.  -fmad=false keeps every fp32 step of the
reference's fixed-order arithmetic un-contracted.
"""
import os
import subprocess
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / 'csrc'
LIB = HERE / 'libornith_moe_b200.so'
# the same library with the debug bounds checks (-DORNITH_DEBUG_BOUNDS=1): data-
# dependent indices outside their buffers raise flag 128 instead of faulting
DEBUG_LIB = HERE / 'libornith_moe_b200_debug.so'
DEBUG_FLAGS = ('-DORNITH_DEBUG_BOUNDS=1',)
SOURCES = ['moe_api.cu', 'moe_generic.cu', 'moe_decode.cu', 'moe_decode1.cu', 'moe_prefill.cu', 'moe_noalloc.cu', 'dense_g256.cu', 'head_i8.cu',
           'ep_plan.cu', 'ep_p2p.cu']
NVCC = os.environ.get('NVCC', '/usr/local/cuda/bin/nvcc')
FLAGS = ['-gencode', 'arch=compute_100a,code=sm_100a', '-lineinfo', '-O3', '-std=c++17',
         '-fmad=false', '-Xcompiler', '-fPIC,-fvisibility=hidden', '-shared', '-rdc=false',
         f'-I{HERE.parent / "include"}']


def stale():
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    deps = [CSRC / s for s in SOURCES] + list(CSRC.glob('*.cuh')) + list(CSRC.glob('*.h')) + list((HERE.parent / 'include').glob('*.h'))
    return any(d.stat().st_mtime > t for d in deps)


def build(force=False, verbose=False, flags=(), out=None):
    """Compile the library.  Extra nvcc flags (the kernels' build-time
    options: -DORNITH_DECODE_GATE_COST=…, -DORNITH_DECODE_DOWN_COST=…, the
    trace builds -DORNITH_DECODE_TRACE / -DORNITH_PREFILL_TRACE) come from `flags` and
    from ORNITH_MOE_B200_NVCC_FLAGS; the default build sets none of them
    (DEBUG_FLAGS make the debug-bounds library).
    `out` writes a variant library elsewhere (always rebuilt), which
    ORNITH_MOE_B200_LIB then selects at run time, so that a default and a
    variant build can be measured side by side."""
    target = Path(out) if out else LIB
    if not out and not force and not stale():
        return LIB
    extra = [*flags, *os.environ.get('ORNITH_MOE_B200_NVCC_FLAGS', '').split()]
    # one object per source, compiled in parallel, then one link step
    objdir = HERE.parent / '_build' / target.stem
    objdir.mkdir(parents=True, exist_ok=True)
    compile_flags = [f for f in FLAGS if f != '-shared']

    def compile_one(src):
        obj = objdir / (Path(src).stem + '.o')
        cmd = [NVCC, *compile_flags, *extra, '-c', str(CSRC / src), '-o', str(obj)]
        if verbose:
            cmd.insert(1, '-Xptxas=-v')
        subprocess.run(cmd, check=True)
        return obj

    from concurrent.futures import ThreadPoolExecutor
    with ThreadPoolExecutor(max_workers=min(len(SOURCES), os.cpu_count() or 1)) as pool:
        objs = list(pool.map(compile_one, SOURCES))
    subprocess.run([NVCC, '-gencode', 'arch=compute_100a,code=sm_100a', '-shared', *map(str, objs),
                    '-o', str(target)], check=True)
    return target


if __name__ == '__main__':
    import argparse
    p = argparse.ArgumentParser(description='build libornith_moe_b200.so for sm_100a')
    p.add_argument('-v', '--verbose', action='store_true', help='print ptxas register and spill counts')
    p.add_argument('--out', default=None, help='write a variant library to this path')
    p.add_argument('--flag', action='append', default=[], help='extra nvcc flag, e.g. --flag=-DORNITH_DECODE_GATE_COST=4')
    a = p.parse_args()
    print(build(force=True, verbose=a.verbose, flags=a.flag, out=a.out))
