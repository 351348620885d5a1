"""Build libcpde_b200.so and bin/cpde_server in-tree for sm_100a.

    python -m cpde_b200.build

nvcc cross-compiles without a GPU. The library is four translation units
compiled in parallel (csrc/library.cu: engine core, C ABI, allocation-free
entry; fast_forward.cu, fast_backward.cu, fast_head.cu: the fast-tier
dispatch and the kernels it instantiates); the server is a host program
linked against it with an $ORIGIN-relative rpath so the pair can be moved
together.
"""
import os
import subprocess
import sys
from pathlib import Path

PACKAGE = Path(__file__).resolve().parent
CSRC = PACKAGE / 'csrc'
LIBRARY = PACKAGE / 'libcpde_b200.so'
SERVER = PACKAGE / 'bin' / 'cpde_server'
BUILD = PACKAGE / '_build'
ARCH = ['-gencode', 'arch=compute_100a,code=sm_100a']
UNITS = ['library', 'fast_forward', 'fast_backward', 'fast_head']


def _run(cmd):
    print(' '.join(str(c) for c in cmd), flush=True)
    subprocess.run([str(c) for c in cmd], check=True)


def _stale(target, sources):
    if not target.exists():
        return True
    mtime = target.stat().st_mtime
    return any(s.stat().st_mtime > mtime for s in sources)


def build(force=False, verbose_ptxas=False):
    from . import codegen
    codegen.write()
    nvcc = os.environ.get('NVCC', 'nvcc')
    sources = sorted(CSRC.glob('*.cu')) + sorted(CSRC.glob('*.cuh')) + sorted(CSRC.glob('*.hpp'))
    sources += sorted((CSRC / 'generated').glob('*.cuh'))
    sources.append(PACKAGE.parent / 'include' / 'cpde_b200.h')
    if force or _stale(LIBRARY, sources):
        # One object per translation unit, compiled in parallel; each unit is
        # compiled whole (no --split-compile, whose partitioning changed the
        # code of unrelated kernels from one build to the next).
        BUILD.mkdir(exist_ok=True)
        procs, objects = [], []
        for unit in UNITS:
            obj = BUILD / (unit + '.o')
            cmd = [nvcc, *ARCH, '-lineinfo', '-O3', '-std=c++17', '-Xcompiler', '-fPIC', '-c',
                   '--expt-relaxed-constexpr', '-o', obj, CSRC / (unit + '.cu')]
            if verbose_ptxas:
                cmd.insert(1, '-Xptxas=-v')
            print(' '.join(map(str, cmd)), flush=True)
            procs.append(subprocess.Popen([str(c) for c in cmd]))
            objects.append(obj)
        failed = [unit for unit, proc in zip(UNITS, procs) if proc.wait() != 0]
        if failed:
            raise RuntimeError(f'nvcc failed on {", ".join(failed)}')
        _run([nvcc, *ARCH, '-shared', '-o', LIBRARY, *objects, '-lnvrtc'])
    SERVER.parent.mkdir(exist_ok=True)
    server_sources = [CSRC / 'server_main.cpp', CSRC / 'wire.hpp', CSRC / 'common.hpp', LIBRARY]
    if force or _stale(SERVER, server_sources):
        cuda = Path(os.environ.get('CUDA_HOME', '/usr/local/cuda'))
        _run(['g++', '-std=c++17', '-O2', '-pthread', f'-I{cuda / "include"}', '-o', SERVER,
              CSRC / 'server_main.cpp', f'-L{PACKAGE}', '-lcpde_b200', f'-L{cuda / "lib64"}', '-lcudart',
              "-Wl,-rpath,$ORIGIN/..", f'-Wl,-rpath,{cuda / "lib64"}',
              '-Wl,--allow-shlib-undefined'])
    return LIBRARY, SERVER


if __name__ == '__main__':
    build(force='--force' in sys.argv, verbose_ptxas='--ptxas' in sys.argv)
