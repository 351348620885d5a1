"""Build libcpde_b200.so and bin/cpde_server in-tree for sm_100a.

    python -m cpde_b200.build

nvcc cross-compiles without a GPU. The library is one translation unit
(csrc/library.cu); the server is a host program linked against it with an
$ORIGIN-relative rpath so the pair can be moved together.
"""
import os
import subprocess
import sys
from pathlib import Path

PACKAGE = Path(__file__).resolve().parent
CSRC = PACKAGE / 'csrc'
LIBRARY = PACKAGE / 'libcpde_b200.so'
SERVER = PACKAGE / 'bin' / 'cpde_server'
ARCH = ['-gencode', 'arch=compute_100a,code=sm_100a']


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
        cmd = [nvcc, *ARCH, '-lineinfo', '-O3', '-std=c++17', '-Xcompiler', '-fPIC', '-shared',
               f'--split-compile={os.cpu_count() or 1}',
               '--expt-relaxed-constexpr', '-o', LIBRARY, CSRC / 'library.cu', '-lnvrtc']
        if verbose_ptxas:
            cmd.insert(1, '-Xptxas=-v')
        _run(cmd)
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
