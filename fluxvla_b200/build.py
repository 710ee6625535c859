"""Build libfluxvla_b200.so in-tree with nvcc for sm_100a.

    python -m fluxvla_b200.build [--verbose]

The library is a single translation unit (csrc/fluxvla_b200.cu including
the kernel headers) exposing the C ABI of include/fluxvla_b200.h.  It links
only the CUDA runtime; the driver entry point for tensor-map encoding is
resolved at run time through cudaGetDriverEntryPoint.
"""
from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
SRC = os.path.join(HERE, 'csrc', 'fluxvla_b200.cu')
OUT = os.path.join(HERE, 'libfluxvla_b200.so')
NVCC = os.environ.get('NVCC', '/usr/local/cuda/bin/nvcc')

FLAGS = ['-gencode', 'arch=compute_100a,code=sm_100a', '-lineinfo', '-O3',
         '-std=c++17', '-Xcompiler', '-fPIC', '-shared',
         '-I' + os.path.join(ROOT, 'include'), '-lcudart']


def sources():
    d = os.path.join(HERE, 'csrc')
    return [os.path.join(d, f) for f in os.listdir(d)] + [
        os.path.join(ROOT, 'include', 'fluxvla_b200.h')]


def needs_build() -> bool:
    if not os.path.exists(OUT):
        return True
    t = os.path.getmtime(OUT)
    return any(os.path.getmtime(s) > t for s in sources())


def build(verbose: bool = False, force: bool = False) -> str:
    if not force and not needs_build():
        return OUT
    cmd = [NVCC] + FLAGS + (['-Xptxas', '-v'] if verbose else []) + [
        SRC, '-o', OUT + '.tmp']
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError('nvcc failed:\n' + r.stdout + r.stderr)
    if verbose:
        print(r.stdout + r.stderr)
    os.replace(OUT + '.tmp', OUT)
    return OUT


EXT_SRC = os.path.join(HERE, 'csrc', 'torch_ext.cpp')


def ext_path() -> str:
    import sysconfig
    return os.path.join(HERE, '_C' + sysconfig.get_config_var('EXT_SUFFIX'))


def build_ext(force: bool = False, verbose: bool = False) -> str:
    """The thin torch C++ extension (fluxvla_b200._C) over the C ABI, linked
    against libfluxvla_b200.so next to it (rpath $ORIGIN)."""
    import sysconfig

    import torch
    from torch.utils import cpp_extension as ce
    out = ext_path()
    hdr = os.path.join(ROOT, 'include', 'fluxvla_b200.h')
    if (not force and os.path.exists(out) and
            os.path.getmtime(out) > max(os.path.getmtime(EXT_SRC),
                                        os.path.getmtime(hdr),
                                        os.path.getmtime(OUT))):
        return out
    cxx = os.environ.get('CXX', 'g++')
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    cmd = [cxx, '-O2', '-std=c++17', '-shared', '-fPIC', EXT_SRC, '-o', out + '.tmp',
           f'-D_GLIBCXX_USE_CXX11_ABI={abi}', '-DTORCH_EXTENSION_NAME=_C',
           '-DTORCH_API_INCLUDE_EXTENSION_H',
           '-I' + sysconfig.get_paths()['include'],
           '-I/usr/local/cuda/include']
    cmd += ['-I' + p for p in ce.include_paths()]
    cmd += ['-L' + p for p in ce.library_paths()]
    cmd += ['-lc10', '-ltorch', '-ltorch_cpu', '-ltorch_python', '-lc10_cuda',
            '-ltorch_cuda', '-L' + HERE, '-lfluxvla_b200',
            '-L/usr/local/cuda/lib64', '-lcudart',
            '-Wl,-rpath,$ORIGIN']
    cmd += ['-Wl,-rpath,' + p for p in ce.library_paths()]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError('torch extension build failed:\n' + r.stdout + r.stderr)
    if verbose:
        print(r.stdout + r.stderr)
    os.replace(out + '.tmp', out)
    return out


if __name__ == '__main__':
    build(verbose='--verbose' in sys.argv, force=True)
    print(OUT)
    print(build_ext(force=True))
