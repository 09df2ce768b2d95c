"""In-tree build of the native libraries.

* ``libbfb_b200.so``: every CUDA kernel plus the C ABI (include/bfb_b200.h),
  compiled by nvcc for sm_100a only.  No torch dependency.
* ``_bfb_torch.so``: the PyTorch custom-op shim (csrc/torch_ops.cpp) linked
  against ``libbfb_b200.so`` with an ``$ORIGIN`` rpath.

Both land next to this file so they travel with the source tree.  Objects go
to ``_build/`` and are rebuilt only when a source or header is newer.
"""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / 'csrc'
INCLUDE = ROOT / 'include'
OBJ = PKG / '_build'
LIB = PKG / 'libbfb_b200.so'
TORCH_LIB = PKG / '_bfb_torch.so'

CUDA_HOME = os.environ.get('CUDA_HOME', '/usr/local/cuda')
NVCC = os.path.join(CUDA_HOME, 'bin', 'nvcc')
GENCODE = ['-gencode', 'arch=compute_100a,code=sm_100a']
CU_SOURCES = ['capi.cu', 'scan.cu', 'radix.cu', 'bev_pool.cu', 'voxelize.cu', 'scatter.cu', 'spconv.cu',
              'spconv_conv.cu']


def _headers() -> list[Path]:
    return list(CSRC.glob('*.cuh')) + list(CSRC.glob('*.h')) + list(INCLUDE.glob('*.h'))


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def _run(cmd: list[str]) -> None:
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(' '.join(cmd) + '\n' + r.stdout + r.stderr)
        raise RuntimeError(f'build step failed: {cmd[0]} (exit {r.returncode})')


DEBUG_DIR = PKG / 'debug'


def build_cuda_lib(verbose: bool = False, debug_checks: bool = False) -> Path:
    """libbfb_b200.so; with ``debug_checks`` the debug variant (device index
    checks counted into an error word, -DBFB_DEBUG_CHECKS) in ``debug/``."""
    obj = OBJ / 'debug' if debug_checks else OBJ
    lib = DEBUG_DIR / LIB.name if debug_checks else LIB
    obj.mkdir(parents=True, exist_ok=True)
    lib.parent.mkdir(exist_ok=True)
    hdrs = _headers()
    objs = []
    for src in CU_SOURCES:
        s = CSRC / src
        if not s.exists():
            continue
        o = obj / (s.stem + '.o')
        objs.append(o)
        if _stale(o, [s] + hdrs):
            cmd = [NVCC, '-std=c++17', *GENCODE, '-lineinfo', '-O3', '-Xcompiler', '-fPIC',
                   f'-I{INCLUDE}', '-c', str(s), '-o', str(o)] + (['-DBFB_DEBUG_CHECKS'] if debug_checks else [])
            if verbose:
                cmd.insert(1, '-Xptxas=-v')
                print(' '.join(cmd))
            _run(cmd)
    if _stale(lib, objs):
        _run([NVCC, '-shared', *GENCODE, '-o', str(lib), *map(str, objs), '-lcudart'])
    return lib


def build_torch_ops() -> Path:
    import torch
    from torch.utils import cpp_extension

    src = CSRC / 'torch_ops.cpp'
    if not _stale(TORCH_LIB, [src, LIB] + list(INCLUDE.glob('*.h'))):
        return TORCH_LIB
    incs = cpp_extension.include_paths(device_type='cuda')
    libdirs = cpp_extension.library_paths(device_type='cuda')
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    cmd = ['g++', '-O2', '-std=c++17', '-shared', '-fPIC', f'-D_GLIBCXX_USE_CXX11_ABI={abi}',
           '-DTORCH_EXTENSION_NAME=_bfb_torch', f'-I{INCLUDE}']
    cmd += [f'-I{p}' for p in incs] + [f'-I{CUDA_HOME}/include']
    cmd += [str(src), '-o', str(TORCH_LIB), f'-L{PKG}', '-lbfb_b200']
    cmd += [f'-L{p}' for p in libdirs] + [f'-L{CUDA_HOME}/lib64']
    cmd += ['-lc10', '-lc10_cuda', '-ltorch_cpu', '-ltorch_cuda', '-ltorch', '-lcudart',
            "-Wl,-rpath,$ORIGIN"]
    cmd += [f'-Wl,-rpath,{p}' for p in libdirs]
    _run(cmd)
    return TORCH_LIB


def build(verbose: bool = False) -> None:
    build_cuda_lib(verbose)
    build_torch_ops()


if __name__ == '__main__':
    if '--debug-checks' in sys.argv:
        print('built', build_cuda_lib('-v' in sys.argv, debug_checks=True))
    else:
        build(verbose='-v' in sys.argv)
        print('built', LIB, TORCH_LIB)
