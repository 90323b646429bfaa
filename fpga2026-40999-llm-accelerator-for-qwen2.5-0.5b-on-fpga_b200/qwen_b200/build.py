"""Builds libqwen_b200.so in-tree: nvcc for the sm_100a kernels and the host
engine, the system gcc for the asset code, linked with a static CUDA runtime.

    python -m qwen_b200.build [--verbose-ptxas]
"""
import argparse
import concurrent.futures
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parents[1]
REPO = PKG.parent
CSRC = PKG / 'csrc'
BUILD = PKG / '_build'
LIB = PKG / 'libqwen_b200.so'
INCLUDE = REPO / 'include'

ARCH = ['-gencode', 'arch=compute_100a,code=sm_100a']
NVCC_FLAGS = ['-O3', '-std=c++17', '-lineinfo', '-Xcompiler', '-fPIC', '-Xcompiler', '-fopenmp',
              f'-I{INCLUDE}', f'-I{CSRC}']


def _gcc():
    # The image exports CC=/opt/gcc/bin/gcc whose driver lacks libgomp.spec.
    return '/usr/bin/gcc' if os.path.exists('/usr/bin/gcc') else 'gcc'


def _nvcc():
    for cand in (shutil.which('nvcc'), '/usr/local/cuda/bin/nvcc'):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError('nvcc not found')


def _run(cmd):
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode:
        raise RuntimeError(f"build step failed: {' '.join(cmd)}\n{proc.stdout}\n{proc.stderr}")
    return proc.stdout + proc.stderr


def sources():
    return sorted(CSRC.glob('*.cu')) + sorted(CSRC.glob('*.c')) + sorted(CSRC.glob('*.cpp'))


def build(verbose_ptxas=False, force=False):
    """Compile every source that is newer than its object, then link."""
    BUILD.mkdir(exist_ok=True)
    headers = list(CSRC.glob('*.h')) + list(CSRC.glob('*.cuh')) + list(INCLUDE.glob('*.h'))
    newest_header = max((p.stat().st_mtime for p in headers), default=0)
    nvcc = _nvcc()
    jobs, objs = [], []
    for src in sources():
        obj = BUILD / (src.name + '.o')
        objs.append(obj)
        stale = force or not obj.exists() or obj.stat().st_mtime < max(src.stat().st_mtime, newest_header)
        if not stale:
            continue
        if src.suffix == '.cu':
            cmd = [nvcc, *ARCH, *NVCC_FLAGS, '-ccbin', _gcc(), '-c', str(src), '-o', str(obj)]
            if verbose_ptxas:
                cmd[1:1] = ['-Xptxas', '-v']
        elif src.suffix == '.cpp':
            gxx = '/usr/bin/g++' if os.path.exists('/usr/bin/g++') else 'g++'
            cmd = [gxx, '-O3', '-fPIC', '-Wall', '-Wextra', '-std=c++17', f'-I{INCLUDE}', f'-I{CSRC}', '-c', str(src),
                   '-o', str(obj)]
        else:
            cmd = [_gcc(), '-O3', '-fPIC', '-fopenmp', '-Wall', '-Wextra', '-Wno-format-truncation', '-std=c11', f'-I{INCLUDE}',
                   f'-I{CSRC}', '-c', str(src), '-o', str(obj)]
        jobs.append(cmd)
    logs = []
    if jobs:
        with concurrent.futures.ThreadPoolExecutor(max_workers=min(8, len(jobs))) as ex:
            logs = list(ex.map(_run, jobs))
    if jobs or not LIB.exists():
        tmp = LIB.with_suffix('.so.tmp')
        _run([nvcc, *ARCH, '-shared', '-ccbin', _gcc(), '-o', str(tmp), *map(str, objs),
              '-Xcompiler', '-fopenmp', '-lgomp', '-lm'])
        os.replace(tmp, LIB)
    return LIB, '\n'.join(logs)


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument('--verbose-ptxas', action='store_true')
    ap.add_argument('--force', action='store_true')
    args = ap.parse_args(argv)
    lib, log = build(args.verbose_ptxas, args.force)
    if log.strip():
        print(log)
    print(lib)


if __name__ == '__main__':
    sys.exit(main())
