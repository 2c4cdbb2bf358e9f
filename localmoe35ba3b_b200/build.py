"""Build the sm_100a CUDA library in-tree: ``localmoe35ba3b_b200/liblocalmoe_b200.so``.

    python -m localmoe35ba3b_b200.build [--force] [--jobs N]

Each ``csrc/*.cu`` is compiled by nvcc to ``_build/<name>.o`` (re-used while
newer than its sources), then linked into one shared library with the CUDA
runtime linked statically, so the library has no dependency on a particular
libcudart and can be loaded with ctypes next to PyTorch.
"""
import argparse
import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, 'csrc')
BUILD = os.path.join(ROOT, '_build')
LIB = os.path.join(PKG, 'liblocalmoe_b200.so')
ARCH = ['-gencode', 'arch=compute_100a,code=sm_100a']
FLAGS = ['-O3', '-lineinfo', '-std=c++17', '-Xcompiler', '-fPIC', '-Xcompiler', '-fvisibility=hidden',
         '--expt-relaxed-constexpr']


def nvcc():
    for cand in (os.environ.get('NVCC'), shutil.which('nvcc'), '/usr/local/cuda/bin/nvcc'):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError('nvcc not found: the CUDA toolkit is required to build localmoe35ba3b_b200')


def _headers():
    return glob.glob(os.path.join(CSRC, '*.cuh')) + glob.glob(os.path.join(ROOT, 'include', '*.h'))


def _stale(obj, deps):
    if not os.path.exists(obj):
        return True
    t = os.path.getmtime(obj)
    return any(os.path.getmtime(d) > t for d in deps)


def _compile(src, force, verbose):
    obj = os.path.join(BUILD, os.path.basename(src)[:-3] + '.o')
    if not force and not _stale(obj, [src] + _headers()):
        return obj, None
    cmd = [nvcc()] + ARCH + FLAGS + ['-c', src, '-o', obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode:
        raise RuntimeError(f'nvcc failed for {src}:\n{r.stdout}\n{r.stderr}')
    return obj, (r.stderr if verbose else None)


def build(force=False, jobs=None, verbose=False):
    os.makedirs(BUILD, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, '*.cu')))
    with cf.ThreadPoolExecutor(jobs or min(8, os.cpu_count() or 1)) as ex:
        results = list(ex.map(lambda s: _compile(s, force, verbose), srcs))
    objs = [o for o, _ in results]
    for _, log in results:
        if log:
            print(log, file=sys.stderr)
    if force or _stale(LIB, objs):
        tmp = LIB + '.tmp'
        cmd = [nvcc()] + ARCH + ['-shared', '-cudart', 'static', '-Xcompiler', '-fPIC', '-o', tmp] + objs
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode:
            raise RuntimeError(f'link failed:\n{r.stdout}\n{r.stderr}')
        os.replace(tmp, LIB)
    return LIB


if __name__ == '__main__':
    ap = argparse.ArgumentParser()
    ap.add_argument('--force', action='store_true')
    ap.add_argument('--jobs', type=int, default=None)
    ap.add_argument('--verbose', action='store_true')
    a = ap.parse_args()
    print(build(a.force, a.jobs, a.verbose))
