"""Build the sm_100a shared library ``slimkv_b200/libslimkv_b200.so`` in-tree.

Every ``csrc/*.cu`` / ``csrc/*.cpp`` file is compiled with nvcc for
``sm_100a`` (``-gencode arch=compute_100a,code=sm_100a``) and linked into one
C-ABI shared library with the CUDA runtime linked statically, so the library
has no dependency on a Python-side CUDA runtime.  Objects are cached under
``slimkv_b200/_build`` and rebuilt when a source or header changes.
"""
import hashlib
import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / 'csrc'
BUILD = PKG / '_build'
LIB = PKG / 'libslimkv_b200.so'
NVCC = os.environ.get('NVCC', '/usr/local/cuda/bin/nvcc')
ARCH = ['-gencode', 'arch=compute_100a,code=sm_100a']
FLAGS = ['-O3', '-std=c++17', '-lineinfo', '-Xcompiler', '-fPIC', '-Xcompiler', '-fvisibility=hidden',
         f'-I{ROOT / "include"}', f'-I{CSRC}', '--expt-relaxed-constexpr']


def _headers_digest():
    h = hashlib.sha256()
    for p in sorted(list(CSRC.glob('*.cuh')) + list(CSRC.glob('*.h')) + list((ROOT / 'include').glob('*.h'))):
        h.update(p.read_bytes())
    return h.hexdigest()[:16]


def _compile(src, digest, verbose):
    obj = BUILD / (src.stem + ('_cu' if src.suffix == '.cu' else '_cc') + '.o')
    stamp = obj.with_suffix('.stamp')
    key = hashlib.sha256(src.read_bytes() + digest.encode() + ' '.join(FLAGS).encode()).hexdigest()
    if obj.exists() and stamp.exists() and stamp.read_text() == key:
        return obj
    cmd = [NVCC, *ARCH, *FLAGS, '-c', str(src), '-o', str(obj)]
    if verbose and src.suffix == '.cu':
        cmd += ['-Xptxas', '-v']
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode:
        raise RuntimeError(f'nvcc failed for {src.name}:\n{r.stderr}')
    if verbose and r.stderr:
        print(r.stderr, file=sys.stderr)
    stamp.write_text(key)
    return obj


def build(verbose=False):
    """Compile and link the library; returns its path."""
    BUILD.mkdir(exist_ok=True)
    digest = _headers_digest()
    sources = sorted(CSRC.glob('*.cu')) + sorted(CSRC.glob('*.cpp'))
    with ThreadPoolExecutor(max_workers=min(8, len(sources))) as pool:
        objs = list(pool.map(lambda s: _compile(s, digest, verbose), sources))
    newest = max(o.stat().st_mtime for o in objs)
    if not LIB.exists() or LIB.stat().st_mtime < newest:
        cmd = [NVCC, *ARCH, '-shared', '-o', str(LIB), *map(str, objs), '-cudart', 'static']
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode:
            raise RuntimeError(f'link failed:\n{r.stderr}')
    return LIB


if __name__ == '__main__':
    print(build(verbose='-v' in sys.argv))
