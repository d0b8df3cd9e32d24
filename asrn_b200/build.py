"""Build libasrn_b200.so in-tree from asrn_b200/csrc/*.cu for sm_100a (B200).

    python -m asrn_b200.build            # incremental: recompiles sources newer than their object
    python -m asrn_b200.build --force

Objects go to asrn_b200/_build/, the shared library to asrn_b200/libasrn_b200.so (both git-ignored; the .so travels
with the repository snapshot to the GPU machine). nvcc cross-compiles, so no GPU is needed to build.
"""
import concurrent.futures
import glob
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, 'csrc')
OBJ = os.path.join(HERE, '_build')
LIB = os.path.join(HERE, 'libasrn_b200.so')
ROOT = os.path.dirname(HERE)

ARCH = ['-gencode', 'arch=compute_100a,code=sm_100a']
FLAGS = ['-O3', '-std=c++17', '-lineinfo', '-Xcompiler', '-fPIC', '--expt-relaxed-constexpr',
         '-I' + os.path.join(ROOT, 'include')]


def nvcc():
    for cand in (os.environ.get('NVCC'), shutil.which('nvcc'), '/usr/local/cuda/bin/nvcc'):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError('nvcc not found: the CUDA toolkit is required to build libasrn_b200.so')


def _deps_mtime():
    files = glob.glob(os.path.join(SRC, '*.cuh')) + glob.glob(os.path.join(SRC, '*.h')) + \
        glob.glob(os.path.join(ROOT, 'include', '*.h'))
    return max((os.path.getmtime(f) for f in files), default=0)


def _compile(src, force, extra):
    obj = os.path.join(OBJ, os.path.basename(src)[:-3] + '.o')
    if not force and os.path.exists(obj) and os.path.getmtime(obj) >= max(os.path.getmtime(src), _deps_mtime()):
        return obj, None
    cmd = [nvcc(), *ARCH, *FLAGS, *extra, '-c', src, '-o', obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        return obj, f'{" ".join(cmd)}\n{r.stdout}\n{r.stderr}'
    return obj, r.stderr if '-Xptxas' in ' '.join(extra) else None


def build(force=False, verbose=False, extra=()):
    os.makedirs(OBJ, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(SRC, '*.cu')))
    objs, errors = [], []
    with concurrent.futures.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        for obj, msg in ex.map(lambda s: _compile(s, force, list(extra)), srcs):
            objs.append(obj)
            if msg and ('error' in msg.lower() and 'ptxas info' not in msg.lower() or verbose):
                errors.append(msg) if 'error' in msg.lower() else print(msg)
    if errors:
        raise RuntimeError('nvcc failed:\n' + '\n\n'.join(errors))
    if force or not os.path.exists(LIB) or any(os.path.getmtime(o) > os.path.getmtime(LIB) for o in objs):
        cmd = [nvcc(), *ARCH, '-shared', '-o', LIB, *objs, '-lcudart']
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f'link failed: {" ".join(cmd)}\n{r.stdout}\n{r.stderr}')
    return LIB


if __name__ == '__main__':
    args = sys.argv[1:]
    ptx = ['-Xptxas', '-v'] if '--ptxas' in args else []
    print(build(force='--force' in args or bool(ptx), verbose=bool(ptx), extra=ptx))
