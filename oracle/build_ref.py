"""Compile the reference's own native ops into oracle/_ref/ (test infrastructure only).

The FERRY reference builds ferry/csrc/expert_ops.{cpp,cu} with
torch.utils.cpp_extension.load at run time (ferry/runtime.py:26-31).  This
recipe compiles the same two source files, where they lie in the reference
checkout, into oracle/_ref/ferry_expert_ops*.so for sm_100a, so that the GPU
parity tests can run the reference's execute_experts / pack_dispatch /
unpack_dispatch / reduce_partials / scatter_returned / H2DEngine on a B200 as
the checker of the CUDA kernels.  The reference sources are never copied into
this repository; the built module is git-ignored and travels to the GPU box.

    python oracle/build_ref.py [--reference /path/to/FERRY]

load_ref() imports the built module (it needs torch and a CUDA device to run).
"""
import argparse
import importlib.util
import os
from pathlib import Path

HERE = Path(__file__).resolve().parent
REF_DIR = HERE / '_ref'
NAME = 'ferry_expert_ops'


def build(reference=None, verbose=False):
    reference = reference or os.environ.get('FERRY_REFERENCE')
    if not reference:
        raise ValueError('no FERRY checkout given: pass --reference or set FERRY_REFERENCE')
    src = Path(reference) / 'ferry' / 'csrc'
    if not (src / 'expert_ops.cpp').exists():
        return None
    from torch.utils.cpp_extension import load
    REF_DIR.mkdir(parents=True, exist_ok=True)
    os.environ.setdefault('MAX_JOBS', '8')
    arch = ['-gencode', 'arch=compute_100a,code=sm_100a']
    load(name=NAME, sources=[str(src / 'expert_ops.cpp'), str(src / 'expert_ops.cu')],
         extra_cflags=['-O2'], extra_cuda_cflags=['-O2'] + arch, build_directory=str(REF_DIR),
         verbose=verbose, is_python_module=True)
    return built_path()


def built_path():
    hits = sorted(REF_DIR.glob(f'{NAME}*.so'))
    return hits[0] if hits else None


def load_ref():
    """Import the prebuilt reference module, or return None when it was not built."""
    path = built_path()
    if path is None:
        return None
    import torch  # noqa: F401  (the module links against libtorch)
    spec = importlib.util.spec_from_file_location(NAME, str(path))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


if __name__ == '__main__':
    p = argparse.ArgumentParser()
    p.add_argument('--reference', default=None, help='FERRY checkout (default: $FERRY_REFERENCE)')
    a = p.parse_args()
    print(build(a.reference, verbose=True))
