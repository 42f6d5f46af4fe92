"""Build libferryb.so (sm_100a) in-tree: python -m ferry_b200.build"""
import os
import subprocess
from pathlib import Path

CSRC = Path(__file__).resolve().parent / 'csrc'


def build(jobs=None, verbose=False):
    jobs = jobs or max(1, min(16, os.cpu_count() or 4))
    out = subprocess.run(['make', '-C', str(CSRC), f'-j{jobs}'], capture_output=not verbose, text=True)
    if out.returncode != 0:
        raise RuntimeError('libferryb build failed:\n' + (out.stdout or '') + (out.stderr or ''))
    return CSRC.parent / 'libferryb.so'


if __name__ == '__main__':
    print(build(verbose=True))
