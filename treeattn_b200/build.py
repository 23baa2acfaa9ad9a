"""Build libtreeattn_b200.so in-tree: `python -m treeattn_b200.build` (nvcc, sm_100a)."""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))


def build(verbose=True):
    csrc = os.path.join(HERE, 'csrc')
    cmd = ['make', '-C', csrc]
    r = subprocess.run(cmd, capture_output=not verbose, text=True)
    if r.returncode != 0:
        raise RuntimeError('building libtreeattn_b200.so failed:\n%s' % ((r.stdout or '') + (r.stderr or '')))
    return os.path.join(HERE, 'lib', 'libtreeattn_b200.so')


if __name__ == '__main__':
    print(build(verbose='-q' not in sys.argv))
