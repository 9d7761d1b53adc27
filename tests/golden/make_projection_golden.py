"""Golden vectors for the quantized-projection oracle, made by the reference's
own independent decoder.

Run in a container where cristianku/redshift is checked out (by default as
``reference/`` beside this repository's checkout; override with
``REDSHIFT_REFERENCE``)::

    python tests/golden/make_projection_golden.py

It imports the reference's ``tests/test_cuda.py`` unchanged and calls its
``quantized(kind, width, rows)`` helper, which builds the packed block bytes
of a seeded weight matrix and decodes them element by element in Python.
The bytes and the decoded weights are stored as ``projection_<kind>_<width>
x<rows>.npz`` next to this script; ``tests/test_projection.py`` checks
``oracle.projection.decode`` against them.  Nothing on the GPU box reads the
reference checkout.
"""
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
CASES = [(8, 512, 7), (8, 96, 7), (12, 512, 7), (12, 768, 3), (14, 512, 7), (14, 768, 3)]


def reference_test_module():
    root = Path(os.environ.get('REDSHIFT_REFERENCE', HERE.parents[2] / 'reference'))
    sys.path.insert(0, str(root))
    sys.path.insert(0, str(root / 'tests'))
    import test_cuda  # noqa: E402  (the reference's own test module, unchanged)
    return test_cuda


def main():
    ref = reference_test_module()
    for kind, width, rows in CASES:
        data, weights = ref.quantized(kind, width, rows)
        np.savez_compressed(HERE / f'projection_{kind}_{width}x{rows}.npz',
                            data=np.frombuffer(data, np.uint8), weights=np.array(weights, np.float64),
                            kind=kind, width=width, rows=rows)
        print(f'kind {kind} {width}x{rows}: {len(data)} bytes')


if __name__ == '__main__':
    main()
