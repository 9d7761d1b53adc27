"""Quantized projections (qv_test_mm, qv_test_mm_fast): the reference's
tests/test_cuda.py:88-145 restated.  CPU tests pin the oracle's block decoding
to the reference's own decoder (golden vectors) and its fast-path arithmetic to
the reference test's error bound; GPU tests compare the CUDA kernels with the
oracle at the reference test's shapes and tolerances."""
import ctypes as ct
import math
from pathlib import Path

import numpy as np
import pytest

from oracle import projection as P

GOLDEN = Path(__file__).resolve().parent / 'golden'
FP16 = {8: [(0, 0.0078125)], 12: [(0, 0.03125), (2, 0.015625)], 14: [(208, 0.00390625)]}


def golden_cases():
    return sorted(GOLDEN.glob('projection_*.npz'))


def make_weights(kind, width, rows, seed):
    """Seeded random blocks with the reference test's fixed fp16 scales (so
    every weight is finite); quants, packed scales and mins are random bytes."""
    cols, nbytes = P.BLOCK[kind]
    rng = np.random.default_rng(seed)
    b = rng.integers(0, 256, size=(rows * (width // cols), nbytes), dtype=np.uint8)
    for off, value in FP16[kind]:
        b[:, off:off + 2] = np.frombuffer(np.float16(value).tobytes(), np.uint8)
    return b.tobytes()


def activations(batch, width, outliers=False):
    x = np.array([math.sin(i * .07) * .13 for i in range(batch * width)], np.float32)
    if outliers:                   # a zero block and an outlier (tests/test_cuda.py:107-122)
        x[:32] = 0.
        if width > 32:
            x[37] = -3.25
    return x


@pytest.mark.parametrize('path', golden_cases(), ids=lambda p: p.stem)
def test_decode_matches_reference_decoder(path):
    z = np.load(path)
    w, _ = P.decode(int(z['kind']), z['data'].tobytes(), int(z['width']), int(z['rows']))
    np.testing.assert_array_equal(w, z['weights'])


@pytest.mark.parametrize('kind', [8, 12, 14])
def test_fast_oracle_within_the_quantisation_bound(kind):
    width, rows, batch = 512, 9, 3
    data = make_weights(kind, width, rows, 5)
    x = activations(batch, width, outliers=True)
    w, off = P.decode(kind, data, width, rows)
    fast = P.mm_fast(kind, data, x, batch, width, rows)
    exact = P.mm(kind, data, x, batch, width, rows)
    qx = P.quantize_activations(x, batch, width)
    bound = np.abs(qx - x.astype(np.float64).reshape(batch, width)) @ np.abs(w + off).T
    assert (np.abs(fast - exact) <= bound + 1e-12).all()


def _run(lib, fn, data, x, kind, batch, width, rows):
    out = np.zeros(batch * rows, np.float32)
    buf = ct.create_string_buffer(data, len(data))
    rc = fn(out.ctypes.data_as(ct.c_void_p), buf, x.ctypes.data_as(ct.c_void_p), kind, batch, width, rows)
    assert rc == 0, lib.qv_error()
    return out.astype(np.float64).reshape(batch, rows)


def _close(actual, expected, tol):
    assert np.isfinite(actual).all()
    bad = np.abs(actual - expected) > tol * (1 + np.abs(expected))
    assert not bad.any(), f'{bad.sum()} mismatches; max |d| {np.abs(actual - expected).max()}'


@pytest.mark.gpu
@pytest.mark.parametrize('kind', [8, 12, 14])
def test_all_formats_all_candidate_rows(lib, kind):
    z = np.load(GOLDEN / f'projection_{kind}_512x7.npz')
    data = z['data'].tobytes()
    for batch in (1, 2, 3, 4, 5, 8):
        x = activations(batch, 512)
        out = _run(lib, lib.qv_test_mm, data, x, kind, batch, 512, 7)
        exp = x.astype(np.float64).reshape(batch, 512) @ z['weights'].T      # the reference's own decode
        _close(out, exp, 2e-5)


@pytest.mark.gpu
@pytest.mark.parametrize('kind', [8, 12, 14])
def test_fast_path_matches_quantised_reference(lib, kind):
    for width in ((32, 96, 512, 768) if kind == 8 else (256, 512, 768)):
        rows = 131 if width == 512 else (35 if width == 768 else 7)
        data = make_weights(kind, width, rows, 100 + width)
        w, off = P.decode(kind, data, width, rows)
        for batch in range(1, 9):
            x = activations(batch, width, outliers=True)
            out = _run(lib, lib.qv_test_mm_fast, data, x, kind, batch, width, rows)
            exp = P.mm_fast(kind, data, x, batch, width, rows)
            _close(out, exp, 3e-5)
            exact = P.mm(kind, data, x, batch, width, rows)
            qx = P.quantize_activations(x, batch, width)
            bound = np.abs(qx - x.astype(np.float64).reshape(batch, width)) @ np.abs(w + off).T
            assert (np.abs(out - exact) <= bound + 3e-5 * (1 + np.abs(exp))).all()


@pytest.mark.gpu
@pytest.mark.parametrize('kind', [8, 12, 14])
def test_model_width_and_ragged_rows(lib, kind):
    width, rows, batch = 5120, 1000, 8            # a model-width row block; rows not a multiple of 32
    data = make_weights(kind, width, rows, 7)
    x = activations(batch, width)
    # ten times the reference test's width: the FP32 accumulation error of a
    # 5120-term sum with cancellation exceeds the 2e-5 of the 512-wide case
    _close(_run(lib, lib.qv_test_mm, data, x, kind, batch, width, rows), P.mm(kind, data, x, batch, width, rows), 1e-4)


@pytest.mark.gpu
@pytest.mark.parametrize('kind', [8, 12, 14])
def test_device_entry_matches_host_entry(lib, hot, kind):
    import torch
    width, rows, batch = 768, 67, 5
    data = make_weights(kind, width, rows, 11)
    x = activations(batch, width, outliers=True)
    assert lib.qv_mm_weight_bytes(kind, width, rows) == len(data)
    w = torch.frombuffer(bytearray(data), dtype=torch.uint8).cuda()
    xd = torch.from_numpy(x).cuda()
    for fast, fn in ((False, lib.qv_test_mm), (True, lib.qv_test_mm_fast)):
        out = torch.empty((batch, rows), device='cuda')
        hot.mm(out, w, xd, kind, batch, width, rows, fast=fast)
        torch.cuda.synchronize()
        host = _run(lib, fn, data, x, kind, batch, width, rows)
        np.testing.assert_array_equal(out.cpu().numpy().astype(np.float64), host)
