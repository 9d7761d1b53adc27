"""The C restatement of the oracle (oracle/c/qv_oracle.c, timed as the CPU
baseline) against the golden vectors made by the reference's own
cpu_reference.py and against the numpy oracle.  CPU only."""
from pathlib import Path

import numpy as np
import pytest

import oracle
from oracle import inputs as I
from oracle import native
from tests.test_oracle import ATTENTION_CASES, DELTA_CASES

GOLDEN = Path(__file__).resolve().parent / 'golden'


@pytest.fixture(scope='module', autouse=True)
def built():
    native.build()


@pytest.mark.parametrize('name', sorted(ATTENTION_CASES))
@pytest.mark.parametrize('threads', [1, 5])
def test_c_attention_matches_reference_golden(name, threads):
    g = np.load(GOLDEN / f'{name}.npz')
    case = ATTENTION_CASES[name]()
    out, kc, vc = native.attention(**case, threads=threads)
    pos = case['position']
    np.testing.assert_allclose(out, g['out'], rtol=0, atol=1e-12)
    assert np.array_equal(kc[pos:].reshape(-1).astype(np.float64), g['new_k'])
    assert np.array_equal(vc[pos:].reshape(-1).astype(np.float64), g['new_v'])


@pytest.mark.parametrize('name', sorted(DELTA_CASES))
def test_c_delta_matches_reference_golden(name):
    g = np.load(GOLDEN / f'{name}.npz')
    case = DELTA_CASES[name]()
    out, state, hist = native.delta(**case, threads=4)
    state = state.reshape(case['value_heads'], case['dim'], case['dim'])
    if 'state_heads' in g:
        state = state[g['state_heads']]
    np.testing.assert_allclose(out, g['out'], rtol=0, atol=1e-12)
    np.testing.assert_allclose(state, g['state'], rtol=0, atol=1e-12)
    np.testing.assert_array_equal(hist, g['history'])


@pytest.mark.parametrize('position,batch', [(0, 8), (2047, 8), (2048, 1), (5000, 3), (9000, 40)])
def test_c_attention_matches_numpy_oracle_across_key_blocks(position, batch):
    """Key blocks of 2048 merged by log-sum-exp == the one-pass softmax (prefill blocks too)."""
    case = I.attention_layer(batch=batch, position=position, seed=6000 + position)
    exp_out, exp_k, exp_v = oracle.attention(**case)
    out, kc, vc = native.attention(**case, threads=3)
    np.testing.assert_allclose(out, exp_out, rtol=0, atol=1e-12)
    # the appended keys may differ from numpy's in the last fp16 bit where numpy's pairwise sum
    # and the reference's sequential sum round a tie differently; the values are exact
    assert np.abs(kc[position:].astype(np.float64) - exp_k[position:].astype(np.float64)).max() <= 2 ** -10
    assert np.array_equal(vc[position:], exp_v[position:])


def test_c_delta_matches_numpy_oracle_long_block():
    case = I.delta_layer(batch=40, seed=6100, key_heads=4, value_heads=12, dim=128, state_std=0.05)
    exp_out, exp_state, exp_hist = oracle.delta(**case)
    out, state, hist = native.delta(**case, threads=6)
    np.testing.assert_allclose(out, exp_out, rtol=0, atol=1e-12)
    np.testing.assert_allclose(state, exp_state, rtol=0, atol=1e-12)
    np.testing.assert_array_equal(hist, exp_hist)


def test_c_half_rounding_matches_numpy():
    """The C port's float64 -> fp16 rounding (ties to even, subnormals, overflow) on the appended
    values equals numpy's cast on a sweep of awkward magnitudes."""
    rng = np.random.default_rng(3)
    vals = np.concatenate([rng.standard_normal(700) * 10.0 ** rng.integers(-9, 6, 700),
                           [65504, 65519.99, 65520, -65520, 6.1e-5, 5.96e-8, 2.98e-8, 2.99e-8, 0.0, -0.0]])
    vals = np.pad(vals, (0, 1024 - len(vals))).astype(np.float32)     # one cache row: 4 heads x 256
    case = I.attention_layer(batch=1, position=0, seed=1)
    case['value'] = vals.reshape(1, 4, 256)
    _, _, vc = native.attention(**case, threads=1)
    with np.errstate(over='ignore'):                                 # 65520 rounds to infinity
        expected = vals.astype(np.float16)
    assert np.array_equal(vc[0].reshape(-1).view(np.uint16), expected.view(np.uint16))
