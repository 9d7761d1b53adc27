"""The CPU oracle against the reference's own outputs (golden vectors) and
against the reference's closed-form known-answer test.  CPU only."""
from pathlib import Path

import numpy as np
import pytest

import oracle
from oracle import closed_form as CF
from oracle import inputs as I

GOLDEN = Path(__file__).resolve().parent / 'golden'

ATTENTION_CASES = {
    'attention_wave': lambda: I.attention_wave(),
    'attention_cfg0': lambda: I.attention_layer(batch=8, position=128),
    'attention_edge': lambda: I.attention_layer(batch=8, position=250, seed=1100),
    'attention_single': lambda: I.attention_layer(batch=1, position=0, seed=1101),
}
DELTA_CASES = {
    'delta_wave_d32': lambda: I.delta_wave(32),
    'delta_wave_d128': lambda: I.delta_wave(128),
    'delta_cfg1': lambda: I.delta_layer(batch=8),
    'delta_small_t1': lambda: I.delta_layer(batch=1, seed=1102, key_heads=4, value_heads=12, dim=128,
                                            state_std=0.05),
}


@pytest.mark.parametrize('name', sorted(ATTENTION_CASES))
def test_attention_oracle_matches_reference_golden(name):
    g = np.load(GOLDEN / f'{name}.npz')
    case = ATTENTION_CASES[name]()
    digest = I.checksum([case[k] for k in ('key_cache', 'value_cache', 'q_gate', 'key', 'value',
                                           'q_norm', 'k_norm')])
    assert digest == str(g['digest']), 'input generator drifted from the one that made the fixture'
    out, kc, vc = oracle.attention(**case)
    pos = case['position']
    np.testing.assert_allclose(out, g['out'], rtol=0, atol=1e-12)
    assert np.array_equal(kc[pos:].reshape(-1).astype(np.float64), g['new_k'])
    assert np.array_equal(vc[pos:].reshape(-1).astype(np.float64), g['new_v'])


@pytest.mark.parametrize('name', sorted(DELTA_CASES))
def test_delta_oracle_matches_reference_golden(name):
    g = np.load(GOLDEN / f'{name}.npz')
    case = DELTA_CASES[name]()
    digest = I.checksum([case[k] for k in ('state', 'history', 'qkv', 'gate', 'alpha', 'beta', 'conv',
                                           'decay', 'bias', 'norm')])
    assert digest == str(g['digest'])
    out, state, hist = oracle.delta(**case)
    state = state.reshape(case['value_heads'], case['dim'], case['dim'])
    if 'state_heads' in g:
        state = state[g['state_heads']]
    np.testing.assert_allclose(out, g['out'], rtol=0, atol=1e-12)
    np.testing.assert_allclose(state, g['state'], rtol=0, atol=1e-12)
    np.testing.assert_array_equal(hist, g['history'])


@pytest.mark.parametrize('position,batch', [(5, 3), (2047, 3), (4100, 2)])
def test_attention_oracle_closed_form(position, batch):
    """The reference's long-context known answer (test_cuda.py:237-273)."""
    out, kc, vc = oracle.attention(**CF.inputs(position, batch))
    np.testing.assert_allclose(out, CF.expected(position, batch), rtol=0, atol=1e-12)


def test_delta_core_is_the_inner_recurrence():
    """delta() == conv/prep + delta_core + gated norm on the same inputs."""
    c = I.delta_layer(batch=5, seed=7, key_heads=2, value_heads=6, dim=32, state_std=0.1)
    out, state, _ = oracle.delta(**c)
    hk, hv, d = 2, 6, 32
    filt = oracle.silu(c['qkv'].astype(np.float64))           # conv taps [0,0,0,1], zero history
    q, k, g, b = oracle.hotpath.prepare_delta_inputs(filt[:, :hk * d].reshape(5, hk, d),
                                                     filt[:, hk * d:2 * hk * d].reshape(5, hk, d),
                                                     c['alpha'], c['beta'])
    core, s2 = oracle.delta_core(c['state'], q, k, filt[:, 2 * hk * d:].reshape(5, hv, d), g, b)
    np.testing.assert_allclose(s2.reshape(-1), state, rtol=0, atol=1e-12)
    scale = 1 / np.sqrt((core ** 2).mean(-1, keepdims=True) + 1e-6)
    gated = core * scale * oracle.silu(c['gate'].astype(np.float64))
    np.testing.assert_allclose(gated.reshape(-1), out, rtol=0, atol=1e-12)


def test_prefill_core_rows_subset_and_scalar():
    q, k, v = (a[:40] for a in I.prefill_attention(length=40, seed=5))
    full, lse = oracle.prefill_attention_core(q, k, v)
    part, plse = oracle.prefill_attention_core(q, k, v, rows=[3, 39], heads=[0, 23])
    np.testing.assert_allclose(part, full[[3, 39]][:, [0, 23]], atol=1e-13)
    np.testing.assert_allclose(plse, lse[[3, 39]][:, [0, 23]], atol=1e-13)
    # scalar restatement of one row: head 13 (KV head 2) at position 17
    qs = q[17, 13].astype(np.float64)
    s = np.array([qs @ k[p, 2].astype(np.float64) / 16 for p in range(18)])
    w = np.exp(s - s.max())
    ref = (w[:, None] * v[:18, 2].astype(np.float64)).sum(0) / w.sum()
    np.testing.assert_allclose(full[17, 13], ref, atol=1e-13)
