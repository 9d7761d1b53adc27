"""The reference's hot-path kernel tests (tests/test_cuda.py:72-87, 150-273 of
cristianku/redshift), restated against this build through the same C ABI with
host buffers.  Expected values come from the CPU oracle (pinned to the
reference's cpu_reference.py by tests/golden) or from the closed form."""
import ctypes as ct
import math

import numpy as np
import pytest

import oracle
from oracle import closed_form as CF
from oracle import inputs as I

pytestmark = pytest.mark.gpu


def ptr(a):
    return a.ctypes.data_as(ct.c_void_p)


def close(actual, expected, tol=3e-5):
    """The reference's criterion |a-e| <= tol*(1+|e|) (test_cuda.py:66-70)."""
    actual = np.asarray(actual, np.float64).reshape(-1)
    expected = np.asarray(expected, np.float64).reshape(-1)
    assert actual.shape == expected.shape
    assert np.isfinite(actual).all()
    bad = np.abs(actual - expected) > tol * (1 + np.abs(expected))
    assert not bad.any(), (f'{bad.sum()} mismatches, first at {np.argmax(bad)}: '
                           f'{actual[np.argmax(bad)]} vs {expected[np.argmax(bad)]}')


def run_delta(lib, c, batch=None, state=None, history=None, rows=None):
    batch = c['batch'] if batch is None else batch
    out = np.zeros(batch * c['value_heads'] * c['dim'], np.float32)
    st = np.array(c['state'] if state is None else state, np.float32).copy()
    hi = np.array(c['history'] if history is None else history, np.float32).copy()
    f = lambda k: np.ascontiguousarray(np.asarray(c[k], np.float32).reshape(-1))  # noqa: E731
    args = {k: f(k) for k in ('qkv', 'gate', 'alpha', 'beta', 'conv', 'decay', 'bias', 'norm')}
    if rows is not None:
        C = (2 * c['key_heads'] + c['value_heads']) * c['dim']
        hv, d = c['value_heads'], c['dim']
        t0, t1 = rows
        args['qkv'] = args['qkv'][t0 * C:t1 * C].copy()
        args['gate'] = args['gate'][t0 * hv * d:t1 * hv * d].copy()
        args['alpha'] = args['alpha'][t0 * hv:t1 * hv].copy()
        args['beta'] = args['beta'][t0 * hv:t1 * hv].copy()
    rc = lib.qv_test_delta(ptr(out), ptr(st), ptr(hi), ptr(args['qkv']), ptr(args['gate']),
                           ptr(args['alpha']), ptr(args['beta']), ptr(args['conv']), ptr(args['decay']),
                           ptr(args['bias']), ptr(args['norm']), batch, c['key_heads'], c['value_heads'],
                           c['dim'], c['epsilon'])
    assert rc == 0, lib.qv_error()
    return out, st, hi


def run_attention(lib, c, kc=None, vc=None, fn=None, batch=None, position=None, rows=None):
    batch = c['batch'] if batch is None else batch
    position = c['position'] if position is None else position
    kc = np.ascontiguousarray(c['key_cache'] if kc is None else kc)
    vc = np.ascontiguousarray(c['value_cache'] if vc is None else vc)
    q_gate = np.ascontiguousarray(np.asarray(c['q_gate'], np.float32).reshape(-1, 12288))
    key = np.ascontiguousarray(np.asarray(c['key'], np.float32).reshape(-1, 1024))
    value = np.ascontiguousarray(np.asarray(c['value'], np.float32).reshape(-1, 1024))
    if rows is not None:
        q_gate, key, value = (np.ascontiguousarray(a[rows[0]:rows[1]]) for a in (q_gate, key, value))
    qn = np.ascontiguousarray(np.asarray(c['q_norm'], np.float32))
    kn = np.ascontiguousarray(np.asarray(c['k_norm'], np.float32))
    out = np.zeros(batch * 6144, np.float32)
    fn = fn or lib.qv_test_attention
    rc = fn(ptr(out), ptr(kc), ptr(vc), ptr(q_gate), ptr(key), ptr(value), ptr(qn), ptr(kn),
            batch, position, c['epsilon'])
    assert rc == 0, lib.qv_error()
    return out, kc, vc


def test_rejection_then_success_clears_error(lib):
    value = (ct.c_float * 1)(1.)
    assert lib.qv_test_attention(*([value] * 8), 8, 139257, 1e-6) == -1
    assert lib.qv_test_norm(value, value, value, 1, 1, 1e-6) == 0, lib.qv_error()
    assert lib.qv_error() == b''


def test_weighted_rms_on_each_row(lib):
    batch, width = 3, 5120
    x = np.array([math.sin(i * .031) for i in range(batch * width)], np.float32)
    w = np.array([.8 + .2 * math.cos(i * .07) for i in range(width)], np.float32)
    out = np.zeros_like(x)
    assert lib.qv_test_norm(ptr(out), ptr(x), ptr(w), batch, width, 1e-6) == 0, lib.qv_error()
    xd = x.astype(np.float64).reshape(batch, width)
    ref = xd / np.sqrt((xd ** 2).mean(1, keepdims=True) + 1e-6) * w
    np.testing.assert_allclose(out.reshape(batch, width), ref, atol=2e-6, rtol=0)


@pytest.mark.parametrize('dim', [32, 128])
def test_delta_matches_cpu_and_sequential_nonzero_state(lib, dim):
    c = I.delta_wave(dim)
    exp_out, exp_state, exp_hist = oracle.delta(**c)
    out, st, hi = run_delta(lib, c)
    close(out, exp_out)
    close(st, exp_state)
    close(hi, exp_hist)
    # Splitting the block must carry both the conv history and the recurrent state.
    seq_s, seq_h, seq = c['state'].copy(), c['history'].copy(), []
    for t in range(c['batch']):
        o, seq_s, seq_h = run_delta(lib, c, batch=1, state=seq_s, history=seq_h, rows=(t, t + 1))
        seq.append(o)
    close(out, np.concatenate(seq))
    close(st, seq_s)
    close(hi, seq_h, 0)


def test_attention_cpu_prefix_causality_and_chunking(lib):
    c = I.attention_wave()
    position, batch = c['position'], c['batch']
    exp_out, exp_k, exp_v = oracle.attention(**c)
    out, kc, vc = run_attention(lib, c, kc=c['key_cache'].copy(), vc=c['value_cache'].copy())
    close(out, exp_out, 3e-4)
    close(kc.astype(np.float64), exp_k.astype(np.float64), 2e-3)
    close(vc.astype(np.float64), exp_v.astype(np.float64), 0)
    assert np.array_equal(kc[:position], c['key_cache'][:position])
    # Sequential single-token calls cannot see later tokens of the block.
    seq_k, seq_v = c['key_cache'].copy(), c['value_cache'].copy()
    seq = []
    for t in range(batch):
        o, seq_k, seq_v = run_attention(lib, c, kc=seq_k, vc=seq_v, batch=1, position=position + t,
                                        rows=(t, t + 1))
        seq.append(o)
    close(out, np.concatenate(seq))
    assert kc.tobytes() == seq_k.tobytes()
    assert vc.tobytes() == seq_v.tobytes()


@pytest.mark.parametrize('position,batch', [(2047, 3), (32767, 1), (139263, 1)])
def test_attention_long_context_against_closed_form(lib, position, batch):
    c = CF.inputs(position, batch)
    prefix_k, prefix_v = c['key_cache'][:position].copy(), c['value_cache'][:position].copy()
    out, kc, vc = run_attention(lib, c)
    close(out, CF.expected(position, batch), 3e-5)
    assert np.array_equal(kc[:position], prefix_k)
    assert np.array_equal(vc[:position], prefix_v)
