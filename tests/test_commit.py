"""Verify/commit transaction of a DeltaNet layer (qv_delta_verify,
qv_delta_commit): the state side of the reference's qv_verify / qv_commit
(src/runtime.cu:363-374, 389-395, 432-454; src/kernels.cu:356-369, 567-574).

CPU tests pin the oracle's commit restatement (replaying the trace of the
first `accepted` tokens equals running the layer on those tokens) and the
entry points' argument checks; GPU tests compare the CUDA path with qv_delta
and with the oracle."""
import ctypes as ct

import numpy as np
import pytest

import oracle
from oracle import inputs as I


def _case(dim, batch=5):
    """The reference's DeltaNet wave case (non-zero history and conv taps, so
    the committed history window and the replayed state both matter)."""
    return I.delta_wave(dim, batch=batch)


@pytest.mark.parametrize('dim,batch', [(32, 5), (128, 5), (32, 8), (128, 1)])
def test_oracle_commit_replays_the_accepted_prefix(dim, batch):
    c = _case(dim, batch)
    hk, hv, batch = c['key_heads'], c['value_heads'], c['batch']
    C = (2 * hk + hv) * dim
    trace = oracle.delta_trace(c['history'], c['qkv'], c['alpha'], c['beta'], c['conv'], c['decay'], c['bias'],
                               batch, hk, hv, dim)
    assert trace.size == 8 * (2 * C + 2 * hv)
    for accepted in range(batch + 1):
        st, hist = oracle.delta_commit(c['state'], c['history'], trace, accepted, hk, hv, dim)
        if accepted == 0:
            np.testing.assert_array_equal(st, np.asarray(c['state'], np.float64).reshape(-1))
            np.testing.assert_array_equal(hist, np.asarray(c['history'], np.float64).reshape(-1))
            continue
        sub = dict(c, batch=accepted,
                   qkv=np.asarray(c['qkv']).reshape(batch, -1)[:accepted],
                   gate=np.asarray(c['gate']).reshape(batch, -1)[:accepted],
                   alpha=np.asarray(c['alpha']).reshape(batch, -1)[:accepted],
                   beta=np.asarray(c['beta']).reshape(batch, -1)[:accepted])
        _, exp_st, exp_hist = oracle.delta(**sub)
        np.testing.assert_allclose(st, exp_st, rtol=0, atol=1e-12)
        np.testing.assert_allclose(hist, exp_hist, rtol=0, atol=0)


def test_verify_and_commit_reject_bad_arguments(lib):
    v = ct.c_void_p(16)               # never dereferenced: validation comes first
    assert lib.qv_delta_trace_floats(16, 48, 128) == 8 * (2 * (2 * 16 + 48) * 128 + 2 * 48)
    assert lib.qv_delta_trace_floats(16, 48, 64) == 0
    assert lib.qv_delta_trace_floats(5, 48, 128) == 0
    args = [v] * 11
    assert lib.qv_delta_verify(*args, 9, 16, 48, 128, 1e-6, v, v, v, None) == -1       # batch > 8
    assert lib.qv_delta_verify(*args, 0, 16, 48, 128, 1e-6, v, v, v, None) == -1
    assert lib.qv_delta_verify(*args, 8, 16, 48, 128, 1e-6, v, v, None, None) == -1    # no trace
    assert lib.qv_delta_verify(*args, 8, 16, 48, 64, 1e-6, v, v, v, None) == -1        # dim
    assert lib.qv_delta_commit(v, v, v, v, v, 9, 8, 16, 48, 128, None) == -1           # accepted > batch
    assert lib.qv_delta_commit(v, v, v, v, v, -1, 8, 16, 48, 128, None) == -1
    assert lib.qv_delta_commit(v, v, v, v, None, 2, 8, 16, 48, 128, None) == -1
    assert lib.qv_delta_commit(v, v, v, v, v, 2, 4, 16, 48, 64, None) == -1           # dim


@pytest.mark.gpu
@pytest.mark.parametrize('dim,batch', [(32, 5), (128, 5), (128, 1), (128, 8)])
def test_verify_records_and_commit_rebuilds(hot, dim, batch):
    import torch
    dev = torch.device('cuda')
    c = _case(dim, batch)
    hk, hv, batch = c['key_heads'], c['value_heads'], c['batch']
    C = (2 * hk + hv) * dim
    t = lambda k: torch.from_numpy(np.ascontiguousarray(np.asarray(c[k], np.float32).reshape(-1))).to(dev)  # noqa: E731
    ins = {k: t(k) for k in ('qkv', 'gate', 'alpha', 'beta', 'conv', 'decay', 'bias', 'norm')}
    start_state, start_hist = t('state'), t('history')
    args = lambda: (ins['qkv'], ins['gate'], ins['alpha'], ins['beta'], ins['conv'], ins['decay'],  # noqa: E731
                    ins['bias'], ins['norm'], batch, hk, hv, dim)
    # plain layer call for reference
    out_p, st_p, hi_p = torch.empty(batch * hv * dim, device=dev), start_state.clone(), start_hist.clone()
    hot.delta(out_p, st_p, hi_p, *args())
    # recorded verify
    out_v, st_v, hi_v = torch.empty_like(out_p), start_state.clone(), start_hist.clone()
    saved_s, saved_h = torch.full_like(st_v, float('nan')), torch.full_like(hi_v, float('nan'))
    trace = torch.zeros(int(hot.lib.qv_delta_trace_floats(hk, hv, dim)), device=dev)
    hot.delta_verify(out_v, st_v, hi_v, *args(), saved_s, saved_h, trace)
    torch.cuda.synchronize()
    assert hot.status() == 0
    # the recording changes nothing in the layer's results
    assert torch.equal(out_v, out_p) and torch.equal(st_v, st_p) and torch.equal(hi_v, hi_p)
    assert torch.equal(saved_s, start_state) and torch.equal(saved_h, start_hist)
    exp_trace = oracle.delta_trace(c['history'], c['qkv'], c['alpha'], c['beta'], c['conv'], c['decay'],
                                   c['bias'], batch, hk, hv, dim)
    got = trace.cpu().numpy().astype(np.float64)
    np.testing.assert_array_equal(got[:batch * C], exp_trace[:batch * C])          # raw rows, exact
    bad = np.abs(got - exp_trace) > 3e-5 * (1 + np.abs(exp_trace))
    assert not bad.any(), f'{bad.sum()} trace mismatches, first at {np.argmax(bad)}'
    # commit each acceptance count from the verify's end state
    for accepted in sorted({0, 1, min(3, batch), batch}):
        st, hi = st_v.clone(), hi_v.clone()
        hot.delta_commit(st, hi, saved_s, saved_h, trace, accepted, batch, hk, hv, dim)
        torch.cuda.synchronize()
        assert hot.status() == 0
        if accepted == batch:
            assert torch.equal(st, st_v) and torch.equal(hi, hi_v)
            continue
        exp_st, exp_hi = oracle.delta_commit(c['state'], c['history'], exp_trace, accepted, hk, hv, dim)
        for a_, e_ in ((st.cpu().numpy(), exp_st), (hi.cpu().numpy(), exp_hi)):
            a_ = a_.astype(np.float64).reshape(-1)
            bad = np.abs(a_ - e_) > 3e-5 * (1 + np.abs(e_))
            assert not bad.any(), f'accepted {accepted}: {bad.sum()} mismatches'
