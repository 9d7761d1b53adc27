"""qv_attention_noalloc: the attention layer for callers that cannot allocate.

A runtime that has handed all of HBM to its own pools, or a plugin host that
owns every allocation, cannot give the library a workspace.  The no-allocation
entry point keeps its scratch in a fixed array that the library places in
device memory.  This file checks, through the C ABI, that two calls in a row
(the second on a shorter context, so it runs on the first call's leftover
scratch contents) give the same output and the same appended cache rows as
qv_attention with a caller-provided workspace.

The file name makes pytest collect it last.
"""
import ctypes as ct

import numpy as np
import pytest

import oracle
from oracle import inputs as I

pytestmark = pytest.mark.gpu


def _run_pair(lib, case):
    """(noalloc out, new rows) and (qv_attention out, new rows) for one case."""
    import torch
    dev = torch.device('cuda')
    batch, position = case['batch'], case['position']
    t = lambda k: torch.from_numpy(np.ascontiguousarray(np.asarray(case[k], np.float32))).to(dev)  # noqa: E731
    args = [t(k) for k in ('q_gate', 'key', 'value', 'q_norm', 'k_norm')]
    ptrs = [ct.c_void_p(a.data_ptr()) for a in args]
    stream = ct.c_void_p(torch.cuda.current_stream().cuda_stream)
    results = []
    for use_noalloc in (True, False):
        kc = torch.from_numpy(case['key_cache']).to(dev)
        vc = torch.from_numpy(case['value_cache']).to(dev)
        out = torch.full((batch, 24, 256), float('nan'), device=dev)
        if use_noalloc:
            rc = lib.qv_attention_noalloc(ct.c_void_p(out.data_ptr()), ct.c_void_p(kc.data_ptr()),
                                          ct.c_void_p(vc.data_ptr()), *ptrs, batch, position, 1e-6, stream)
        else:
            ws = torch.zeros(lib.qv_attention_workspace(batch, position), dtype=torch.uint8, device=dev)
            rc = lib.qv_attention(ct.c_void_p(out.data_ptr()), ct.c_void_p(kc.data_ptr()),
                                  ct.c_void_p(vc.data_ptr()), *ptrs, batch, position, 1e-6,
                                  ct.c_void_p(ws.data_ptr()), ws.numel(), stream)
        assert rc == 0, lib.qv_error()
        torch.cuda.synchronize()
        assert lib.qv_status() == 0
        results.append((out.cpu().numpy(), kc[position:].cpu().numpy(), vc[position:].cpu().numpy()))
    return results


def test_no_alloc_matches_the_workspace_entry_point_twice_in_a_row(lib):
    cases = [I.attention_layer(batch=8, position=40000, seed=5100),   # many splits
             I.attention_layer(batch=3, position=700, seed=5101)]     # fewer splits, stale scratch beyond
    for case in cases:
        (out_a, k_a, v_a), (out_b, k_b, v_b) = _run_pair(lib, case)
        assert np.isfinite(out_a).all()
        bad = np.abs(out_a - out_b) > 3e-4 * (1 + np.abs(out_b))
        assert not bad.any()
        assert np.array_equal(k_a, k_b) and np.array_equal(v_a, v_b)
        # and both against the CPU oracle (max-abs <= 2e-3)
        expected, _, _ = oracle.attention(**case)
        assert np.abs(out_a.reshape(-1) - expected).max() <= 2e-3


def test_no_alloc_rejects_batches_beyond_the_fixed_scratch(lib):
    v = ct.c_void_p(8)   # never dereferenced: the arguments are rejected first
    assert lib.qv_attention_noalloc(v, v, v, v, v, v, v, v, 9, 100, 1e-6, None) == -1
    assert b'batch must be between 1 and 8' in lib.qv_error()
    assert lib.qv_attention_noalloc(v, v, v, v, v, v, v, v, 8, 139257, 1e-6, None) == -1
