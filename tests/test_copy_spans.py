"""Checkpoint / restore of layer state in one launch (qv_copy_spans), the
layer-level equivalent of the reference's Model::copy_state
(src/runtime.cu:455-485): every attention layer's valid KV prefix and every
DeltaNet state and history, copied as one span list."""
import ctypes as ct

import numpy as np
import pytest


def _table(spans):
    n = len(spans)
    dst = (ct.c_void_p * n)(*[d for d, _, _ in spans])
    src = (ct.c_void_p * n)(*[s for _, s, _ in spans])
    nb = (ct.c_size_t * n)(*[b for _, _, b in spans])
    return dst, src, nb, n


def test_rejects_bad_tables_before_reading(lib):
    v = 16
    dst, src, nb, n = _table([(v, v, 64)])
    assert lib.qv_copy_spans(dst, src, nb, 0, None) == -1
    assert lib.qv_copy_spans(dst, src, nb, 161, None) == -1
    assert b'1..160' in lib.qv_error()
    assert lib.qv_copy_spans(None, src, nb, 1, None) == -1
    dst0, src0, nb0, _ = _table([(0, v, 64)])
    assert lib.qv_copy_spans(dst0, src0, nb0, 1, None) == -1
    assert b'null span address' in lib.qv_error()


@pytest.mark.gpu
def test_checkpoint_and_restore_round_trip(lib):
    import torch
    dev = torch.device('cuda')
    g = torch.Generator(device=dev)
    g.manual_seed(5)
    prefix = 1000
    # 2 attention layers (K and V caches with capacity beyond the prefix) and
    # 6 DeltaNet layers (state, history), as in the model's layer pattern
    kv = [torch.randn((prefix + 64, 4, 256), generator=g, device=dev).half() for _ in range(4)]
    states = [torch.randn((48, 128, 128), generator=g, device=dev) for _ in range(6)]
    hists = [torch.randn((3, 10240), generator=g, device=dev) for _ in range(6)]
    live = kv + states + hists
    sizes = [prefix * 2048] * 4 + [s.numel() * 4 for s in states] + [h.numel() * 4 for h in hists]
    snap = [torch.empty(sz, dtype=torch.uint8, device=dev) for sz in sizes]
    orig = [t.clone() for t in live]
    dst, src, nb, n = _table([(s.data_ptr(), t.data_ptr(), sz) for s, t, sz in zip(snap, live, sizes)])
    assert lib.qv_copy_spans(dst, src, nb, n, None) == 0, lib.qv_error()
    torch.cuda.synchronize()
    for s, t, sz in zip(snap, orig, sizes):
        assert torch.equal(s, t.view(torch.uint8).reshape(-1)[:sz])
    for t in live:                                   # the layers move on
        t.add_(1)
    dst, src, nb, n = _table([(t.data_ptr(), s.data_ptr(), sz) for s, t, sz in zip(snap, live, sizes)])
    assert lib.qv_copy_spans(dst, src, nb, n, None) == 0, lib.qv_error()
    torch.cuda.synchronize()
    for t, o, sz in zip(live, orig, sizes):          # restored prefix / state; the rest untouched
        assert torch.equal(t.view(torch.uint8).reshape(-1)[:sz], o.view(torch.uint8).reshape(-1)[:sz])
    assert torch.equal(kv[0][prefix:], (orig[0][prefix:].float() + 1).half())


@pytest.mark.gpu
def test_unaligned_and_odd_spans(lib):
    import torch
    dev = torch.device('cuda')
    src = torch.randint(0, 256, (1 << 20,), dtype=torch.uint8, device=dev)
    dst = torch.zeros_like(src)
    spans, off = [], 0
    for k, (so, nbytes) in enumerate([(0, 16), (1, 15), (3, 1000), (16, 4096), (5, 1), (32, 65536), (7, 77777)]):
        spans.append((dst.data_ptr() + off, src.data_ptr() + so + off, nbytes))
        off += nbytes + 64
    spans.append((dst.data_ptr() + off, src.data_ptr() + off, 0))      # an empty span
    t = _table(spans)
    assert lib.qv_copy_spans(*t, None) == 0, lib.qv_error()
    torch.cuda.synchronize()
    s, d = src.cpu().numpy(), dst.cpu().numpy()
    expect = np.zeros_like(s)
    off = 0
    for so, nbytes in [(0, 16), (1, 15), (3, 1000), (16, 4096), (5, 1), (32, 65536), (7, 77777)]:
        expect[off:off + nbytes] = s[off + so:off + so + nbytes]
        off += nbytes + 64
    np.testing.assert_array_equal(d, expect)
