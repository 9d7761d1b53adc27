"""One process, two GPUs: the kernels that raise their shared-memory limit
(decode attention, causal prefill, chunked DeltaNet, quantized projection) set
it per device, so a call on device 1 after calls on device 0 runs, and gives
the same bits for the same inputs.  Skipped with fewer than two GPUs."""
import numpy as np
import pytest

from oracle import inputs as I

pytestmark = pytest.mark.gpu


def _run_on(hot, dev_index, case, pre, dc, w, x):
    import torch
    dev = torch.device('cuda', dev_index)
    out = {}
    with torch.cuda.device(dev_index):
        t = lambda a, dt=torch.float32: torch.from_numpy(np.ascontiguousarray(a)).to(dev, dt)  # noqa: E731
        # decode / verify attention (split-KV, 232 KB of shared memory per CTA)
        kc, vc = t(case['key_cache'], torch.float16), t(case['value_cache'], torch.float16)
        o = torch.empty((case['batch'], 24, 256), device=dev)
        hot.attention(o, kc, vc, t(case['q_gate']), t(case['key']), t(case['value']), t(case['q_norm']),
                      t(case['k_norm']), case['batch'], case['position'])
        out['attention'] = o
        # causal prefill core
        q, k, v = (torch.from_numpy(a.view(np.uint16).copy()).to(dev).view(torch.float16) for a in pre)
        L = q.shape[0]
        o = torch.empty((L, 24, 256), device=dev)
        hot.prefill_attention(o, q, k, v, L)
        out['prefill'] = o
        # chunked DeltaNet core
        f16 = lambda a: torch.from_numpy(a.view(np.uint16).copy()).to(dev).view(torch.float16)  # noqa: E731
        state = torch.zeros((48, 128, 128), device=dev)
        o = torch.empty((dc['q'].shape[0], 48, 128), device=dev)
        decay, bias = torch.full((48,), -1.0, device=dev), torch.zeros(48, device=dev)
        hot.delta_chunked(o, state, f16(dc['q']), f16(dc['k']), f16(dc['v']), t(dc['alpha']), t(dc['beta']),
                          decay, bias, dc['q'].shape[0], 16, 48, 128)
        out['delta_chunked'] = o
        out['delta_state'] = state
        # Q4_K projection on the tensor cores
        o = torch.empty((3, 256), device=dev)
        hot.mm(o, torch.from_numpy(w).to(dev), t(x), 12, 3, 512, 256)
        out['mm'] = o
        torch.cuda.synchronize(dev)
        assert hot.status() == 0
    return {k: v.cpu().numpy() for k, v in out.items()}


def test_kernels_on_a_second_device_in_the_same_process(hot):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip('needs two GPUs')
    case = I.attention_layer(batch=8, position=40000, seed=5200)
    pre = I.prefill_attention(length=256, seed=5201)
    dc = I.delta_prefill(length=128, seed=5202)
    rng = np.random.default_rng(5203)
    w = rng.integers(0, 256, size=(256 * 2, 144), dtype=np.uint8)
    w[:, 0:2] = np.frombuffer(np.float16(0.03125).tobytes(), np.uint8)     # finite d, dmin
    w[:, 2:4] = np.frombuffer(np.float16(0.015625).tobytes(), np.uint8)
    w = w.reshape(-1)
    x = np.sin(np.arange(3 * 512, dtype=np.float32) * 0.07) * 0.13
    first = _run_on(hot, 0, case, pre, dc, w, x)
    second = _run_on(hot, 1, case, pre, dc, w, x)
    for name in first:
        assert np.isfinite(first[name]).all(), name
        assert np.array_equal(first[name], second[name]), name
