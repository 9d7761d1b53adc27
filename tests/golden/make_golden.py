"""Generate golden vectors by running the reference's own CPU oracle.

Run in a container where cristianku/redshift is checked out (by default as
``reference/`` beside this repository's checkout; override with
``REDSHIFT_REFERENCE``)::

    python tests/golden/make_golden.py

It imports the reference's ``tests/cpu_reference.py`` unchanged, feeds it the
inputs produced by ``oracle.inputs`` (seeded / deterministic) and stores the
reference outputs as compressed ``.npz`` files next to this script, together
with a digest of the inputs so that a drift of the input generators is
detected.  The fixtures pin the numpy restatement in ``oracle/``; the GPU
tests then compare the CUDA kernels to that restatement.  Nothing on the GPU
box reads the reference checkout.
"""
import os
import sys
import time
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1]))
from oracle import inputs as I  # noqa: E402


def reference_module():
    root = Path(os.environ.get('REDSHIFT_REFERENCE', HERE.parents[2] / 'reference'))
    sys.path.insert(0, str(root / 'tests'))
    import cpu_reference  # noqa: E402  (the reference's own oracle, unchanged)
    return cpu_reference


def flat(a):
    return [float(x) for x in np.asarray(a, dtype=np.float64).reshape(-1)]


def run_attention(ref, case):
    c = dict(case)
    pos, batch = c['position'], c['batch']
    t0 = time.time()
    out, kc, vc = ref.attention(flat(c['key_cache'])[:pos * 1024], flat(c['value_cache'])[:pos * 1024],
                                flat(c['q_gate']), flat(c['key']), flat(c['value']),
                                flat(c['q_norm']), flat(c['k_norm']), batch, pos, c['epsilon'])
    dt = time.time() - t0
    digest = I.checksum([c[k] for k in ('key_cache', 'value_cache', 'q_gate', 'key', 'value',
                                        'q_norm', 'k_norm')])
    return dict(out=np.array(out), new_k=np.array(kc[pos * 1024:]), new_v=np.array(vc[pos * 1024:]),
                position=pos, batch=batch, digest=digest, seconds=dt)


def run_delta(ref, case, state_heads=None):
    c = dict(case)
    t0 = time.time()
    out, state, hist = ref.delta(flat(c['state']), flat(c['history']), flat(c['qkv']), flat(c['gate']),
                                 flat(c['alpha']), flat(c['beta']), flat(c['conv']), flat(c['decay']),
                                 flat(c['bias']), flat(c['norm']), c['batch'], c['key_heads'],
                                 c['value_heads'], c['dim'], c['epsilon'])
    dt = time.time() - t0
    digest = I.checksum([c[k] for k in ('state', 'history', 'qkv', 'gate', 'alpha', 'beta', 'conv',
                                        'decay', 'bias', 'norm')])
    state = np.array(state).reshape(c['value_heads'], c['dim'], c['dim'])
    res = dict(out=np.array(out), history=np.array(hist), digest=digest, seconds=dt)
    if state_heads is None:
        res['state'] = state
    else:
        res['state_heads'] = np.array(state_heads)
        res['state'] = state[state_heads]
    return res


def main():
    ref = reference_module()
    cases = {
        'attention_wave': (run_attention, I.attention_wave(), {}),
        'attention_cfg0': (run_attention, I.attention_layer(batch=8, position=128), {}),
        'attention_edge': (run_attention, I.attention_layer(batch=8, position=250, seed=1100), {}),
        'attention_single': (run_attention, I.attention_layer(batch=1, position=0, seed=1101), {}),
        'delta_wave_d32': (run_delta, I.delta_wave(32), {}),
        'delta_wave_d128': (run_delta, I.delta_wave(128), {}),
        'delta_cfg1': (run_delta, I.delta_layer(batch=8), {'state_heads': [0, 17, 47]}),
        'delta_small_t1': (run_delta, I.delta_layer(batch=1, seed=1102, key_heads=4, value_heads=12,
                                                    dim=128, state_std=0.05), {'state_heads': [0, 5, 11]}),
    }
    for name, (fn, case, kw) in cases.items():
        res = fn(ref, case, **kw)
        np.savez_compressed(HERE / f'{name}.npz', **res)
        print(f'{name}: {res["seconds"]:.2f} s', flush=True)


if __name__ == '__main__':
    main()
