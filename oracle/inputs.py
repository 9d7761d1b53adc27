"""Seeded synthetic inputs for the five benchmark configurations and the
deterministic "wave" inputs of the reference's kernel tests.

TEST INFRASTRUCTURE ONLY.  Shapes and distributions follow the reference's
benchmark configurations (24 query / 4 KV heads of dim 256; 16 key / 48 value
DeltaNet heads of dim 128; fp16 N(0,1) activations, DeltaNet state N(0,0.02)).
The wave inputs restate the generators of ``tests/test_cuda.py:164-235``.
Numpy's ``default_rng`` (PCG64) is used with a fixed seed per configuration.
"""
import math

import numpy as np

SEED_BASE = 1000                  # seed = 1000 + configuration index
H, HKV, D = 24, 4, 256
HK, HV, DK = 16, 48, 128
CHANNELS = (2 * HK + HV) * DK     # 10240, runtime.cu:206


def f16(x):
    """fp16-round (values stay float32 arrays, exactly representable)."""
    return np.asarray(x).astype(np.float16).astype(np.float32)


_QUANTILES = None


def normal_f16(rng, shape):
    """Fast fp16 N(0,1) sample: uniform 16-bit indices into the table of the
    65536 mid-point quantiles of N(0,1), rounded to fp16.  Used for caches of
    long contexts, where drawing ~10^8 float normals would dominate."""
    global _QUANTILES
    if _QUANTILES is None:
        from scipy.special import ndtri
        _QUANTILES = ndtri((np.arange(65536) + 0.5) / 65536).astype(np.float16)
    return _QUANTILES[rng.integers(0, 65536, size=shape, dtype=np.uint16)]


def attention_layer(batch=8, position=128, seed=SEED_BASE + 0, prefix=True, fast=None):
    """ABI-level inputs of one attention call (configs 0 and 2).

    Caches hold the fp16 prefix ``[position,4,256]`` plus ``batch`` empty rows.
    ``q_gate`` [batch,24,512], ``key``/``value`` [batch,4,256] are fp16-rounded
    N(0,1) float32; both RMSNorm weights are 1, epsilon 1e-6.  Prefixes longer
    than 16384 rows use ``normal_f16`` (``fast``) unless told otherwise.
    """
    rng = np.random.default_rng(seed)
    n = position + batch
    kc = np.zeros((n, HKV, D), dtype=np.float16)
    vc = np.zeros((n, HKV, D), dtype=np.float16)
    fast = position > 16384 if fast is None else fast
    if prefix and position:
        if fast:
            kc[:position] = normal_f16(rng, (position, HKV, D))
            vc[:position] = normal_f16(rng, (position, HKV, D))
        else:
            kc[:position] = rng.standard_normal((position, HKV, D), dtype=np.float32).astype(np.float16)
            vc[:position] = rng.standard_normal((position, HKV, D), dtype=np.float32).astype(np.float16)
    return dict(
        key_cache=kc, value_cache=vc,
        q_gate=f16(rng.standard_normal((batch, H, 2 * D), dtype=np.float32)),
        key=f16(rng.standard_normal((batch, HKV, D), dtype=np.float32)),
        value=f16(rng.standard_normal((batch, HKV, D), dtype=np.float32)),
        q_norm=np.ones(D, np.float32), k_norm=np.ones(D, np.float32),
        batch=batch, position=position, epsilon=1e-6)


def delta_layer(batch=8, seed=SEED_BASE + 1, key_heads=HK, value_heads=HV, dim=DK,
                state_std=0.02):
    """ABI-level inputs of one DeltaNet call (config 1).

    State N(0,0.02) float32; raw qkv fp16 N(0,1); conv taps [0,0,0,1] so the
    conv output is SiLU(raw); zero history; alpha N(0,1) with decay -1 and
    bias 0 (so the log decay is -softplus(alpha)); raw beta N(0,1); gate z
    N(0,1); norm weight 1; epsilon 1e-6.
    """
    rng = np.random.default_rng(seed)
    C = (2 * key_heads + value_heads) * dim
    conv = np.zeros((C, 4), np.float32)
    conv[:, 3] = 1.0
    return dict(
        state=(rng.standard_normal((value_heads, dim, dim)) * state_std).astype(np.float32),
        history=np.zeros((3, C), np.float32),
        qkv=f16(rng.standard_normal((batch, C), dtype=np.float32)),
        gate=rng.standard_normal((batch, value_heads, dim), dtype=np.float32),
        alpha=rng.standard_normal((batch, value_heads), dtype=np.float32),
        beta=rng.standard_normal((batch, value_heads), dtype=np.float32),
        conv=conv,
        decay=np.full(value_heads, -1.0, np.float32),
        bias=np.zeros(value_heads, np.float32),
        norm=np.ones(dim, np.float32),
        batch=batch, key_heads=key_heads, value_heads=value_heads, dim=dim, epsilon=1e-6)


def prefill_attention(length=4096, seed=SEED_BASE + 3):
    """Core-level causal prefill inputs (config 3): fp16 N(0,1) Q/K/V."""
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((length, H, D), dtype=np.float32).astype(np.float16)
    k = rng.standard_normal((length, HKV, D), dtype=np.float32).astype(np.float16)
    v = rng.standard_normal((length, HKV, D), dtype=np.float32).astype(np.float16)
    return q, k, v


def delta_prefill(length=4096, seed=SEED_BASE + 4, key_heads=HK, value_heads=HV, dim=DK):
    """Core-level chunked-DeltaNet inputs (config 4).

    Raw q, k fp16 N(0,1) [L,Hk,D] (L2-normalised inside the kernel, q also by
    1/sqrt(D)); v fp16 N(0,1) [L,Hv,D]; alpha N(0,1) (log decay
    -softplus(alpha)); raw beta N(0,1) (beta = sigmoid); zero initial state.
    """
    rng = np.random.default_rng(seed)
    return dict(
        q=rng.standard_normal((length, key_heads, dim), dtype=np.float32).astype(np.float16),
        k=rng.standard_normal((length, key_heads, dim), dtype=np.float32).astype(np.float16),
        v=rng.standard_normal((length, value_heads, dim), dtype=np.float32).astype(np.float16),
        alpha=rng.standard_normal((length, value_heads), dtype=np.float32),
        beta=rng.standard_normal((length, value_heads), dtype=np.float32))


# ----------------------------------------------------------------------------
# Deterministic wave inputs (restating tests/test_cuda.py:164-235)
# ----------------------------------------------------------------------------

def wave(n, phase, scale, step):
    """``scale*sin(i*step+phase)`` for i < n, rounded to float32."""
    return np.array([scale * math.sin(i * step + phase) for i in range(n)], np.float32)


def delta_wave(dim, batch=3, key_heads=2, value_heads=4):
    """The DeltaNet case of test_cuda.py:164-176 (step 0.037)."""
    C = (2 * key_heads + value_heads) * dim
    w = lambda n, phase, scale=.1: wave(n, phase, scale, .037)  # noqa: E731
    return dict(
        state=w(value_heads * dim * dim, .3, .01), history=w(3 * C, .7),
        qkv=w(batch * C, 1.1), gate=w(batch * value_heads * dim, 1.7, .8),
        alpha=w(batch * value_heads, .2), beta=w(batch * value_heads, .9),
        conv=w(C * 4, .6, .4),
        decay=np.array([-.5 - h * .1 for h in range(value_heads)], np.float32),
        bias=w(value_heads, .4),
        norm=np.array([.8 + i / dim * .2 for i in range(dim)], np.float32),
        batch=batch, key_heads=key_heads, value_heads=value_heads, dim=dim, epsilon=1e-6)


def attention_wave(batch=3, position=5):
    """The attention case of test_cuda.py:201-213 (step 0.051)."""
    w = lambda n, phase, scale=.3: wave(n, phase, scale, .051)  # noqa: E731
    n = position + batch
    kc = np.zeros((n, HKV, D), np.float16)
    vc = np.zeros((n, HKV, D), np.float16)
    kc[:position] = w(position * 1024, .5).astype(np.float16).reshape(position, HKV, D)
    vc[:position] = w(position * 1024, .9).astype(np.float16).reshape(position, HKV, D)
    return dict(
        key_cache=kc, value_cache=vc, q_gate=w(batch * 12288, 1.5),
        key=w(batch * 1024, .1), value=w(batch * 1024, .7),
        q_norm=np.array([1 + i / 512 for i in range(256)], np.float32),
        k_norm=np.array([1 - i / 512 for i in range(256)], np.float32),
        batch=batch, position=position, epsilon=1e-6)


def checksum(arrays):
    """Order-sensitive digest of input arrays (detects generator drift)."""
    import hashlib
    h = hashlib.sha256()
    for a in arrays:
        a = np.ascontiguousarray(a)
        h.update(str(a.dtype).encode())
        h.update(str(a.shape).encode())
        h.update(a.tobytes())
    return h.hexdigest()
