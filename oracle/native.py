"""The C restatement of the oracle (``oracle/c/qv_oracle.c``): build and bindings.

TEST INFRASTRUCTURE ONLY, like the rest of ``oracle/``: the product library
never loads it.  ``build()`` compiles it with gcc into
``oracle/_build/libqvoracle.so`` (x86-64-v3 code: AVX2 + FMA, so the library
built here also runs on the GPU box's host); ``attention`` and ``delta`` call
it with numpy arrays and return what ``oracle.attention`` / ``oracle.delta``
return, computed in float64 on ``threads`` host threads.
"""
import ctypes as ct
import os
import shutil
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
SOURCE = HERE / 'c' / 'qv_oracle.c'
LIBRARY = HERE / '_build' / 'libqvoracle.so'
FLAGS = ['-O3', '-march=x86-64-v3', '-fPIC', '-shared', '-pthread', '-Wall', '-Wextra']


def build(force=False):
    """Compile the C oracle (incremental)."""
    LIBRARY.parent.mkdir(exist_ok=True)
    if force or not LIBRARY.exists() or SOURCE.stat().st_mtime > LIBRARY.stat().st_mtime:
        cc = shutil.which('gcc') or shutil.which('cc') or 'gcc'
        subprocess.run([cc, *FLAGS, str(SOURCE), '-o', str(LIBRARY), '-lm'], check=True)
    return LIBRARY


_lib = None


def load():
    """The compiled library (built on first use where a compiler exists)."""
    global _lib
    if _lib is None:
        if not LIBRARY.exists():
            build()
        lib = ct.CDLL(str(LIBRARY))
        P, I, D = ct.c_void_p, ct.c_int, ct.c_double
        lib.qvo_attention.argtypes = [P] * 8 + [I, I, D, I]
        lib.qvo_attention.restype = I
        lib.qvo_delta.argtypes = [P] * 11 + [I, I, I, I, D, I, I]
        lib.qvo_delta.restype = I
        _lib = lib
    return _lib


def default_threads():
    return len(os.sched_getaffinity(0)) if hasattr(os, 'sched_getaffinity') else (os.cpu_count() or 1)


def _f32(a):
    return np.ascontiguousarray(np.asarray(a, np.float32).reshape(-1))


def _ptr(a):
    return a.ctypes.data_as(ct.c_void_p)


def attention(key_cache, value_cache, q_gate, key, value, q_norm, k_norm, batch, position, epsilon,
              threads=None, caches_in_place=False):
    """cpu_reference.attention: returns (out float64 [batch*24*256], kc, vc float16 [position+batch,4,256]).

    With ``caches_in_place`` the given float16 caches (capacity >= position+batch rows) are
    appended to in place instead of copied (what a timed step does)."""
    n = position + batch
    if caches_in_place:
        kc, vc = key_cache, value_cache
    else:
        kc = np.zeros((n, 4, 256), np.float16)
        vc = np.zeros((n, 4, 256), np.float16)
        kc.reshape(-1)[:position * 1024] = np.asarray(key_cache, np.float16).reshape(-1)[:position * 1024]
        vc.reshape(-1)[:position * 1024] = np.asarray(value_cache, np.float16).reshape(-1)[:position * 1024]
    out = np.empty(batch * 24 * 256, np.float64)
    args = [_f32(x) for x in (q_gate, key, value, q_norm, k_norm)]
    rc = load().qvo_attention(_ptr(out), _ptr(kc), _ptr(vc), *map(_ptr, args), batch, position, float(epsilon),
                              threads or default_threads())
    if rc:
        raise ValueError('qvo_attention rejected its arguments')
    return out, kc, vc


def delta(state, history, qkv, gate, alpha, beta, conv, decay, bias, norm, batch, key_heads, value_heads, dim,
          epsilon, threads=None, round_filtered=False):
    """cpu_reference.delta: returns (out, state, history) as float64 flat arrays.  With
    ``round_filtered`` the conv + SiLU outputs are rounded to fp16 first (a model of a kernel that
    takes them as fp16 operands, as the chunked layer prefill does; the reference does not round)."""
    st = np.array(state, np.float64).reshape(-1).copy()
    hi = np.array(history, np.float64).reshape(-1).copy()
    out = np.empty(batch * value_heads * dim, np.float64)
    args = [_f32(x) for x in (qkv, gate, alpha, beta, conv, decay, bias, norm)]
    rc = load().qvo_delta(_ptr(out), _ptr(st), _ptr(hi), *map(_ptr, args), batch, key_heads, value_heads, dim,
                          float(epsilon), threads or default_threads(), int(bool(round_filtered)))
    if rc:
        raise ValueError('qvo_delta rejected its arguments')
    return out, st, hi
