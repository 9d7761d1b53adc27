"""The C ABI without a GPU: the header is valid C11, the library exports every
declared symbol, and argument validation happens before any buffer or CUDA
call (restating tests/test_native_abi.py and the rejection half of
tests/test_cuda.py:72-87 of the reference)."""
import ctypes as ct
import math
import re
import shutil
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / 'include' / 'runtime.h'


def declared_symbols():
    text = re.sub(r'/\*.*?\*/', '', HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r'\b(qv_[a-z0-9_]+)\s*\(', text)))


@pytest.mark.skipif(not shutil.which('cc'), reason='a C compiler is required')
def test_header_is_strict_c11(tmp_path):
    src = tmp_path / 'abi.c'
    src.write_text('''
#include "runtime.h"
int main(void) {
    const char *(*error)(void) = qv_error;
    int (*mm)(float *, const void *, const float *, int, int, int, int) = qv_test_mm;
    int (*norm)(float *, const float *, const float *, int, int, float) = qv_test_norm;
    int (*verify)(void *, const int *, int, float *) = qv_verify;
    int (*commit)(void *, int) = qv_commit;
    int (*attn)(float *, void *, void *, const float *, const float *, const float *,
                const float *, const float *, int, int, float) = qv_test_attention;
    int (*delta)(float *, float *, float *, const float *, const float *, const float *,
                 const float *, const float *, const float *, const float *, const float *,
                 int, int, int, int, float) = qv_test_delta;
    size_t (*ws)(int, int) = qv_attention_workspace;
    return error == 0 || mm == 0 || norm == 0 || verify == 0 || commit == 0 ||
           attn == 0 || delta == 0 || ws == 0;
}
''')
    r = subprocess.run(['cc', '-std=c11', '-Wall', '-Wextra', '-Werror', '-fsyntax-only',
                        f'-I{ROOT / "include"}', str(src)], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr


def test_reference_symbols_are_declared():
    names = set(declared_symbols())
    reference = {'qv_error', 'qv_test_mm', 'qv_test_mm_fast', 'qv_test_norm', 'qv_test_delta',
                 'qv_test_attention', 'qv_create', 'qv_upload', 'qv_evaluate', 'qv_verify',
                 'qv_commit', 'qv_advance', 'qv_reset', 'qv_checkpoint', 'qv_restore',
                 'qv_position', 'qv_destroy'}
    assert reference <= names


def test_library_exports_every_declared_symbol(lib):
    out = subprocess.run(['nm', '-D', '--defined-only', lib._name], capture_output=True, text=True).stdout
    exported = set(re.findall(r'\sT\s(qv_\w+)', out))
    missing = [n for n in declared_symbols() if n not in exported]
    assert not missing, missing
    for name in declared_symbols():
        assert getattr(lib, name) is not None


def floats(values):
    return (ct.c_float * len(values))(*values)


def test_rejects_invalid_arguments_before_accessing_buffers(lib):
    value = floats([1.])
    for projection in (lib.qv_test_mm, lib.qv_test_mm_fast):
        for kind, batch, width, rows in ((0, 1, 256, 1), (8, 0, 32, 1), (12, 9, 256, 1),
                                         (14, 1, 255, 1), (8, 1, 32, 0)):
            assert projection(value, value, value, kind, batch, width, rows) == -1
            assert lib.qv_error()
        assert projection(None, value, value, 8, 1, 32, 1) == -1
    for eps in (0., -1., math.nan, math.inf):
        assert lib.qv_test_norm(value, value, value, 1, 1, eps) == -1
    assert lib.qv_test_delta(*([value] * 11), 1, 1, 1, 64, 1e-6) == -1
    assert lib.qv_test_attention(*([value] * 8), 8, 139257, 1e-6) == -1
    assert lib.qv_error() == b'attention context exceeds 139264'
    # more rejections of the hot-path entry points
    assert lib.qv_test_attention(*([value] * 8), 9, 0, 1e-6) == -1
    assert lib.qv_test_attention(*([value] * 8), 1, -1, 1e-6) == -1
    assert lib.qv_test_attention(*([value] * 7), None, 1, 0, 1e-6) == -1
    assert lib.qv_test_delta(*([value] * 11), 9, 1, 1, 32, 1e-6) == -1
    assert lib.qv_test_delta(*([value] * 11), 1, 3, 4, 32, 1e-6) == -1       # 4 % 3 != 0
    assert lib.qv_test_delta(*([value] * 11), 1, 1, 49, 32, 1e-6) == -1      # > 48 heads
    assert lib.qv_test_delta(*([value] * 11), 1, 2, 1, 32, 1e-6) == -1       # Hv < Hk
    assert lib.qv_test_attention_prefill(*([value] * 8), 139265, 0, 1e-6) == -1
    assert lib.qv_test_delta_prefill(*([value] * 11), 0, 1, 1, 32, 1e-6) == -1


def test_model_abi_fails_cleanly(lib):
    handle = ct.c_void_p()
    assert lib.qv_create(None, b'x', 16, 1e-6) == -1
    assert lib.qv_create(ct.byref(handle), b'x', 0, 1e-6) == -1
    assert b'context capacity' in lib.qv_error()
    assert lib.qv_create(ct.byref(handle), b'x', 16, 1e-6) == -1
    assert not handle.value
    assert lib.qv_evaluate(None, None, 1, None) == -1
    assert lib.qv_error() == b'null model handle'
    position = ct.c_int()
    assert lib.qv_position(None, ct.byref(position)) == -1
    lib.qv_destroy(None)


def test_device_entry_points_validate_first(lib):
    v = ct.c_void_p(8)   # never dereferenced: validation fails first
    assert lib.qv_attention_workspace(0, 0) == 0
    assert lib.qv_attention(v, v, v, v, v, v, v, v, 1, 139264, 1e-6, v, 1, None) == -1
    assert lib.qv_attention_shard(v, v, v, v, 0, 10, v, v, v, v, v, 11, 100, 1e-6, v, 1, None) == -1
    assert lib.qv_attention_shard(v, v, v, v, 0, 101, v, v, v, v, v, 1, 100, 1e-6, v, 1, None) == -1
    assert b'past the verify position' in lib.qv_error()
    assert lib.qv_attention_merge(v, v, v, 0, 1, v, None) == -1
    assert lib.qv_prefill_attention(v, None, v, v, v, 0, 0, None) == -1
    assert lib.qv_delta(v, v, v, v, v, v, v, v, v, v, v, 1, 16, 48, 64, 1e-6, None) == -1
    assert lib.qv_delta_core(v, v, v, v, v, v, v, v, v, 0, 16, 48, 128, None) == -1
    assert lib.qv_delta_chunked_workspace(0, 48) == 0
    assert lib.qv_delta_chunked_workspace(4096, 48) > 0
    need = lib.qv_delta_chunked_workspace(64, 48)
    assert lib.qv_delta_chunked(v, v, v, v, v, v, v, v, v, 64, 16, 48, 32, v, need, None) == -1   # dim 32
    assert lib.qv_delta_chunked(v, v, v, v, v, v, v, v, v, 64, 16, 48, 128, v, need - 1, None) == -1
    assert lib.qv_delta_chunked(v, v, v, v, v, v, v, v, v, 64, 16, 48, 128, None, need, None) == -1
    # the tensor-core projection streams 16-byte pieces: unaligned weights or activations are rejected
    a16, odd = ct.c_void_p(4096), ct.c_void_p(4098)
    assert lib.qv_mm(a16, odd, a16, 12, 8, 512, 7, 0, None) == -1
    assert b'16-byte aligned' in lib.qv_error()
    assert lib.qv_mm(a16, a16, odd, 8, 8, 512, 7, 1, None) == -1
    assert b'16-byte aligned' in lib.qv_error()


def _prototype_arg_counts():
    text = re.sub(r'/\*.*?\*/', '', HEADER.read_text(), flags=re.S)
    counts = {}
    for m in re.finditer(r'\b(qv_[a-z0-9_]+)\s*\(([^)]*)\)\s*;', text):
        args = m.group(2).strip()
        counts[m.group(1)] = 0 if args in ('', 'void') else args.count(',') + 1
    return counts


def test_ctypes_signatures_match_the_header():
    """Every ctypes argtypes list has exactly as many entries as the C prototype."""
    from redshift_b200.runtime import ADDITIVE_SIGNATURES, MODEL_SIGNATURES, REFERENCE_SIGNATURES
    counts = _prototype_arg_counts()
    tables = dict(REFERENCE_SIGNATURES)
    tables.update(MODEL_SIGNATURES)
    tables.update({k: v[0] for k, v in ADDITIVE_SIGNATURES.items()})
    for name, argtypes in tables.items():
        assert name in counts, name
        assert len(argtypes) == counts[name], (name, len(argtypes), counts[name])


def test_no_alloc_scratch_covers_every_accepted_call(lib):
    """qv_attention_noalloc's fixed scratch (10 MiB per GPU, the size include/runtime.h states)
    must hold the workspace of every call it accepts: batch 1..8 at every context up to 139,264.
    A change to the split-KV plan that outgrows the array fails here, not in a serving call."""
    scratch = 10 << 20
    for batch in range(1, 9):
        positions = sorted(set(range(0, 139264 - batch + 1, 997)) | {139264 - batch})
        need = max(lib.qv_attention_workspace(batch, p) for p in positions)
        assert 0 < need <= scratch, (batch, need)
    v = ct.c_void_p(8)   # never dereferenced: the exchange sequence number is validated first
    assert lib.qv_attention_shard_exchange(v, v, v, 0, 10, v, v, v, v, v, 8, 100, 1e-6, v, 2, 0, -1, v, 1 << 30,
                                           None) == -1
    assert b'sequence number' in lib.qv_error()
