"""ctypes bindings of ``build/libqvelox.so`` (sm_100a build of the hot path).

``load_library`` binds the same symbols with the same ctypes signatures as the
reference loader (cristianku/redshift ``qvelox/runtime.py:6-22``), then the
additive entry points of ``include/runtime.h``.  A missing library raises at
once: there is no CPU fallback anywhere in this package.

``HotPath`` is a thin convenience layer over the device-resident entry points
for callers that hold their buffers as torch CUDA tensors (torch supplies the
device memory and the current stream; all arithmetic runs in the library's
own kernels).
"""
import ctypes as ct
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
DEFAULT_LIBRARY = ROOT / 'build' / 'libqvelox.so'

_P, _I, _F, _S = ct.c_void_p, ct.c_int, ct.c_float, ct.c_size_t

# The reference loader's table (qvelox/runtime.py:11-17), unchanged.
REFERENCE_SIGNATURES = {
    'qv_test_mm': [_P] * 3 + [_I] * 4,
    'qv_test_mm_fast': [_P] * 3 + [_I] * 4,
    'qv_test_norm': [_P] * 3 + [_I] * 2 + [_F],
    'qv_test_delta': [_P] * 11 + [_I] * 4 + [_F],
    'qv_test_attention': [_P] * 8 + [_I] * 2 + [_F],
}
# Model ABI of the reference (qvelox/runtime.py:37-46).
MODEL_SIGNATURES = {
    'qv_create': [ct.POINTER(_P), ct.c_char_p, _I, _F],
    'qv_upload': [_P, _I, ct.c_uint64, ct.c_uint64],
    'qv_evaluate': [_P, ct.POINTER(_I), _I, ct.POINTER(_F)],
    'qv_verify': [_P, ct.POINTER(_I), _I, ct.POINTER(_F)],
    'qv_commit': [_P, _I],
    'qv_advance': [_P, ct.POINTER(_I), _I, ct.POINTER(_I)],
    'qv_position': [_P, ct.POINTER(_I)],
    'qv_reset': [_P], 'qv_checkpoint': [_P], 'qv_restore': [_P],
}
# Additive entry points (include/runtime.h, part 2).
ADDITIVE_SIGNATURES = {
    'qv_test_attention_prefill': ([_P] * 8 + [_I] * 2 + [_F], _I),
    'qv_test_delta_prefill': ([_P] * 11 + [_I] * 4 + [_F], _I),
    'qv_attention_workspace': ([_I, _I], _S),
    'qv_attention': ([_P] * 8 + [_I, _I, _F, _P, _S, _P], _I),
    'qv_delta': ([_P] * 11 + [_I] * 4 + [_F, _P], _I),
    'qv_delta_trace_floats': ([_I, _I, _I], _S),
    'qv_mm_weight_bytes': ([_I, _I, _I], _S),
    'qv_copy_spans': ([_P, _P, _P, _I, _P], _I),
    'qv_mm': ([_P] * 3 + [_I] * 5 + [_P], _I),
    'qv_delta_verify': ([_P] * 11 + [_I] * 4 + [_F] + [_P] * 4, _I),
    'qv_delta_commit': ([_P] * 5 + [_I] * 5 + [_P], _I),
    'qv_attention_shard_workspace': ([_I, _I], _S),
    'qv_attention_shard': ([_P] * 4 + [_I, _I] + [_P] * 5 + [_I, _I, _F, _P, _S, _P], _I),
    'qv_attention_merge': ([_P] * 3 + [_I, _I, _P, _P], _I),
    'qv_attention_exchange_bytes': ([_I], _S),
    'qv_attention_shard_exchange': ([_P] * 3 + [_I, _I] + [_P] * 5 + [_I, _I, _F] + [_P, _I, _I, _I, _P, _S, _P], _I),
    'qv_prefill_attention': ([_P] * 5 + [_I, _I, _P], _I),
    'qv_delta_core': ([_P] * 9 + [_I] * 4 + [_P], _I),
    'qv_delta_chunked_workspace': ([_I, _I], _S),
    'qv_delta_chunked': ([_P] * 9 + [_I] * 4 + [_P, _S, _P], _I),
    'qv_delta_prefill_workspace': ([_I, _I, _I], _S),
    'qv_delta_prefill': ([_P] * 11 + [_I] * 4 + [_F, _P, _S, _P], _I),
    'qv_status': ([], _I),
    'qv_attention_noalloc': ([_P] * 8 + [_I, _I, _F, _P], _I),
}


def load_library(path=None):
    """Load the library and declare every exported signature.

    Raises ``OSError`` when the library is missing: build it with
    ``python -m redshift_b200.build``.
    """
    path = Path(path) if path is not None else DEFAULT_LIBRARY
    if not path.exists():
        raise OSError(f'{path} is missing; build it with `python -m redshift_b200.build`')
    lib = ct.CDLL(str(path.resolve()))
    lib.qv_error.argtypes = []
    lib.qv_error.restype = ct.c_char_p
    for table in (REFERENCE_SIGNATURES, MODEL_SIGNATURES):
        for name, signature in table.items():
            fn = getattr(lib, name)
            fn.argtypes = signature
            fn.restype = _I
    lib.qv_destroy.argtypes = [_P]
    lib.qv_destroy.restype = None
    for name, (signature, restype) in ADDITIVE_SIGNATURES.items():
        fn = getattr(lib, name)
        fn.argtypes = signature
        fn.restype = restype
    return lib


class NativeError(RuntimeError):
    """A library call returned -1; the message is ``qv_error()``."""


class HotPath:
    """Device-resident hot-path calls on torch CUDA tensors.

    Every method validates shapes/dtypes on the host, then calls one entry
    point of the library on torch's current CUDA stream.  Buffers are used in
    place; nothing is copied or converted here.
    """

    def __init__(self, library=None):
        self.lib = load_library(library)
        self._workspace = None

    # -- helpers ---------------------------------------------------------
    def check(self, code):
        if code:
            raise NativeError(self.lib.qv_error().decode('utf-8', errors='replace'))

    @staticmethod
    def _stream():
        import torch
        return ct.c_void_p(torch.cuda.current_stream().cuda_stream)

    @staticmethod
    def _ptr(t):
        return ct.c_void_p(t.data_ptr()) if t is not None else None

    def workspace(self, nbytes, device):
        """A cached device workspace of at least ``nbytes`` bytes, zero-filled when it is made (the
        attention workspace's barrier words must start at zero; the calls keep them so)."""
        import torch
        if self._workspace is None or self._workspace.numel() < nbytes or self._workspace.device != device:
            self._workspace = torch.zeros(max(int(nbytes), 256), dtype=torch.uint8, device=device)
        return self._workspace

    # -- attention --------------------------------------------------------
    def attention(self, out, key_cache, value_cache, q_gate, key, value, q_norm, k_norm,
                  batch, position, epsilon=1e-6, workspace=None):
        """One attention layer (prepare + decode/verify or prefill) in place."""
        need = self.lib.qv_attention_workspace(batch, position)
        ws = workspace if workspace is not None else self.workspace(need, out.device)
        p = self._ptr
        self.check(self.lib.qv_attention(p(out), p(key_cache), p(value_cache), p(q_gate), p(key), p(value),
                                         p(q_norm), p(k_norm), batch, position, epsilon, p(ws),
                                         ws.numel() * ws.element_size(), self._stream()))

    def attention_shard(self, partial, lse, key_cache, value_cache, shard_begin, shard_rows, q_gate, key,
                        value, q_norm, k_norm, batch, position, epsilon=1e-6, workspace=None):
        need = self.lib.qv_attention_shard_workspace(batch, shard_rows)
        ws = workspace if workspace is not None else self.workspace(need, partial.device)
        p = self._ptr
        self.check(self.lib.qv_attention_shard(p(partial), p(lse), p(key_cache), p(value_cache), shard_begin,
                                               shard_rows, p(q_gate), p(key), p(value), p(q_norm), p(k_norm),
                                               batch, position, epsilon, p(ws), ws.numel() * ws.element_size(),
                                               self._stream()))

    def attention_shard_exchange(self, out, key_cache, value_cache, shard_begin, shard_rows, q_gate, key, value,
                                 q_norm, k_norm, batch, position, peers, world, rank, sequence, epsilon=1e-6,
                                 workspace=None):
        """Shard attention + peer-memory exchange + merge (``peers``: int64 device tensor of buffer
        addresses; ``sequence``: the call's number on these buffers, +1 per call, the same on every rank)."""
        need = self.lib.qv_attention_shard_workspace(batch, shard_rows)
        ws = workspace if workspace is not None else self.workspace(need, out.device)
        p = self._ptr
        self.check(self.lib.qv_attention_shard_exchange(
            p(out), p(key_cache), p(value_cache), shard_begin, shard_rows, p(q_gate), p(key), p(value), p(q_norm),
            p(k_norm), batch, position, epsilon, p(peers), world, rank, sequence, p(ws), ws.numel() * ws.element_size(),
            self._stream()))

    def attention_merge(self, out, partials, lses, shards, batch, q_gate):
        p = self._ptr
        self.check(self.lib.qv_attention_merge(p(out), p(partials), p(lses), shards, batch, p(q_gate),
                                               self._stream()))

    def prefill_attention(self, out, q, key_cache, value_cache, tokens, position=0, lse=None):
        p = self._ptr
        self.check(self.lib.qv_prefill_attention(p(out), p(lse), p(q), p(key_cache), p(value_cache), tokens,
                                                 position, self._stream()))

    # -- DeltaNet ---------------------------------------------------------
    def delta(self, out, state, history, qkv, gate, alpha, beta, conv, decay, bias, norm,
              batch, key_heads, value_heads, dim, epsilon=1e-6):
        p = self._ptr
        self.check(self.lib.qv_delta(p(out), p(state), p(history), p(qkv), p(gate), p(alpha), p(beta),
                                     p(conv), p(decay), p(bias), p(norm), batch, key_heads, value_heads, dim,
                                     epsilon, self._stream()))

    def copy_spans(self, pairs):
        """qv_copy_spans over [(dst_tensor, src_tensor[, bytes]), ...] (whole tensors by default)."""
        import ctypes
        n = len(pairs)
        dst = (ctypes.c_void_p * n)(*[d.data_ptr() for d, s, *_ in pairs])
        src = (ctypes.c_void_p * n)(*[s.data_ptr() for d, s, *_ in pairs])
        nb = (ctypes.c_size_t * n)(*[(rest[0] if rest else s.numel() * s.element_size()) for d, s, *rest in pairs])
        self.check(self.lib.qv_copy_spans(dst, src, nb, n, self._stream()))

    def mm(self, out, weights, x, kind, batch, width, rows, fast=False):
        """qv_mm: out [batch][rows] = W x for a block-quantized W on the device."""
        p = self._ptr
        self.check(self.lib.qv_mm(p(out), p(weights), p(x), kind, batch, width, rows, int(bool(fast)),
                                  self._stream()))

    def delta_verify(self, out, state, history, qkv, gate, alpha, beta, conv, decay, bias, norm,
                     batch, key_heads, value_heads, dim, saved_state, saved_history, trace, epsilon=1e-6):
        """qv_delta_verify: qv_delta that also saves the start state / history and
        writes the transition trace that qv_delta_commit replays."""
        p = self._ptr
        self.check(self.lib.qv_delta_verify(p(out), p(state), p(history), p(qkv), p(gate), p(alpha), p(beta),
                                            p(conv), p(decay), p(bias), p(norm), batch, key_heads, value_heads,
                                            dim, epsilon, p(saved_state), p(saved_history), p(trace),
                                            self._stream()))

    def delta_commit(self, state, history, saved_state, saved_history, trace, accepted, batch,
                     key_heads, value_heads, dim):
        """qv_delta_commit: keep the first `accepted` tokens of a recorded verify."""
        p = self._ptr
        self.check(self.lib.qv_delta_commit(p(state), p(history), p(saved_state), p(saved_history), p(trace),
                                            accepted, batch, key_heads, value_heads, dim, self._stream()))

    def delta_core(self, out, state, q, k, v, alpha, beta, decay, bias, tokens, key_heads, value_heads, dim):
        p = self._ptr
        self.check(self.lib.qv_delta_core(p(out), p(state), p(q), p(k), p(v), p(alpha), p(beta), p(decay),
                                          p(bias), tokens, key_heads, value_heads, dim, self._stream()))

    def delta_chunked(self, out, state, q, k, v, alpha, beta, decay, bias, tokens, key_heads, value_heads, dim,
                      workspace=None):
        """qv_delta_chunked; allocates the workspace when none is given."""
        p = self._ptr
        need = self.lib.qv_delta_chunked_workspace(tokens, value_heads)
        if workspace is None:
            import torch
            workspace = torch.empty(max(need, 1), dtype=torch.uint8, device=out.device)
        self.check(self.lib.qv_delta_chunked(p(out), p(state), p(q), p(k), p(v), p(alpha), p(beta), p(decay),
                                             p(bias), tokens, key_heads, value_heads, dim, p(workspace),
                                             workspace.numel() * workspace.element_size(), self._stream()))

    def delta_prefill(self, out, state, history, qkv, gate, alpha, beta, conv, decay, bias, norm,
                      tokens, key_heads, value_heads, dim, epsilon=1e-6, workspace=None):
        """qv_delta_prefill: the DeltaNet layer over a long block in the chunked form; allocates the
        workspace when none is given."""
        p = self._ptr
        need = self.lib.qv_delta_prefill_workspace(tokens, key_heads, value_heads)
        if workspace is None:
            import torch
            workspace = torch.empty(max(need, 1), dtype=torch.uint8, device=out.device)
        self.check(self.lib.qv_delta_prefill(p(out), p(state), p(history), p(qkv), p(gate), p(alpha), p(beta),
                                             p(conv), p(decay), p(bias), p(norm), tokens, key_heads, value_heads,
                                             dim, epsilon, p(workspace), workspace.numel() * workspace.element_size(),
                                             self._stream()))

    def status(self):
        """Synchronise and return the kernel status word (0 = no timeout)."""
        code = self.lib.qv_status()
        if code < 0:
            raise NativeError(self.lib.qv_error().decode('utf-8', errors='replace'))
        return code
