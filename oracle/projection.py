"""Quantized projections: float64 restatement of the reference's block formats.

TEST INFRASTRUCTURE ONLY (see the package docstring).  The block layouts are
the GGUF formats the reference model reads and its kernels decode
(src/kernels.cu:31-273); the decoding below follows the reference's own
independent decoder in tests/test_cuda.py:17-52, element for element, and is
pinned to it by ``tests/golden/projection_*.npz`` (written by running that
decoder, ``tests/golden/make_projection_golden.py``):

* kind 8, Q8_0: blocks of 32 columns, 34 bytes: fp16 scale d, 32 int8 q;
  w = d q.
* kind 12, Q4_K: super-blocks of 256 columns, 144 bytes: fp16 d, fp16 dmin,
  12 bytes of packed 6-bit (scale, min) pairs for 8 groups of 32, 128 bytes of
  4-bit quants (groups 2j and 2j+1 share 32 bytes, low / high nibble);
  w = d s q - dmin z.
* kind 14, Q6_K: super-blocks of 256 columns, 210 bytes: 128 bytes of low
  nibbles, 64 bytes of 2-bit highs, 16 int8 scales (one per 16 columns), fp16
  d; w = (16 high + low - 32) scale d.

``mm`` is qv_test_mm (out[t][row] = sum_k w[row][k] x[t][k]); ``mm_fast`` is
the reference's 16-bit activation-block path as its test states it
(tests/test_cuda.py:105-145): per 32-column block of each token,
scale = f32(max|x| / 32639), q = round-half-away(f32(x / scale)), and
out = sum_k (w + offset)_k qx_k - offset_k x_k with the Q4_K minimum as the
offset.
"""
import numpy as np

BLOCK = {8: (32, 34), 12: (256, 144), 14: (256, 210)}   # columns, bytes per block


def _half(b, off):
    return np.ascontiguousarray(b[:, off:off + 2]).view(np.float16).astype(np.float64)[:, 0]


def decode(kind, data, width, rows):
    """Dequantised weights [rows][width] (float64) and, for Q4_K, the per-column
    minimum offsets (dmin z) that the fast path keeps exact."""
    cols, nbytes = BLOCK[kind]
    nb = width // cols
    b = np.frombuffer(bytes(data), np.uint8)[:nb * nbytes * rows].reshape(rows * nb, nbytes)
    offsets = np.zeros((rows * nb, cols))
    if kind == 8:
        d = _half(b, 0)
        q = b[:, 2:34].view(np.int8).astype(np.float64)
        w = d[:, None] * q
    elif kind == 12:
        d, dmin = _half(b, 0), _half(b, 2)
        sc = b[:, 4:16].astype(np.int64)
        packed = b[:, 16:144].astype(np.int64)
        w = np.empty((rows * nb, 256))
        for g in range(8):
            if g < 4:
                s, z = sc[:, g] & 63, sc[:, g + 4] & 63
            else:
                s = (sc[:, g + 4] & 15) | ((sc[:, g - 4] >> 6) << 4)
                z = (sc[:, g + 4] >> 4) | ((sc[:, g] >> 6) << 4)
            q = (packed[:, (g // 2) * 32:(g // 2) * 32 + 32] >> (4 * (g % 2))) & 15
            off = (dmin * z)[:, None]
            w[:, g * 32:(g + 1) * 32] = (d * s)[:, None] * q - off
            offsets[:, g * 32:(g + 1) * 32] = off
    else:
        lo = b[:, :128].astype(np.int64)
        hi = b[:, 128:192].astype(np.int64)
        sc = b[:, 192:208].view(np.int8).astype(np.float64)
        d = _half(b, 208)
        w = np.empty((rows * nb, 256))
        for i in range(256):
            half, within = divmod(i, 128)
            quarter, lane = divmod(within, 32)
            low = (lo[:, half * 64 + (quarter % 2) * 32 + lane] >> (4 * (quarter // 2))) & 15
            high = (hi[:, half * 32 + lane] >> (2 * quarter)) & 3
            w[:, i] = ((high * 16 + low) - 32) * sc[:, i // 16] * d
    return w.reshape(rows, width), offsets.reshape(rows, width)


def mm(kind, data, x, batch, width, rows):
    """out [batch][rows] float64 of the exact-activation projection."""
    w, _ = decode(kind, data, width, rows)
    xs = np.asarray(x, np.float64).reshape(batch, width)
    return xs @ w.T


def quantize_activations(x, batch, width):
    """The 16-bit block quantisation of the fast path, in float32 as the
    reference test computes it (ctypes c_float roundings)."""
    xs = np.asarray(x, np.float32).reshape(batch, width // 32, 32)
    m = np.abs(xs).max(axis=2, keepdims=True)
    scale = (m.astype(np.float64) / 32639).astype(np.float32)
    with np.errstate(divide='ignore', invalid='ignore'):
        ratio = np.where(scale != 0, (xs.astype(np.float64) / scale).astype(np.float32), np.float32(0))
    rounded = np.copysign(np.floor(np.abs(ratio.astype(np.float64)) + 0.5), ratio)
    return (scale.astype(np.float64) * rounded).reshape(batch, width)


def mm_fast(kind, data, x, batch, width, rows):
    """out [batch][rows] float64 of the 16-bit activation-block projection."""
    w, off = decode(kind, data, width, rows)
    xs = np.asarray(x, np.float32).astype(np.float64).reshape(batch, width)
    qx = quantize_activations(x, batch, width)
    return qx @ (w + off).T - xs @ off.T
