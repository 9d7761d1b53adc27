"""Vectorised float64 restatement of the reference hot-path oracle.

TEST INFRASTRUCTURE ONLY (see the package docstring).  Every function follows
``tests/cpu_reference.py`` of cristianku/redshift step for step; the line
citations below name the reference statement each block restates.  The
restatement changes the evaluation order only where numpy vectorises a sum
(float64 either way); the golden vectors in ``tests/golden/`` pin it to the
reference oracle's own outputs.
"""
import math

import numpy as np

ATTN_HEADS, KV_HEADS, HEAD_DIM = 24, 4, 256   # runtime.h:38 "24 query heads, 4 KV heads, 256"
ROPE_PAIRS = 32                                # cpu_reference.py:63 rotates pairs (i, i+32), i < 32
ROPE_BASE = 10000000.0                         # cpu_reference.py:64
SCORE_SCALE = 1.0 / 16.0                       # cpu_reference.py:81 "/ 16" == 1/sqrt(256)


def half(x):
    """Round to IEEE binary16 and back (cpu_reference.py:14-15, ``struct '<e'``)."""
    return np.asarray(x, dtype=np.float64).astype(np.float16).astype(np.float64)


def sigmoid(x):
    """cpu_reference.py:6-7."""
    return 1.0 / (1.0 + np.exp(-np.asarray(x, dtype=np.float64)))


def silu(x):
    """cpu_reference.py:10-11."""
    x = np.asarray(x, dtype=np.float64)
    return x * sigmoid(x)


def softplus(x):
    """``log1p(exp(x))`` exactly as cpu_reference.py:37 writes it."""
    return np.log1p(np.exp(np.asarray(x, dtype=np.float64)))


def _as64(x, shape=None):
    a = np.asarray(x)
    a = a.astype(np.float64) if a.dtype != np.float64 else a
    return a.reshape(shape) if shape is not None else a


# --------------------------------------------------------------------------
# Full attention (cpu_reference.py:55-89)
# --------------------------------------------------------------------------

def rope_angles(pos):
    """Angles of the partial rotary embedding at absolute position(s) ``pos``.

    cpu_reference.py:63-64: ``angle = pos * 10000000 ** (-i / 32)`` for i < 32.
    Returns shape ``pos.shape + (32,)``.
    """
    inv = np.array([ROPE_BASE ** (-i / ROPE_PAIRS) for i in range(ROPE_PAIRS)])
    return np.multiply.outer(np.asarray(pos, dtype=np.float64), inv)


def prepare_rows(rows, weight, pos, epsilon):
    """RMSNorm·gamma then partial RoPE on the last axis (cpu_reference.py:60-68).

    ``rows``: [..., 256]; ``pos``: broadcastable to rows.shape[:-1].
    """
    rows = _as64(rows)
    inv = 1.0 / np.sqrt(np.sum(rows * rows, axis=-1, keepdims=True) / HEAD_DIM + epsilon)
    out = rows * inv * _as64(weight)
    ang = rope_angles(np.broadcast_to(np.asarray(pos), rows.shape[:-1]))
    c, s = np.cos(ang), np.sin(ang)
    x, y = out[..., :ROPE_PAIRS].copy(), out[..., ROPE_PAIRS:2 * ROPE_PAIRS].copy()
    out[..., :ROPE_PAIRS] = x * c - y * s
    out[..., ROPE_PAIRS:2 * ROPE_PAIRS] = x * s + y * c
    return out


def attention(key_cache, value_cache, q_gate, key, value, q_norm, k_norm,
              batch, position, epsilon, return_lse=False):
    """Decode / verify / prefill attention of one full-attention layer.

    Restates ``cpu_reference.attention`` (cpu_reference.py:55-89): for every new
    token t the 4 key rows are RMSNorm+RoPE'd at position ``position+t`` and
    rounded to fp16 into the cache together with the fp16-rounded value rows
    (cpu_reference.py:70-74); each of the 24 query heads is prepared the same
    way (cpu_reference.py:76-77), attends causally over cache rows
    ``[0, position+t]`` of KV head ``h // 6`` with scale 1/16
    (cpu_reference.py:79-85) and is multiplied by ``sigmoid(gate)``
    (cpu_reference.py:86-88).

    Arguments mirror the reference: caches are any array-like of fp16 values
    of which the first ``position*1024`` entries are read; ``q_gate``
    [batch,24,512], ``key``/``value`` [batch,4,256], norms [256].

    Returns ``(out, kc, vc)``: out float64 [batch*24*256] (flattened like the
    reference), kc/vc float16 arrays [position+batch, 4, 256].  With
    ``return_lse`` also returns the natural-log LSE of the scaled scores
    [batch, 24] (not part of the reference's output; used by split-KV tests).
    """
    row = KV_HEADS * HEAD_DIM
    kc = np.empty((position + batch, KV_HEADS, HEAD_DIM), dtype=np.float16)
    vc = np.empty_like(kc)
    kc[:position] = np.asarray(key_cache, dtype=np.float16).reshape(-1)[:position * row] \
        .reshape(position, KV_HEADS, HEAD_DIM)
    vc[:position] = np.asarray(value_cache, dtype=np.float16).reshape(-1)[:position * row] \
        .reshape(position, KV_HEADS, HEAD_DIM)
    qg = _as64(q_gate).reshape(batch, ATTN_HEADS, 2 * HEAD_DIM)
    pos = position + np.arange(batch)
    # cpu_reference.py:70-74: append prepared keys and raw values, fp16-rounded.
    kc[position:] = prepare_rows(_as64(key).reshape(batch, KV_HEADS, HEAD_DIM),
                                 k_norm, pos[:, None], epsilon).astype(np.float16)
    vc[position:] = _as64(value).reshape(batch, KV_HEADS, HEAD_DIM).astype(np.float16)
    query = prepare_rows(qg[:, :, :HEAD_DIM], q_norm, pos[:, None], epsilon)  # [T,24,256]
    gate = qg[:, :, HEAD_DIM:]
    n = position + batch
    out = np.empty((batch, ATTN_HEADS, HEAD_DIM))
    lse = np.empty((batch, ATTN_HEADS))
    group = ATTN_HEADS // KV_HEADS
    causal = np.arange(n)[None, :] <= pos[:, None]          # token t sees p <= position+t
    for g in range(KV_HEADS):
        kg = kc[:, g, :].astype(np.float64)                  # [n,256]
        vg = vc[:, g, :].astype(np.float64)
        q = query[:, g * group:(g + 1) * group, :].reshape(batch * group, HEAD_DIM)
        scores = (q @ kg.T).reshape(batch, group, n) * SCORE_SCALE
        scores = np.where(causal[:, None, :], scores, -np.inf)
        peak = scores.max(axis=-1, keepdims=True)             # cpu_reference.py:82
        w = np.exp(scores - peak)                             # cpu_reference.py:83
        total = w.sum(axis=-1, keepdims=True)                 # cpu_reference.py:84
        pv = (w.reshape(batch * group, n) @ vg).reshape(batch, group, HEAD_DIM)
        out[:, g * group:(g + 1) * group, :] = pv / total
        lse[:, g * group:(g + 1) * group] = (peak + np.log(total))[..., 0]
    out = out * sigmoid(gate)                                 # cpu_reference.py:87-88
    if return_lse:
        return out.reshape(-1), kc, vc, lse
    return out.reshape(-1), kc, vc


def prefill_attention_core(q, k, v, position=0, scale=SCORE_SCALE, rows=None, heads=None):
    """Core causal GQA attention without norm/RoPE/gate (the prefill contraction).

    Semantics of cpu_reference.py:79-85 for a block of ``L`` query rows at
    absolute positions ``position..position+L-1``: query head h reads KV head
    h // 6 over keys ``[0, position+i]``.  ``q`` [L,24,256]; ``k``/``v``
    [position+L,4,256].  ``rows`` / ``heads`` restrict the evaluation to a
    subset of query rows / heads (the result then has those shapes).
    Returns ``(out [rows,heads,256], lse [rows,heads])`` in float64.
    """
    q = np.asarray(q)
    L = q.shape[0]
    rows = np.arange(L) if rows is None else np.asarray(rows)
    heads = list(range(ATTN_HEADS)) if heads is None else list(heads)
    n = position + int(rows.max()) + 1
    out = np.empty((len(rows), len(heads), HEAD_DIM))
    lse = np.empty((len(rows), len(heads)))
    group = ATTN_HEADS // KV_HEADS
    causal = np.arange(n)[None, :] <= (position + rows)[:, None]
    for col, h in enumerate(heads):
        g = h // group
        kg = np.asarray(k)[:n, g, :].astype(np.float64)
        vg = np.asarray(v)[:n, g, :].astype(np.float64)
        s = (q[rows, h, :].astype(np.float64) @ kg.T) * scale
        s = np.where(causal, s, -np.inf)
        peak = s.max(axis=-1, keepdims=True)
        w = np.exp(s - peak)
        total = w.sum(axis=-1, keepdims=True)
        out[:, col, :] = (w @ vg) / total
        lse[:, col] = (peak + np.log(total))[:, 0]
    return out, lse


# --------------------------------------------------------------------------
# Gated DeltaNet (cpu_reference.py:18-52)
# --------------------------------------------------------------------------

def delta(state, history, qkv, gate, alpha, beta, conv, decay, bias, norm,
          batch, key_heads, value_heads, dim, epsilon):
    """One gated-DeltaNet layer over ``batch`` tokens (cpu_reference.py:18-52).

    Per token (cpu_reference.py:22-50):
      * causal depthwise conv over [history(3 rows), raw] with 4 taps, SiLU
        (cpu_reference.py:24-26); the history shifts in the raw row
        (cpu_reference.py:27);
      * q, k of each key head are L2-normalised with +1e-6 inside the root and
        q additionally scaled by 1/sqrt(dim) (cpu_reference.py:28-33);
      * value head h uses key head ``h % key_heads`` (cpu_reference.py:35);
        decay ``a = exp(decay*log1p(exp(alpha+bias)))``, ``b = sigmoid(beta)``
        (cpu_reference.py:37-38);
      * every state row: scale by a, delta-rule residual, rank-1 update, then
        read out with q (cpu_reference.py:40-47);
      * gated RMSNorm of the head output with ``silu(gate)``
        (cpu_reference.py:48-50).

    Returns ``(out [batch*Hv*D], state [Hv*D*D], history [3*C])`` float64.
    """
    C = (2 * key_heads + value_heads) * dim
    S = _as64(state).reshape(value_heads, dim, dim).copy()
    hist = _as64(history).reshape(3, C).copy()
    raw_all = _as64(qkv).reshape(batch, C)
    z = _as64(gate).reshape(batch, value_heads, dim)
    al = _as64(alpha).reshape(batch, value_heads)
    be = _as64(beta).reshape(batch, value_heads)
    w = _as64(conv).reshape(C, 4)
    dec, bi, nw = _as64(decay), _as64(bias), _as64(norm)
    out = np.empty((batch, value_heads, dim))
    for t in range(batch):
        raw = raw_all[t]
        filt = silu(((w[:, 0] * hist[0] + w[:, 1] * hist[1]) + w[:, 2] * hist[2]) + w[:, 3] * raw)
        hist = np.concatenate([hist[1:], raw[None, :]], axis=0)
        qs = filt[:key_heads * dim].reshape(key_heads, dim)
        ks = filt[key_heads * dim:2 * key_heads * dim].reshape(key_heads, dim)
        vs = filt[2 * key_heads * dim:].reshape(value_heads, dim)
        qs = qs / np.sqrt(np.sum(qs * qs, axis=1, keepdims=True) + 1e-6) / math.sqrt(dim)
        ks = ks / np.sqrt(np.sum(ks * ks, axis=1, keepdims=True) + 1e-6)
        a = np.exp(dec * softplus(al[t] + bi))
        b = sigmoid(be[t])
        for h in range(value_heads):
            q, k = qs[h % key_heads], ks[h % key_heads]
            S[h] *= a[h]
            resid = b[h] * (vs[h] - S[h] @ k)
            S[h] += np.outer(resid, k)
            o = S[h] @ q
            scale = 1.0 / math.sqrt(float(np.sum(o * o)) / dim + epsilon)
            out[t, h] = o * scale * nw * silu(z[t, h])
    return out.reshape(-1), S.reshape(-1), hist.reshape(-1)



def delta_trace(history, qkv, alpha, beta, conv, decay, bias, batch, key_heads, value_heads, dim):
    """Transition trace of a recorded verify call, in the reference's layout.

    The reference copies the raw qkv rows into the trace before the layer
    (src/runtime.cu:389-390) and ``record_transition`` copies the prepared
    rows and gates after conv and gdn_prep (src/kernels.cu:356-360, called at
    src/kernels.cu:562): ``[8][C]`` raw rows, ``[8][C]`` prepared rows (q, k
    L2-normalised with +1e-6, q times 1/sqrt(dim); v filtered; conv + SiLU as
    cpu_reference.py:24-33), ``[8][Hv]`` decays ``exp(decay*softplus(alpha+bias))``
    and ``[8][Hv]`` betas ``sigmoid(beta)`` (cpu_reference.py:37-38).  Rows of
    tokens >= batch are left at zero.  Returns a float64 array of
    ``8 * (2C + 2Hv)`` values.
    """
    C = (2 * key_heads + value_heads) * dim
    hist = _as64(history).reshape(3, C).copy()
    raw_all = _as64(qkv).reshape(batch, C)
    al = _as64(alpha).reshape(batch, value_heads)
    be = _as64(beta).reshape(batch, value_heads)
    w = _as64(conv).reshape(C, 4)
    dec, bi = _as64(decay), _as64(bias)
    trace = np.zeros(8 * (2 * C + 2 * value_heads))
    raw_t = trace[:8 * C].reshape(8, C)
    prep_t = trace[8 * C:16 * C].reshape(8, C)
    a_t = trace[16 * C:16 * C + 8 * value_heads].reshape(8, value_heads)
    b_t = trace[16 * C + 8 * value_heads:].reshape(8, value_heads)
    kd = key_heads * dim
    for t in range(batch):
        raw = raw_all[t]
        filt = silu(((w[:, 0] * hist[0] + w[:, 1] * hist[1]) + w[:, 2] * hist[2]) + w[:, 3] * raw)
        hist = np.concatenate([hist[1:], raw[None, :]], axis=0)
        qs = filt[:kd].reshape(key_heads, dim)
        ks = filt[kd:2 * kd].reshape(key_heads, dim)
        raw_t[t] = raw
        prep_t[t, :kd] = (qs / np.sqrt(np.sum(qs * qs, axis=1, keepdims=True) + 1e-6) / math.sqrt(dim)).reshape(-1)
        prep_t[t, kd:2 * kd] = (ks / np.sqrt(np.sum(ks * ks, axis=1, keepdims=True) + 1e-6)).reshape(-1)
        prep_t[t, 2 * kd:] = filt[2 * kd:]
        a_t[t] = np.exp(dec * softplus(al[t] + bi))
        b_t[t] = sigmoid(be[t])
    return trace


def delta_commit(saved_state, saved_history, trace, accepted, key_heads, value_heads, dim):
    """State and conv history after committing ``accepted`` tokens of a
    recorded verify (src/runtime.cu:432-454).

    The start state and history are copied back, ``commit_history`` shifts the
    accepted raw rows into the history window (src/kernels.cu:362-369), and
    ``gdn_scan`` replays the accepted tokens' prepared rows and gates on the
    state (src/kernels.cu:567-574; the row update of cpu_reference.py:40-45:
    S *= a; S += outer(b (v - S k), k)).  Returns ``(state, history)`` float64.
    """
    C = (2 * key_heads + value_heads) * dim
    S = _as64(saved_state).reshape(value_heads, dim, dim).copy()
    hist = _as64(saved_history).reshape(3, C).copy()
    tr = _as64(trace)
    raw_t = tr[:8 * C].reshape(8, C)
    prep_t = tr[8 * C:16 * C].reshape(8, C)
    a_t = tr[16 * C:16 * C + 8 * value_heads].reshape(8, value_heads)
    b_t = tr[16 * C + 8 * value_heads:].reshape(8, value_heads)
    kd = key_heads * dim
    for t in range(accepted):
        hist = np.concatenate([hist[1:], raw_t[t][None, :]], axis=0)
        ks = prep_t[t, kd:2 * kd].reshape(key_heads, dim)
        vs = prep_t[t, 2 * kd:].reshape(value_heads, dim)
        for h in range(value_heads):
            k = ks[h % key_heads]
            S[h] *= a_t[t, h]
            S[h] += np.outer(b_t[t, h] * (vs[h] - S[h] @ k), k)
    return S.reshape(-1), hist.reshape(-1)

def delta_core(state, q, k, v, log_decay, beta):
    """The bare delta-rule recurrence on prepared inputs (cpu_reference.py:35-47).

    ``state`` [Hv,D,D] (row = value dim, column = key dim); ``q``/``k``
    [T,Hk,D] already normalised (q includes 1/sqrt(D)); ``v`` [T,Hv,D];
    ``log_decay`` [T,Hv] (so a = exp(log_decay)); ``beta`` [T,Hv] already
    passed through the sigmoid.  Value head h uses key head h % Hk.

    Returns ``(out [T,Hv,D] (state readout before the gated norm),
    state [Hv,D,D])`` in float64.
    """
    S = _as64(state).copy()
    q, k, v = _as64(q), _as64(k), _as64(v)
    g, b = _as64(log_decay), _as64(beta)
    T, Hk = q.shape[0], q.shape[1]
    Hv = v.shape[1]
    kidx = np.arange(Hv) % Hk
    out = np.empty((T, Hv, S.shape[1]))
    for t in range(T):
        kt, qt = k[t, kidx], q[t, kidx]                          # [Hv,D]
        S *= np.exp(g[t])[:, None, None]
        resid = b[t][:, None] * (v[t] - np.einsum('hvk,hk->hv', S, kt))
        S += resid[:, :, None] * kt[:, None, :]
        out[t] = np.einsum('hvk,hk->hv', S, qt)
    return out, S


def prepare_delta_inputs(q_raw, k_raw, alpha, beta_raw, decay=-1.0, bias=0.0):
    """gdn prep on raw (post-conv) inputs, as cpu_reference.py:31-38 does it.

    q,k [T,Hk,D] -> L2-normalised (q also / sqrt(D)); returns
    ``(q, k, log_decay, beta)`` with ``log_decay = decay*softplus(alpha+bias)``.
    """
    q_raw, k_raw = _as64(q_raw), _as64(k_raw)
    D = q_raw.shape[-1]
    q = q_raw / np.sqrt(np.sum(q_raw ** 2, axis=-1, keepdims=True) + 1e-6) / math.sqrt(D)
    k = k_raw / np.sqrt(np.sum(k_raw ** 2, axis=-1, keepdims=True) + 1e-6)
    g = _as64(decay) * softplus(_as64(alpha) + _as64(bias))
    return q, k, g, sigmoid(beta_raw)
