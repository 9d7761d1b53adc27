"""Closed-form long-context attention known-answer case.

TEST INFRASTRUCTURE ONLY.  Restates the reference's known-answer test
``tests/test_cuda.py:237-273``: keys are periodic with period 7 and values
with period 11, both exactly representable in fp16, so the softmax over any
context length has a closed form that needs no O(context) reference pass.

Layout (test_cuda.py:241-247): key row p (all 4 heads) is 64 zeros followed by
192 copies of ``(p%7 - 3)*0.25``; value row p, head h, dim d is
``(p%11-5)*0.125 + h*0.03125 + (d%4)*0.0625``.  The query is 64 zeros then
``(i%4+1)*0.03125`` for i < 192, with a zero gate (sigmoid 0.5) and unit
norms; new key rows are zero and new value rows are
``(t+1)*0.125 + h*0.03125 + (d%4)*0.0625``.
"""
import math

import numpy as np


def key_rows():
    return np.array([[0.0] * 64 + [(i - 3) * .25] * 192 for i in range(7)], np.float16)


def value_rows():
    return np.array([[(p - 5) * .125 + h * .03125 + (d % 4) * .0625
                      for h in range(4) for d in range(256)] for p in range(11)], np.float16)


def query():
    return [0.0] * 64 + [(i % 4 + 1) * .03125 for i in range(192)]


def caches(position, batch):
    """fp16 caches [position+batch, 4, 256] with the periodic prefix."""
    kr = np.repeat(key_rows()[:, None, :], 4, axis=1)            # [7,4,256]
    vr = value_rows().reshape(11, 4, 256)
    p = np.arange(position)
    kc = np.zeros((position + batch, 4, 256), np.float16)
    vc = np.zeros_like(kc)
    kc[:position] = kr[p % 7]
    vc[:position] = vr[p % 11]
    return kc, vc


def inputs(position, batch):
    kc, vc = caches(position, batch)
    q = query()
    q_gate = np.array((q + [0.0] * 256) * (batch * 24), np.float32)
    key = np.zeros(batch * 1024, np.float32)
    value = np.array([(t + 1) * .125 + h * .03125 + (d % 4) * .0625
                      for t in range(batch) for h in range(4) for d in range(256)], np.float32)
    norm = np.ones(256, np.float32)
    return dict(key_cache=kc, value_cache=vc, q_gate=q_gate, key=key, value=value,
                q_norm=norm, k_norm=norm, batch=batch, position=position, epsilon=1e-6)


def expected(position, batch):
    """Closed-form outputs [batch*24*256] (test_cuda.py:259-269)."""
    q = query()
    scale = 1 / math.sqrt(sum(x * x for x in q) / 256 + 1e-6)
    qsum = sum(q) * scale
    # Sum the exponentials per residue class of the 77-periodic pattern.
    p = np.arange(position)
    weights = np.exp(qsum * ((p % 7 - 3) * .25) / 16)
    total = float(weights.sum())
    numerator = float((weights * ((p % 11 - 5) * .125)).sum())
    out = []
    hd = np.array([(h // 6) * .03125 for h in range(24)])[:, None] + \
        np.array([(d % 4) * .0625 for d in range(256)])[None, :]
    for t in range(batch):
        total += 1
        numerator += (t + 1) * .125
        out.append(.5 * (numerator / total + hd))
    return np.concatenate([o.reshape(-1) for o in out])
