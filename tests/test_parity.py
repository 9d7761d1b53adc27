"""Parity of the CUDA path with the CPU oracle on the seeded benchmark
configurations (0-4), through the C ABI.

Tolerances: the north-star bounds (attention max-abs <= 2e-3, DeltaNet state
relative <= 1e-3) and, where the reference defines one, its own scaled
criterion |a-e| <= tol*(1+|e|)."""
from pathlib import Path

import numpy as np
import pytest

import oracle
from oracle import inputs as I
from tests.test_cuda import close, run_attention, run_delta

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / 'golden'
ATTN_MAX_ABS = 2e-3
DELTA_STATE_REL = 1e-3


def rel_err(a, e):
    a, e = np.asarray(a, np.float64).reshape(-1), np.asarray(e, np.float64).reshape(-1)
    return np.abs(a - e).max() / max(np.abs(e).max(), 1e-30)


# ------------------------------------------------------------------ config 0
def test_config0_attention_against_reference_golden(lib):
    c = I.attention_layer(batch=8, position=128)
    g = np.load(GOLDEN / 'attention_cfg0.npz')
    out, kc, vc = run_attention(lib, c, kc=c['key_cache'].copy(), vc=c['value_cache'].copy())
    assert np.abs(out - g['out']).max() <= ATTN_MAX_ABS
    close(out, g['out'], 3e-4)
    close(kc[128:].reshape(-1).astype(np.float64), g['new_k'], 2e-3)
    assert np.array_equal(vc[128:].reshape(-1).astype(np.float64), g['new_v'])


@pytest.mark.parametrize('name', ['attention_edge', 'attention_single'])
def test_attention_golden_edges(lib, name):
    g = np.load(GOLDEN / f'{name}.npz')
    c = {'attention_edge': lambda: I.attention_layer(batch=8, position=250, seed=1100),
         'attention_single': lambda: I.attention_layer(batch=1, position=0, seed=1101)}[name]()
    out, _, _ = run_attention(lib, c, kc=c['key_cache'].copy(), vc=c['value_cache'].copy())
    close(out, g['out'], 3e-4)


# ------------------------------------------------------------------ config 1
def test_config1_delta_against_reference_golden(lib):
    c = I.delta_layer(batch=8)
    g = np.load(GOLDEN / 'delta_cfg1.npz')
    out, st, hi = run_delta(lib, c)
    close(out, g['out'])
    st = st.reshape(48, 128, 128)[g['state_heads']]
    assert rel_err(st, g['state']) <= DELTA_STATE_REL
    close(st, g['state'])
    np.testing.assert_array_equal(hi.reshape(-1), g['history'])


def test_config1_full_state_against_oracle(lib):
    c = I.delta_layer(batch=8)
    exp_out, exp_state, exp_hist = oracle.delta(**c)
    out, st, hi = run_delta(lib, c)
    assert rel_err(st, exp_state) <= DELTA_STATE_REL
    close(st, exp_state)
    close(out, exp_out)


def test_delta_golden_small(lib):
    g = np.load(GOLDEN / 'delta_small_t1.npz')
    c = I.delta_layer(batch=1, seed=1102, key_heads=4, value_heads=12, dim=128, state_std=0.05)
    out, st, _ = run_delta(lib, c)
    close(out, g['out'])
    close(st.reshape(12, 128, 128)[g['state_heads']], g['state'])


# ------------------------------------------------------------------ config 2
@pytest.mark.parametrize('context', [32768, 139264])
def test_config2_long_context_attention(lib, context):
    c = I.attention_layer(batch=8, position=context - 8, seed=1002)
    exp_out, exp_k, _ = oracle.attention(**c)
    out, kc, vc = run_attention(lib, c, kc=c['key_cache'].copy(), vc=c['value_cache'].copy())
    assert np.abs(out - exp_out).max() <= ATTN_MAX_ABS
    close(out, exp_out, 3e-4)
    close(kc[-8:].astype(np.float64), exp_k[-8:].astype(np.float64), 2e-3)


@pytest.mark.parametrize('position,batch', [(0, 8), (63, 1), (64, 8), (1000, 5), (2041, 8), (2047, 1)])
def test_attention_tile_edges(lib, position, batch):
    c = I.attention_layer(batch=batch, position=position, seed=2000 + position)
    exp_out, _, _ = oracle.attention(**c)
    out, _, _ = run_attention(lib, c, kc=c['key_cache'].copy(), vc=c['value_cache'].copy())
    close(out, exp_out, 3e-4)


# ------------------------------------------------------------------ prefill (ABI level)
@pytest.mark.parametrize('position,batch', [(0, 9), (100, 21), (37, 300), (0, 1000), (4000, 130), (127, 64)])
def test_attention_prefill_abi(lib, position, batch):
    c = I.attention_layer(batch=batch, position=position, seed=3000 + batch)
    exp_out, exp_k, exp_v = oracle.attention(**c)
    out, kc, vc = run_attention(lib, c, kc=c['key_cache'].copy(), vc=c['value_cache'].copy(),
                                fn=lib.qv_test_attention_prefill)
    assert np.abs(out - exp_out).max() <= ATTN_MAX_ABS
    close(out, exp_out, 3e-4)
    assert np.array_equal(vc.astype(np.float64), exp_v.astype(np.float64))


def test_delta_prefill_abi(lib):
    c = I.delta_layer(batch=100, seed=3100, key_heads=4, value_heads=12, dim=128, state_std=0.05)
    exp_out, exp_state, exp_hist = oracle.delta(**c)
    out = np.zeros(100 * 12 * 128, np.float32)
    st, hi = c['state'].copy(), c['history'].copy()
    f = lambda k: np.ascontiguousarray(np.asarray(c[k], np.float32).reshape(-1))  # noqa: E731
    from tests.test_cuda import ptr
    a = {k: f(k) for k in ('qkv', 'gate', 'alpha', 'beta', 'conv', 'decay', 'bias', 'norm')}
    rc = lib.qv_test_delta_prefill(ptr(out), ptr(st), ptr(hi), ptr(a['qkv']), ptr(a['gate']), ptr(a['alpha']),
                                   ptr(a['beta']), ptr(a['conv']), ptr(a['decay']), ptr(a['bias']),
                                   ptr(a['norm']), 100, 4, 12, 128, 1e-6)
    assert rc == 0, lib.qv_error()
    close(out, exp_out, 1e-4)
    assert rel_err(st, exp_state) <= DELTA_STATE_REL
    close(hi, exp_hist, 0)


# ------------------------------------------------------------------ config 3 (core prefill)
def _prefill_gpu(hot, q, k, v, position=0):
    import torch
    L = q.shape[0]
    dev = torch.device('cuda')
    qt = torch.from_numpy(q.view(np.uint16).copy()).to(dev).view(torch.float16)
    kt = torch.from_numpy(k.view(np.uint16).copy()).to(dev).view(torch.float16)
    vt = torch.from_numpy(v.view(np.uint16).copy()).to(dev).view(torch.float16)
    out = torch.empty((L, 24, 256), dtype=torch.float32, device=dev)
    lse = torch.empty((L, 24), dtype=torch.float32, device=dev)
    hot.prefill_attention(out, qt, kt, vt, L, position, lse=lse)
    assert hot.status() == 0
    return out.cpu().numpy(), lse.cpu().numpy()


def test_config3_prefill_sampled_rows(hot):
    """Config 3 (4,096-token causal prefill) against the oracle: every query head on 49 sampled rows
    (tile edges and random rows), and for every KV head one full 128-row query tile of all six query
    heads that read it (tiles 31, 0, 16 and 5: the longest, the shortest and two in between)."""
    q, k, v = I.prefill_attention(length=4096)
    out, lse = _prefill_gpu(hot, q, k, v)
    rng = np.random.default_rng(99)
    rows = np.unique(np.concatenate([[0, 1, 63, 64, 127, 128, 2047, 4094, 4095], rng.integers(0, 4096, 40)]))
    exp, exp_lse = oracle.prefill_attention_core(q, k, v, rows=rows)
    # fp16 probabilities (FAST mode): the north-star bound, max-abs <= 2e-3.
    assert np.abs(out[rows] - exp).max() <= ATTN_MAX_ABS
    np.testing.assert_allclose(lse[rows], exp_lse, atol=1e-3, rtol=0)
    for kv_head, tile in enumerate((31, 0, 16, 5)):
        tile_rows = np.arange(128 * tile, 128 * tile + 128)
        heads = list(range(6 * kv_head, 6 * kv_head + 6))
        exp, exp_lse = oracle.prefill_attention_core(q, k, v, rows=tile_rows, heads=heads)
        assert np.abs(out[tile_rows][:, heads] - exp).max() <= ATTN_MAX_ABS, (kv_head, tile)
        np.testing.assert_allclose(lse[tile_rows][:, heads], exp_lse, atol=1e-3, rtol=0)


@pytest.mark.parametrize('L,position', [(1000, 0), (200, 77), (1, 0), (129, 5), (64, 3000)])
def test_prefill_core_full(hot, L, position):
    q, k, v = I.prefill_attention(length=L + position, seed=1200 + L)
    q = q[position:]
    out, lse = _prefill_gpu(hot, q, k, v, position)
    exp, exp_lse = oracle.prefill_attention_core(q, k, v, position=position)
    assert np.abs(out - exp).max() <= ATTN_MAX_ABS
    np.testing.assert_allclose(lse, exp_lse, atol=1e-3, rtol=0)


# ------------------------------------------------------------------ config 4 (core DeltaNet)
def _delta_core_gpu(hot, c, state):
    import torch
    dev = torch.device('cuda')
    L, hk, d = c['q'].shape
    hv = c['v'].shape[1]
    t16 = lambda a: torch.from_numpy(a.view(np.uint16).copy()).to(dev).view(torch.float16)  # noqa: E731
    t32 = lambda a: torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(dev)  # noqa: E731
    st = t32(state)
    out = torch.empty((L, hv, d), dtype=torch.float32, device=dev)
    hot.delta_core(out, st, t16(c['q']), t16(c['k']), t16(c['v']), t32(c['alpha']), t32(c['beta']),
                   t32(np.full(hv, -1.0)), t32(np.zeros(hv)), L, hk, hv, d)
    assert hot.status() == 0
    return out.cpu().numpy(), st.cpu().numpy()


def _delta_chunked_gpu(hot, c, state):
    import torch
    dev = torch.device('cuda')
    L, hk, d = c['q'].shape
    hv = c['v'].shape[1]
    t16 = lambda a: torch.from_numpy(a.view(np.uint16).copy()).to(dev).view(torch.float16)  # noqa: E731
    t32 = lambda a: torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(dev)  # noqa: E731
    st = t32(state)
    out = torch.empty((L, hv, d), dtype=torch.float32, device=dev)
    hot.delta_chunked(out, st, t16(c['q']), t16(c['k']), t16(c['v']), t32(c['alpha']), t32(c['beta']),
                      t32(np.full(hv, -1.0)), t32(np.zeros(hv)), L, hk, hv, d)
    assert hot.status() == 0
    return out.cpu().numpy(), st.cpu().numpy()


@pytest.mark.parametrize('length,with_state', [(1, False), (64, False), (65, True), (200, True), (512, False)])
def test_chunked_delta_against_recurrence(hot, length, with_state):
    """qv_delta_chunked (chunks of 64 on tensor cores) == the fp64 token recurrence:
    a single token, exactly one chunk, a ragged last chunk, a non-zero initial state."""
    c = I.delta_prefill(length=length, seed=7000 + length)
    q, k, g, b = oracle.hotpath.prepare_delta_inputs(c['q'], c['k'], c['alpha'], c['beta'])
    s0 = (np.random.default_rng(length).standard_normal((48, 128, 128)) * 0.02 if with_state
          else np.zeros((48, 128, 128)))
    exp_out, exp_state = oracle.delta_core(s0, q, k, c['v'], g, b)
    out, st = _delta_chunked_gpu(hot, c, s0.astype(np.float32))
    assert rel_err(st, exp_state) <= DELTA_STATE_REL
    close(out, exp_out, 1e-4)


def test_config4_chunked_prefill_then_verify(hot):
    """Config 4 end to end: a 4,096-token chunked prefill from a zero state, its state handed to 8
    recurrent verify tokens (qv_delta_core), every value head checked against the token-by-token
    fp64 CPU recurrence over all 4,104 tokens: the prefill outputs and state, then the verify
    outputs and the final state."""
    L = 4096
    c = I.delta_prefill(length=L + 8)
    pre = {k: v[:L] for k, v in c.items()}
    ver = {k: v[L:] for k, v in c.items()}
    out_c, st_c = _delta_chunked_gpu(hot, pre, np.zeros((48, 128, 128), np.float32))
    out_v, st_v = _delta_core_gpu(hot, ver, st_c)
    q, k, g, b = oracle.hotpath.prepare_delta_inputs(c['q'], c['k'], c['alpha'], c['beta'])
    exp_pre, exp_state = oracle.delta_core(np.zeros((48, 128, 128)), q[:L], k[:L], c['v'][:L], g[:L], b[:L])
    exp_ver, exp_final = oracle.delta_core(exp_state, q[L:], k[L:], c['v'][L:], g[L:], b[L:])
    for h in range(48):          # the north-star bound on every head's state, after the prefill and the verify
        assert rel_err(st_c[h], exp_state[h]) <= DELTA_STATE_REL, h
        assert rel_err(st_v[h], exp_final[h]) <= DELTA_STATE_REL, h
    close(out_c, exp_pre, 1e-4)
    close(out_v, exp_ver, 1e-4)


def test_config4_delta_core_against_recurrence(hot):
    c = I.delta_prefill(length=512)
    q, k, g, b = oracle.hotpath.prepare_delta_inputs(c['q'], c['k'], c['alpha'], c['beta'])
    exp_out, exp_state = oracle.delta_core(np.zeros((48, 128, 128)), q, k, c['v'], g, b)
    out, st = _delta_core_gpu(hot, c, np.zeros((48, 128, 128), np.float32))
    assert rel_err(st, exp_state) <= DELTA_STATE_REL
    close(out, exp_out, 1e-4)


# ------------------------------------------------------------------ multi-GPU kernels on one GPU
@pytest.mark.parametrize('shards,position,batch', [(3, 5000, 8), (2, 139256, 8), (4, 100, 1), (2, 64, 3)])
def test_sequence_shards_merge_to_the_full_layer(hot, shards, position, batch):
    """qv_attention_shard over every shard of the plan + qv_attention_merge == qv_attention."""
    import torch
    from redshift_b200.sharding import plan, shard_capacity
    c = I.attention_layer(batch=batch, position=position, seed=4000 + shards)
    dev = torch.device('cuda')
    t = lambda k: torch.from_numpy(np.ascontiguousarray(np.asarray(c[k], np.float32))).to(dev)  # noqa: E731
    qg, key, value, qn, kn = t('q_gate'), t('key'), t('value'), t('q_norm'), t('k_norm')
    parts = torch.empty((shards, batch, 24, 256), device=dev)
    lses = torch.empty((shards, batch, 24), device=dev)
    new_rows = None
    for g in range(shards):
        s = plan(position, shards, g, batch)
        kc = torch.zeros((shard_capacity(s, batch), 4, 256), dtype=torch.float16, device=dev)
        vc = torch.zeros_like(kc)
        kc[:s.rows] = torch.from_numpy(c['key_cache'][s.begin:s.begin + s.rows]).to(dev)
        vc[:s.rows] = torch.from_numpy(c['value_cache'][s.begin:s.begin + s.rows]).to(dev)
        hot.attention_shard(parts[g], lses[g], kc, vc, s.begin, s.rows, qg, key, value, qn, kn, batch, position)
        if s.appends:
            new_rows = (kc[s.rows:].cpu().numpy(), vc[s.rows:].cpu().numpy())
    out = torch.empty((batch, 24, 256), device=dev)
    hot.attention_merge(out, parts, lses, shards, batch, qg)
    assert hot.status() == 0
    exp_out, exp_k, exp_v = oracle.attention(**c)
    got = out.cpu().numpy().reshape(-1)
    assert np.abs(got - exp_out).max() <= ATTN_MAX_ABS
    close(got, exp_out, 3e-4)
    close(new_rows[0].astype(np.float64), exp_k[position:].astype(np.float64), 2e-3)
    assert np.array_equal(new_rows[1], exp_v[position:])


def test_peer_exchange_with_a_single_rank_equals_the_layer(hot):
    """qv_attention_shard_exchange with world=1 (the buffer is this GPU's own) == qv_attention."""
    import torch
    c = I.attention_layer(batch=8, position=3000, seed=4100)
    dev = torch.device('cuda')
    t = lambda k: torch.from_numpy(np.ascontiguousarray(np.asarray(c[k], np.float32))).to(dev)  # noqa: E731
    kc = torch.from_numpy(c['key_cache']).to(dev)
    vc = torch.from_numpy(c['value_cache']).to(dev)
    nwords = hot.lib.qv_attention_exchange_bytes(1) // 4
    buf = torch.zeros(nwords, dtype=torch.float32, device=dev)
    peers = torch.tensor([buf.data_ptr()], dtype=torch.int64, device=dev)
    exp_out, _, _ = oracle.attention(**c)
    for seq in range(3):             # consecutive calls count up
        out = torch.empty((8, 24, 256), device=dev)
        hot.attention_shard_exchange(out, kc, vc, 0, 3000, t('q_gate'), t('key'), t('value'), t('q_norm'),
                                     t('k_norm'), 8, 3000, peers, 1, 0, seq)
        assert hot.status() == 0
        close(out.cpu().numpy().reshape(-1), exp_out, 3e-4)
    flags = buf[nwords - 2 * 240:].view(torch.int32)
    assert int(flags.abs().sum()) == 0, 'consumers reset every flag'


def _plant_peer_words(buf, part, lse, world, peer, seq):
    """Write `peer`'s (partial, LSE) of every row into a receive buffer as the exchange kernel's
    tagged 64-bit words (low half: the float's bits; high half: 0x51000000 | (seq & 0xFFFFFF)),
    at buffer slot seq & 1.  Buffer layout: [2 slots][world][240 rows][264 words], row = t*24 + h,
    words 0..255 the partial, word 256 the LSE."""
    import torch
    rows, words = 240, 264
    tag = np.uint64(0x51000000 | (seq & 0xFFFFFF)) << np.uint64(32)
    batch = part.shape[0]
    img = np.zeros((batch * 24, words), np.uint64)
    img[:, :256] = part.reshape(batch * 24, 256).view(np.uint32).astype(np.uint64) | tag
    img[:, 256] = lse.reshape(-1).view(np.uint32).astype(np.uint64) | tag
    view = buf.view(2, world, rows, words)
    view[seq & 1, peer, :batch * 24] = torch.from_numpy(img.view(np.int64)).to(buf.device)


def test_peer_exchange_merges_a_planted_peer_partial(hot):
    """The two-rank exchange on one GPU: rank 1's (partial, LSE) are planted in rank 0's receive
    buffer as the words rank 1 would store, so rank 0's kernel finds them without waiting on
    another kernel.  Rank 0's call must merge them into the full layer's output and zero the words
    it read.  A planted word with the tag of two calls back is refused: the bounded wait gives up
    and qv_status reports the timeout, and the next call on the same buffers is correct again."""
    import torch
    from redshift_b200.sharding import plan, shard_capacity
    batch, position, world = 8, 3000, 2
    c = I.attention_layer(batch=batch, position=position, seed=4200)
    dev = torch.device('cuda')
    t = lambda k: torch.from_numpy(np.ascontiguousarray(np.asarray(c[k], np.float32))).to(dev)  # noqa: E731
    args = (t('q_gate'), t('key'), t('value'), t('q_norm'), t('k_norm'))
    caches = []
    for rank in range(world):
        s = plan(position, world, rank, batch)
        kc = torch.zeros((shard_capacity(s, batch), 4, 256), dtype=torch.float16, device=dev)
        vc = torch.zeros_like(kc)
        kc[:s.rows] = torch.from_numpy(c['key_cache'][s.begin:s.begin + s.rows]).to(dev)
        vc[:s.rows] = torch.from_numpy(c['value_cache'][s.begin:s.begin + s.rows]).to(dev)
        caches.append((s, kc, vc))
    s1, kc1, vc1 = caches[1]
    part1 = torch.empty((batch, 24, 256), device=dev)
    lse1 = torch.empty((batch, 24), device=dev)
    hot.attention_shard(part1, lse1, kc1, vc1, s1.begin, s1.rows, *args, batch, position)
    part1, lse1 = part1.cpu().numpy(), lse1.cpu().numpy()
    nwords = hot.lib.qv_attention_exchange_bytes(world) // 8
    bufs = [torch.zeros(nwords, dtype=torch.int64, device=dev) for _ in range(world)]
    peers = torch.tensor([b.data_ptr() for b in bufs], dtype=torch.int64, device=dev)
    s0, kc0, vc0 = caches[0]
    exp_out, _, _ = oracle.attention(**c)

    def call(seq):
        out = torch.full((batch, 24, 256), float('nan'), device=dev)
        hot.attention_shard_exchange(out, kc0, vc0, s0.begin, s0.rows, *args, batch, position, peers, world, 0,
                                     seq)
        return out, hot.status()

    for seq in (5, 6):
        _plant_peer_words(bufs[0], part1, lse1, world, 1, seq)
        out, status = call(seq)
        assert status == 0
        got = out.cpu().numpy().reshape(-1)
        assert np.abs(got - exp_out).max() <= ATTN_MAX_ABS
        close(got, exp_out, 3e-4)
        assert int(bufs[0].view(2, world, 240, 264)[seq & 1, 1].abs().sum()) == 0, 'read words are zeroed'
    # a leftover word from call 5 in slot 1 (two calls before 7) must not be taken for call 7's data
    _plant_peer_words(bufs[0], part1, lse1, world, 1, 5)
    _, status = call(7)
    assert status == 1, 'the stale words are refused and the bounded wait reports a timeout'
    _plant_peer_words(bufs[0], part1, lse1, world, 1, 8)
    out, status = call(8)
    assert status == 0
    close(out.cpu().numpy().reshape(-1), exp_out, 3e-4)


# ------------------------------------------------------------------ DeltaNet layer prefill (chunked)
def _layer_prefill_case(length, seed, state_std):
    """Reference-semantics layer inputs with random conv taps and a random conv history."""
    c = I.delta_layer(batch=length, seed=seed, state_std=state_std)
    rng = np.random.default_rng(seed + 1)
    c['conv'] = (rng.standard_normal(c['conv'].shape) * 0.5).astype(np.float32)
    c['history'] = rng.standard_normal(c['history'].shape).astype(np.float32)
    return c


@pytest.mark.parametrize('length,seed,state_std', [(4096, 8000, 0.0), (1000, 8001, 0.02), (70, 8002, 0.02)])
def test_delta_layer_prefill_chunked(hot, length, seed, state_std):
    """qv_delta_prefill (conv + SiLU, norms, chunked delta rule on tensor cores, gated RMSNorm) against
    the float64 restatement of the reference layer (cpu_reference.py:18-52) over all 48 value heads.

    Bounds: the state within the north-star 1e-3 relative, per head; the conv history bit-exact; the
    outputs within 1e-2 at the 99.99th percentile and 6e-2 at the maximum (absolute).  The output
    bounds are the chunked form's: the filtered q, k, v and the state images enter the tensor cores
    as fp16 (about 5e-4 relative each), and the gated RMSNorm divides by the row's RMS, so rows of
    small norm carry that error as an absolute one of up to a few 1e-2 on O(1) outputs (measured:
    p99.99 4.4e-3, max 3.1e-2 at 4096 tokens).  qv_delta is the exact path."""
    import torch
    from oracle import native
    c = _layer_prefill_case(length, seed, state_std)
    exp_out, exp_state, exp_hist = native.delta(**c)
    dev = torch.device('cuda')
    t32 = lambda a: torch.from_numpy(np.ascontiguousarray(np.asarray(a, np.float32))).to(dev)  # noqa: E731
    st, hi = t32(c['state']), t32(c['history'])
    out = torch.empty((length, 48, 128), device=dev)
    hot.delta_prefill(out, st, hi, t32(c['qkv']), t32(c['gate']), t32(c['alpha']), t32(c['beta']), t32(c['conv']),
                      t32(c['decay']), t32(c['bias']), t32(c['norm']), length, 16, 48, 128)
    assert hot.status() == 0
    st = st.cpu().numpy().reshape(48, 128, 128)
    exp_state = exp_state.reshape(48, 128, 128)
    for h in range(48):
        assert rel_err(st[h], exp_state[h]) <= DELTA_STATE_REL, h
    err = np.abs(out.cpu().numpy().reshape(-1) - exp_out)
    assert np.quantile(err, 0.9999) <= 1e-2
    assert err.max() <= 6e-2
    assert np.array_equal(hi.cpu().numpy().reshape(-1).astype(np.float64), exp_hist)
