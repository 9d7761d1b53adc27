"""The multi-GPU split-KV plan and its collective choreography, on CPU.

Two (and three) ``gloo`` ranks run ``ShardedAttention`` with a numpy stand-in
for the two library calls; the merged output must equal the single-device
oracle.  The stand-in restates what the CUDA entry points compute (shard
partial + LSE; LSE-weighted merge), so this covers the host-side plan, the
append placement and the all-gather/merge order without a GPU."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
from oracle import inputs as I
from redshift_b200.sharding import ShardedAttention, plan, shard_capacity


def test_plan_covers_every_position_once():
    for world in (1, 2, 3, 4, 8):
        for position in (0, 1, 7, 64, 1000, 139256):
            shards = [plan(position, world, r) for r in range(world)]
            assert shards[0].begin == 0
            assert sum(s.rows for s in shards) == position
            for a, b in zip(shards, shards[1:]):
                assert a.begin + a.rows == b.begin
            assert [s.appends for s in shards] == [False] * (world - 1) + [True]
            assert shard_capacity(shards[-1], 8) == shards[-1].rows + 8


def test_plan_rejects_bad_arguments():
    with pytest.raises(ValueError):
        plan(10, 0, 0)
    with pytest.raises(ValueError):
        plan(10, 2, 2)
    with pytest.raises(ValueError):
        plan(-1, 2, 0)


class NumpyShardHot:
    """numpy stand-in for HotPath.attention_shard / attention_merge."""

    def attention_shard(self, part, lse, kc, vc, begin, rows, q_gate, key, value, q_norm, k_norm,
                        batch, position, epsilon, workspace=None):
        from oracle.hotpath import prepare_rows
        appends = begin + rows == position
        kcn = kc.numpy()
        vcn = vc.numpy()
        pos = position + np.arange(batch)
        if appends:
            kcn[rows:rows + batch] = prepare_rows(key.numpy().astype(np.float64), k_norm.numpy(),
                                                  pos[:, None], epsilon).astype(np.float16)
            vcn[rows:rows + batch] = value.numpy().astype(np.float16)
        n = rows + (batch if appends else 0)
        q = prepare_rows(q_gate.numpy()[:, :, :256].astype(np.float64), q_norm.numpy(), pos[:, None], epsilon)
        absolute = begin + np.arange(n)
        for h in range(24):
            K = kcn[:n, h // 6].astype(np.float64)
            V = vcn[:n, h // 6].astype(np.float64)
            s = q[:, h] @ K.T / 16
            s = np.where(absolute[None, :] <= pos[:, None], s, -np.inf)
            m = s.max(1, keepdims=True)
            ok = np.isfinite(m[:, 0])
            w = np.where(ok[:, None], np.exp(s - np.where(ok[:, None], m, 0)), 0)
            tot = w.sum(1)
            o = np.where(ok[:, None], (w @ V) / np.where(ok, tot, 1)[:, None], 0)
            part.numpy()[:, h] = o
            lse.numpy()[:, h] = np.where(ok, m[:, 0] + np.log(np.where(ok, tot, 1)), -np.inf)

    def attention_merge(self, out, parts, lses, shards, batch, q_gate):
        L = lses.numpy().astype(np.float64)                     # [G,T,24]
        M = L.max(0)
        w = np.exp(L - M)
        o = (w[..., None] * parts.numpy()).sum(0) / w.sum(0)[..., None]
        out.numpy()[:] = o * oracle.sigmoid(q_gate.numpy()[:, :, 256:])


def _worker(rank, world, port, position, batch, result):
    os.environ.update(MASTER_ADDR='127.0.0.1', MASTER_PORT=str(port))
    import datetime
    dist.init_process_group('gloo', rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        c = I.attention_layer(batch=batch, position=position, seed=77)
        shard = plan(position, world, rank, batch)
        cap = shard_capacity(shard, batch)
        kc = torch.zeros((cap, 4, 256), dtype=torch.float16)
        vc = torch.zeros_like(kc)
        kc[:shard.rows] = torch.from_numpy(c['key_cache'][shard.begin:shard.begin + shard.rows])
        vc[:shard.rows] = torch.from_numpy(c['value_cache'][shard.begin:shard.begin + shard.rows])
        t = lambda k: torch.from_numpy(np.asarray(c[k], np.float32).copy())  # noqa: E731
        out = torch.zeros((batch, 24, 256))
        part, lse = torch.zeros((batch, 24, 256)), torch.zeros((batch, 24))
        gp, gl = torch.zeros((world, batch, 24, 256)), torch.zeros((world, batch, 24))
        ShardedAttention(NumpyShardHot(), dist, shard)(
            out, kc, vc, t('q_gate'), t('key'), t('value'), t('q_norm'), t('k_norm'), batch, position,
            part, lse, gp, gl)
        if rank == 0:
            result.put(out.numpy().copy())
        if shard.appends:
            result.put(('kc', kc[shard.rows:].numpy().copy()))
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(('127.0.0.1', 0))
        return s.getsockname()[1]


@pytest.mark.parametrize('world,position,batch', [(2, 300, 8), (3, 130, 5), (2, 5, 3)])
def test_sharded_attention_matches_single_device_oracle(world, position, batch):
    ctx = mp.get_context('spawn')
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, position, batch, q)) for r in range(world)]
    for p in procs:
        p.start()
    try:
        got = [q.get(timeout=180) for _ in range(2)]      # drain before joining: puts block on large items
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.exitcode is None:
                p.kill()
    assert all(p.exitcode == 0 for p in procs)
    out = next(g for g in got if not isinstance(g, tuple))
    new_k = next(g for g in got if isinstance(g, tuple))[1]
    c = I.attention_layer(batch=batch, position=position, seed=77)
    exp, kc, _ = oracle.attention(**c)
    np.testing.assert_allclose(out.reshape(-1), exp, atol=1e-5, rtol=0)
    np.testing.assert_array_equal(new_k, kc[position:])
