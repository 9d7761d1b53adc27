"""Sequence-split verify across two or four GPUs through the library's fused peer-memory
exchange (and the NCCL all-gather variant), compared with the single-device
CPU oracle.  Each case is skipped on machines with fewer GPUs than its ranks."""
import datetime
import os
import queue
import socket
import time

import numpy as np
import pytest

import oracle
from oracle import inputs as I

pytestmark = pytest.mark.gpu


def _gpus():
    try:
        import torch
        return torch.cuda.device_count()
    except Exception:
        return 0


def _free_port():
    with socket.socket() as s:
        s.bind(('127.0.0.1', 0))
        return s.getsockname()[1]


def _worker(rank, world, port, position, batch, mode, result):
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR='127.0.0.1', MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group('nccl', rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device('cuda', rank))
    try:
        from redshift_b200 import HotPath
        from redshift_b200.sharding import PeerExchange, ShardedAttention, plan, shard_capacity
        hot = HotPath()
        c = I.attention_layer(batch=batch, position=position, seed=91)
        s = plan(position, world, rank, batch)
        dev = torch.device('cuda', rank)
        kc = torch.zeros((shard_capacity(s, batch), 4, 256), dtype=torch.float16, device=dev)
        vc = torch.zeros_like(kc)
        kc[:s.rows] = torch.from_numpy(c['key_cache'][s.begin:s.begin + s.rows]).to(dev)
        vc[:s.rows] = torch.from_numpy(c['value_cache'][s.begin:s.begin + s.rows]).to(dev)
        t = lambda k: torch.from_numpy(np.ascontiguousarray(np.asarray(c[k], np.float32))).to(dev)  # noqa: E731
        args = (t('q_gate'), t('key'), t('value'), t('q_norm'), t('k_norm'), batch, position)
        out = torch.empty((batch, 24, 256), device=dev)
        if mode == 'peer':
            ex = PeerExchange(hot, dist, s)
            for seq in range(4):
                ex(out, kc, vc, *args, seq)
        else:
            part, lse = torch.empty((batch, 24, 256), device=dev), torch.empty((batch, 24), device=dev)
            gp, gl = torch.empty((world, batch, 24, 256), device=dev), torch.empty((world, batch, 24), device=dev)
            ShardedAttention(hot, dist, s)(out, kc, vc, *args, part, lse, gp, gl)
        torch.cuda.synchronize()
        status = hot.status()
        result.put((rank, status, out.cpu().numpy()))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize('world', [2, 4])
@pytest.mark.parametrize('mode', ['peer', 'nccl'])
def test_sequence_split_verify(mode, world):
    if _gpus() < world:
        pytest.skip(f'needs {world} GPUs')
    import torch.multiprocessing as mp
    position, batch = 70000, 8
    ctx = mp.get_context('spawn')
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, position, batch, mode, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = []
    try:
        deadline = time.time() + 300
        while len(got) < world and time.time() < deadline:
            try:
                got.append(q.get(timeout=5))
            except queue.Empty:
                if all(not p.is_alive() for p in procs):
                    break          # the workers are gone: no result can still arrive
    finally:
        for p in procs:
            p.join(timeout=120)
            if p.exitcode is None:
                p.kill()
    assert all(p.exitcode == 0 for p in procs)
    assert len(got) == world
    c = I.attention_layer(batch=batch, position=position, seed=91)
    exp, _, _ = oracle.attention(**c)
    for rank, status, out in got:
        assert status == 0, f'rank {rank}: a kernel timed out'
        err = np.abs(out.reshape(-1) - exp)
        assert err.max() <= 2e-3
        assert (err <= 3e-4 * (1 + np.abs(exp))).all()
