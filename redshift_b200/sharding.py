"""Sequence-split (split-KV) decode attention across the GPUs of one node.

The reference runs on one GPU only; long-context decode is the one part of
the hot path that partitions: rank g of G keeps the cache rows of absolute
positions ``[g*P//G, (g+1)*P//G)`` (P = verify position) in its own HBM, and
the last rank also receives the block's new rows.  Each rank attends its
queries over its shard (``qv_attention_shard``: prepare + split-KV kernel +
in-shard combine, producing a normalised partial O and its LSE), the pairs
are all-gathered (one NCCL collective pair per attention layer; 197 KB per
rank at verify-8), and every rank merges them with ``qv_attention_merge``:
O = sum_g exp(LSE_g - LSE) O_g, times sigmoid(gate).

The DeltaNet layers do not shard (the recurrence is sequential): every rank
computes them redundantly.
"""
from dataclasses import dataclass


@dataclass(frozen=True)
class Shard:
    rank: int
    world: int
    begin: int        # absolute position of local row 0
    rows: int         # prefix rows held locally before the verify block
    appends: bool     # this rank receives the block's new rows

    @property
    def capacity(self):
        return self.rows


def plan(position, world, rank, batch=8):
    """The shard of ``rank`` for a verify block at ``position``.

    Prefix rows are split as evenly as whole rows allow; the last rank holds
    the newest prefix rows and appends the block (so its capacity is
    ``rows + batch``).
    """
    if world < 1 or not 0 <= rank < world:
        raise ValueError('invalid rank / world size')
    if position < 0:
        raise ValueError('negative position')
    begin = rank * position // world
    end = (rank + 1) * position // world
    return Shard(rank, world, begin, end - begin, rank == world - 1)


def shard_capacity(shard, batch):
    return shard.rows + (batch if shard.appends else 0)


class ShardedAttention:
    """One attention layer's sequence-split verify step on a process group.

    ``hot`` provides ``attention_shard`` and ``attention_merge`` (the
    library's ``HotPath``); ``dist`` is ``torch.distributed``.  Buffers are
    preallocated by the caller so the step can be replayed (or captured in a
    CUDA graph) without allocation:
      part [batch,24,256] f32, lse [batch,24] f32,
      gathered_part [world,batch,24,256] f32, gathered_lse [world,batch,24] f32.
    """

    def __init__(self, hot, dist, shard, group=None):
        self.hot, self.dist, self.shard, self.group = hot, dist, shard, group

    def __call__(self, out, key_cache, value_cache, q_gate, key, value, q_norm, k_norm, batch, position,
                 part, lse, gathered_part, gathered_lse, epsilon=1e-6, workspace=None):
        s = self.shard
        self.hot.attention_shard(part, lse, key_cache, value_cache, s.begin, s.rows, q_gate, key, value,
                                 q_norm, k_norm, batch, position, epsilon, workspace=workspace)
        # [world*batch, ...] views: the layout every backend accepts for all-gather.
        self.dist.all_gather_into_tensor(gathered_part.view(-1, *part.shape[1:]), part, group=self.group)
        self.dist.all_gather_into_tensor(gathered_lse.view(-1, *lse.shape[1:]), lse, group=self.group)
        self.hot.attention_merge(out, gathered_part, gathered_lse, s.world, batch, q_gate)


class PeerExchange:
    """Fused multi-GPU verify through peer memory (``qv_attention_shard_exchange``).

    Allocates each rank's exchange buffer in torch symmetric memory (mapped
    into every rank of ``group``), zeroes it and publishes the rank-ordered
    array of buffer addresses.  Each call runs the shard's attention, stores
    its (partial, LSE) into every rank's buffer, tagged with the call's
    sequence number, waits for the other ranks' words of this call and merges;
    no collective library is on the path.  ``sequence`` numbers the calls on
    these buffers, +1 per call and the same on every rank (e.g. the attention
    layer's index within a step whose layer count is even).
    """

    def __init__(self, hot, dist, shard, group=None):
        import torch
        import torch.distributed._symmetric_memory as symm_mem
        self.hot, self.shard = hot, shard
        nbytes = hot.lib.qv_attention_exchange_bytes(shard.world)
        if nbytes == 0:
            raise ValueError('world size not supported by the peer exchange')
        self.buffer = symm_mem.empty(nbytes // 4, dtype=torch.float32, device='cuda')
        self.buffer.zero_()
        self.handle = symm_mem.rendezvous(self.buffer, group if group is not None else dist.group.WORLD)
        self.peers = torch.tensor(list(self.handle.buffer_ptrs), dtype=torch.int64, device='cuda')
        torch.cuda.synchronize()
        dist.barrier(group=group)

    def __call__(self, out, key_cache, value_cache, q_gate, key, value, q_norm, k_norm, batch, position, sequence,
                 epsilon=1e-6, workspace=None):
        s = self.shard
        self.hot.attention_shard_exchange(out, key_cache, value_cache, s.begin, s.rows, q_gate, key, value, q_norm,
                                          k_norm, batch, position, self.peers, s.world, s.rank, sequence, epsilon,
                                          workspace=workspace)
