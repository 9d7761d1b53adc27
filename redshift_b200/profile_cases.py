"""Run one hot-path case a few times, for profilers (ncu) and quick timing.

    python -m redshift_b200.profile_cases decode  [context]   # one verify-8 attention layer
    python -m redshift_b200.profile_cases decode_exchange [context]  # the same through the peer exchange (1 rank)
    python -m redshift_b200.profile_cases delta   [tokens]    # one DeltaNet layer (16/48 heads, d128)
    python -m redshift_b200.profile_cases prefill [tokens]    # core causal prefill attention
    python -m redshift_b200.profile_cases attention_prefill [tokens]  # attention layer, prefill regime
    python -m redshift_b200.profile_cases delta_core [tokens] # DeltaNet prefill recurrence (core)
    python -m redshift_b200.profile_cases delta_chunked [tokens] # DeltaNet prefill, chunked tcgen05 form
    python -m redshift_b200.profile_cases mm_q8_0 [rows]      # verify-8 projection, width 5120 (also mm_q4_k, mm_q6_k)

Options: ``--reps N`` launches (default 3), ``--time`` prints the mean
CUDA-event time of the last N launches.  Inputs are seeded N(0,1) (DeltaNet
state N(0,0.02)), device-resident, with the benchmark configurations' shapes.
"""
import argparse
import sys

import torch

from .runtime import HotPath

H, HKV, HD = 24, 4, 256
HK, HV, DK = 16, 48, 128
C = (2 * HK + HV) * DK


def make_case(hot, case, size):
    dev = torch.device('cuda')
    g = torch.Generator(device=dev)
    g.manual_seed(0)
    f32 = dict(device=dev, dtype=torch.float32)
    if case == 'decode':
        T, ctx = 8, size or 139264
        kc = torch.randn((ctx, HKV, HD), generator=g, device=dev, dtype=torch.float16)
        vc = torch.randn((ctx, HKV, HD), generator=g, device=dev, dtype=torch.float16)
        qg = torch.randn((T, H, 2 * HD), generator=g, **f32)
        key = torch.randn((T, HKV, HD), generator=g, **f32)
        val = torch.randn((T, HKV, HD), generator=g, **f32)
        ones = torch.ones(HD, **f32)
        out = torch.empty((T, H, HD), **f32)
        ws = torch.zeros(hot.lib.qv_attention_workspace(T, ctx - T), dtype=torch.uint8, device=dev)
        return lambda: hot.attention(out, kc, vc, qg, key, val, ones, ones, T, ctx - T, workspace=ws)
    if case == 'decode_exchange':
        # one rank of the fused peer exchange, exchanging with itself (world = 1)
        T, ctx = 8, size or 139264
        kc = torch.randn((ctx, HKV, HD), generator=g, device=dev, dtype=torch.float16)
        vc = torch.randn((ctx, HKV, HD), generator=g, device=dev, dtype=torch.float16)
        qg = torch.randn((T, H, 2 * HD), generator=g, **f32)
        key = torch.randn((T, HKV, HD), generator=g, **f32)
        val = torch.randn((T, HKV, HD), generator=g, **f32)
        ones = torch.ones(HD, **f32)
        out = torch.empty((T, H, HD), **f32)
        ws = torch.zeros(hot.lib.qv_attention_shard_workspace(T, ctx - T), dtype=torch.uint8, device=dev)
        buf = torch.zeros(hot.lib.qv_attention_exchange_bytes(1) // 4, dtype=torch.float32, device=dev)
        peers = torch.tensor([buf.data_ptr()], dtype=torch.int64, device=dev)
        state = {'seq': 0}

        def run():
            hot.attention_shard_exchange(out, kc, vc, 0, ctx - T, qg, key, val, ones, ones, T, ctx - T, peers, 1, 0,
                                         state['seq'], workspace=ws)
            state['seq'] += 1
        run.keep = (buf, peers)
        return run
    if case in ('delta', 'delta_core', 'delta_chunked'):
        T = size or (8 if case == 'delta' else 4096)
        state = torch.randn((HV, DK, DK), generator=g, **f32) * 0.02
        alpha = torch.randn((T, HV), generator=g, **f32)
        beta = torch.randn((T, HV), generator=g, **f32)
        decay = torch.full((HV,), -1.0, **f32)
        bias = torch.zeros(HV, **f32)
        if case == 'delta':
            conv = torch.zeros((C, 4), **f32)
            conv[:, 3] = 1
            args = dict(out=torch.empty((T, HV, DK), **f32), state=state, history=torch.zeros((3, C), **f32),
                        qkv=torch.randn((T, C), generator=g, **f32), gate=torch.randn((T, HV, DK), generator=g, **f32),
                        alpha=alpha, beta=beta, conv=conv, decay=decay, bias=bias, norm=torch.ones(DK, **f32))
            return lambda: hot.delta(**args, batch=T, key_heads=HK, value_heads=HV, dim=DK)
        q = torch.randn((T, HK, DK), generator=g, device=dev, dtype=torch.float16)
        k = torch.randn((T, HK, DK), generator=g, device=dev, dtype=torch.float16)
        v = torch.randn((T, HV, DK), generator=g, device=dev, dtype=torch.float16)
        out = torch.empty((T, HV, DK), **f32)
        if case == 'delta_chunked':
            ws = torch.empty(hot.lib.qv_delta_chunked_workspace(T, HV), dtype=torch.uint8, device=dev)
            return lambda: hot.delta_chunked(out, state, q, k, v, alpha, beta, decay, bias, T, HK, HV, DK, workspace=ws)
        return lambda: hot.delta_core(out, state, q, k, v, alpha, beta, decay, bias, T, HK, HV, DK)
    if case.startswith('mm_'):
        kind = {'mm_q8_0': 8, 'mm_q4_k': 12, 'mm_q6_k': 14}[case]
        T, width, rows = 8, 5120, size or 17408
        nbytes = int(hot.lib.qv_mm_weight_bytes(kind, width, rows))
        blk = 34 if kind == 8 else (144 if kind == 12 else 210)
        w = torch.randint(0, 256, (nbytes,), generator=g, device=dev, dtype=torch.uint8)
        v = w.view(-1, blk)                 # finite fp16 block scales: 2^-7 (Q8_0, Q4_K d and dmin), 2^-8 (Q6_K)
        if kind == 14:
            v[:, 208] = 0x00
            v[:, 209] = 0x1c
        else:
            v[:, 0] = 0x00
            v[:, 1] = 0x20
            if kind == 12:
                v[:, 2] = 0x00
                v[:, 3] = 0x20
        x = torch.randn((T, width), generator=g, **f32)
        out = torch.empty((T, rows), **f32)
        return lambda: hot.mm(out, w, x, kind, T, width, rows)
    if case == 'prefill':
        L = size or 4096
        q = torch.randn((L, H, HD), generator=g, device=dev, dtype=torch.float16)
        k = torch.randn((L, HKV, HD), generator=g, device=dev, dtype=torch.float16)
        v = torch.randn((L, HKV, HD), generator=g, device=dev, dtype=torch.float16)
        out = torch.empty((L, H, HD), **f32)
        return lambda: hot.prefill_attention(out, q, k, v, L)
    if case == 'attention_prefill':
        # the attention layer's prefill regime: prepare (norms, rotary, append) + precise causal block
        L = size or 4096
        kc = torch.zeros((L, HKV, HD), device=dev, dtype=torch.float16)
        vc = torch.zeros_like(kc)
        qg = torch.randn((L, H, 2 * HD), generator=g, **f32)
        key = torch.randn((L, HKV, HD), generator=g, **f32)
        val = torch.randn((L, HKV, HD), generator=g, **f32)
        ones = torch.ones(HD, **f32)
        out = torch.empty((L, H, HD), **f32)
        ws = torch.zeros(hot.lib.qv_attention_workspace(L, 0), dtype=torch.uint8, device=dev)
        return lambda: hot.attention(out, kc, vc, qg, key, val, ones, ones, L, 0, workspace=ws)
    raise ValueError(f'unknown case {case}')


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument('case', choices=['decode', 'decode_exchange', 'delta', 'prefill', 'attention_prefill', 'delta_core',
                                     'delta_chunked', 'mm_q8_0', 'mm_q4_k', 'mm_q6_k'])
    ap.add_argument('size', type=int, nargs='?', default=0)
    ap.add_argument('--reps', type=int, default=3)
    ap.add_argument('--time', action='store_true')
    args = ap.parse_args(argv)
    hot = HotPath()
    run = make_case(hot, args.case, args.size)
    run()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.reps):
        run()
    e1.record()
    torch.cuda.synchronize()
    if hot.status():
        raise RuntimeError('a kernel reported a timeout')
    if args.time:
        print(f'{args.case} {args.size}: {e0.elapsed_time(e1) / args.reps * 1e3:.2f} us per call')
    return 0


if __name__ == '__main__':
    sys.exit(main())
