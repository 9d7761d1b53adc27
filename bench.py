#!/usr/bin/env python
"""Benchmark of the Redshift hot path on B200: the verify-8 step of the
64-layer model's attention/DeltaNet layers, without the projections.

One step = 16 full-attention layers (verify block of 8 tokens at context
139,264: position 139,256, each layer with its own 570 MB fp16 KV cache) +
48 gated-DeltaNet layers (8 tokens, each with its own 3 MB fp32 state), in
the model's layer order (every 4th layer is attention).  Reported as
microseconds per step (lower is better).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

N > 1 runs under torchrun: each rank holds a 1/N sequence shard of every
attention layer's KV cache, attends over it, and the (partial O, LSE) pairs
are exchanged through peer memory by the library's fused exchange kernel
(``--nccl-merge``: NCCL all-gather + merge kernel instead) and merged on
every rank; DeltaNet layers are replicated.  ``--impl reference`` times the CPU oracle
(the numpy restatement of the reference's cpu_reference.py) on a bounded
sample of the same step, on rank 0 only.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = 'verify-8 attn+DeltaNet µs/step at ctx 32k/139k; % HBM roofline; prefill TFLOP/s'
UNIT = 'us/step'
H, HKV, HD = 24, 4, 256
HK, HV, DK = 16, 48, 128
C = (2 * HK + HV) * DK
LAYERS = 64
# DRAM bytes (read + write) of one decode fa_kernel launch at context 139,264,
# from `ncu --metrics dram__bytes_read.sum,dram__bytes_write.sum` on
# `python -m redshift_b200.profile_cases decode 139264` (profiles/fa_kernel_decode_139k.md).
FA_TRAFFIC_139K = 570991360 + 199424


RESULT_OUT = sys.stdout


def emit(line):
    RESULT_OUT.write(json.dumps(line) + '\n')
    RESULT_OUT.flush()


def parse():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument('--gpus', type=int, default=1)
    ap.add_argument('--steps', type=int, default=30)
    ap.add_argument('--warmup', type=int, default=5)
    ap.add_argument('--impl', choices=['b200', 'reference'], default='b200')
    ap.add_argument('--context', type=int, default=139264)
    ap.add_argument('--tokens', type=int, default=8)
    ap.add_argument('--no-e2e', action='store_true')
    ap.add_argument('--no-cpu-baseline', action='store_true')
    ap.add_argument('--no-extras', action='store_true', help='skip the 32k / prefill side measurements')
    ap.add_argument('--no-graph', action='store_true', help='launch eagerly instead of replaying a CUDA graph')
    ap.add_argument('--nccl-merge', action='store_true', help='N>1: NCCL all-gather instead of the peer exchange')
    return ap.parse_args()


def peaks():
    try:
        d = json.loads((ROOT / 'MEASURED_PEAKS.json').read_text())
        return float(d['hbm_gbs']), float(d['bf16_tflops']), 'measured'
    except Exception:
        return 6650.0, 1590.0, 'fallback'


# ----------------------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons during a region."""
    FIELDS = ('index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,'
              'clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,'
              'clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap')

    def __init__(self, index):
        self.index, self.proc, self.lines = index, None, []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(['nvidia-smi', f'--id={self.index}', f'--query-gpu={self.FIELDS}',
                                          '--format=csv,noheader,nounits', '-lms', '100'],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        if self.proc:
            time.sleep(0.2)
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except Exception:
                self.proc.kill()
                out = ''
            self.lines = [line for line in out.splitlines() if line.strip()]

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ('hw_slowdown', 'hw_thermal_slowdown', 'sw_thermal_slowdown', 'sw_power_cap')
        for line in self.lines:
            parts = [p.strip() for p in line.split(',')]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for name, val in zip(names, parts[5:9]):
                if val.lower().startswith('active'):
                    reasons.add(name)
        if not sm:
            return {'sm_mhz': None, 'sm_max_mhz': None, 'reasons': [], 'samples': 0}
        return {'sm_mhz': statistics.median(sm), 'sm_max_mhz': mx, 'reasons': sorted(reasons),
                'samples': len(sm)}


# ----------------------------------------------------------------------------- workload
class Step:
    """Device-resident buffers of the 64 layers and the per-step dispatch."""

    def __init__(self, hot, context, tokens, rank, world, seed=1234, attention_only=False):
        import torch
        self.torch, self.hot = torch, hot
        self.dev = torch.device('cuda', torch.cuda.current_device())
        self.T, self.world, self.rank = tokens, world, rank
        self.position = context - tokens
        P = self.position
        self.begin = rank * P // world
        self.rows = (rank + 1) * P // world - self.begin            # prefix rows of this shard
        self.last = rank == world - 1                                # the shard that receives the new rows
        cap = self.rows + (tokens if self.last else 0)
        g = torch.Generator(device=self.dev)
        g.manual_seed(seed + rank)
        f32 = dict(device=self.dev, dtype=torch.float32)
        self.attn, self.delta = [], []
        for layer in range(LAYERS):
            if attention_only and layer % 4 != 3:
                continue
            if layer % 4 == 3:
                kc = torch.randn((cap, HKV, HD), generator=g, device=self.dev, dtype=torch.float16)
                vc = torch.randn((cap, HKV, HD), generator=g, device=self.dev, dtype=torch.float16)
                self.attn.append(dict(
                    kc=kc, vc=vc,
                    q_gate=torch.randn((tokens, H, 2 * HD), generator=g, **f32),
                    key=torch.randn((tokens, HKV, HD), generator=g, **f32),
                    value=torch.randn((tokens, HKV, HD), generator=g, **f32),
                    out=torch.empty((tokens, H, HD), **f32)))
            else:
                conv = torch.zeros((C, 4), **f32)
                conv[:, 3] = 1
                self.delta.append(dict(
                    state=torch.randn((HV, DK, DK), generator=g, **f32) * 0.02,
                    history=torch.zeros((3, C), **f32),
                    qkv=torch.randn((tokens, C), generator=g, **f32).half().float(),
                    gate=torch.randn((tokens, HV, DK), generator=g, **f32),
                    alpha=torch.randn((tokens, HV), generator=g, **f32),
                    beta=torch.randn((tokens, HV), generator=g, **f32),
                    conv=conv, out=torch.empty((tokens, HV, DK), **f32)))
        self.ones = torch.ones(HD, **f32)
        self.decay = torch.full((HV,), -1.0, **f32)
        self.bias = torch.zeros(HV, **f32)
        self.norm = torch.ones(DK, **f32)
        self.exchange = None
        if world > 1:
            need = hot.lib.qv_attention_shard_workspace(tokens, self.rows)
            self.part = torch.empty((tokens, H, HD), **f32)
            self.lse = torch.empty((tokens, H), **f32)
            self.gpart = torch.empty((world, tokens, H, HD), **f32)
            self.glse = torch.empty((world, tokens, H), **f32)
        else:
            need = hot.lib.qv_attention_workspace(tokens, self.position)
        self.ws = torch.zeros(max(int(need), 256), dtype=torch.uint8, device=self.dev)   # barrier words start at 0
        self.launches_per_step = len(self.attn) + len(self.delta)   # one launch per layer (split combine / exchange in the tail)
        if not attention_only:
            self.pack()

    IN_KEYS = {True: ('q_gate', 'key', 'value'), False: ('qkv', 'gate', 'alpha', 'beta')}

    def layers(self):
        """(is_attention, buffers) of the 64 layers in step order."""
        ai = di = 0
        for layer in range(LAYERS):
            if layer % 4 == 3:
                yield True, self.attn[ai]
                ai += 1
            else:
                yield False, self.delta[di]
                di += 1

    def pack(self):
        """Every layer's inputs, and separately every layer's output, as views of one device
        buffer in step order (each view 256-byte aligned), so that the end-to-end step moves
        them host<->device as one copy per group of four layers instead of one per tensor."""
        torch, align = self.torch, 64

        def build(entries):
            offs, n = [], 0
            for d, k in entries:
                offs.append(n)
                n += -(-d[k].numel() // align) * align
            buf = torch.empty(n, device=self.dev, dtype=torch.float32)
            for (d, k), o in zip(entries, offs):
                view = buf[o:o + d[k].numel()].view(d[k].shape)
                view.copy_(d[k])
                d[k] = view
            return buf, offs

        ins, outs, first_in = [], [], []
        for is_attn, d in self.layers():
            first_in.append(len(ins))
            ins += [(d, k) for k in self.IN_KEYS[is_attn]]
            outs.append((d, 'out'))
        self.in_dev, in_offs = build(ins)
        self.out_dev, out_offs = build(outs)
        starts = [in_offs[i] for i in first_in[::4]] + [self.in_dev.numel()]
        self.in_groups = list(zip(starts[:-1], starts[1:]))
        starts = out_offs[::4] + [self.out_dev.numel()]
        self.out_groups = list(zip(starts[:-1], starts[1:]))

    def use_peer_exchange(self, dist):
        """Switch the N>1 attention layers to the fused peer-memory exchange."""
        from redshift_b200.sharding import PeerExchange, plan
        self.exchange = PeerExchange(self.hot, dist, plan(self.position, self.world, self.rank, self.T))

    def attention_layer(self, a, seq=0):
        hot, T = self.hot, self.T
        if self.world == 1:
            hot.attention(a['out'], a['kc'], a['vc'], a['q_gate'], a['key'], a['value'], self.ones, self.ones,
                          T, self.position, workspace=self.ws)
        elif self.exchange is not None:
            self.exchange(a['out'], a['kc'], a['vc'], a['q_gate'], a['key'], a['value'], self.ones, self.ones,
                          T, self.position, seq, workspace=self.ws)
        else:
            import torch.distributed as dist
            hot.attention_shard(self.part, self.lse, a['kc'], a['vc'], self.begin, self.rows, a['q_gate'],
                                a['key'], a['value'], self.ones, self.ones, T, self.position, workspace=self.ws)
            dist.all_gather_into_tensor(self.gpart.view(-1, H, HD), self.part)
            dist.all_gather_into_tensor(self.glse.view(-1, H), self.lse)
            hot.attention_merge(a['out'], self.gpart, self.glse, self.world, T, a['q_gate'])

    def attention_only(self):
        """The step's attention layers back to back (what the attention scaling figure times)."""
        for ai, a in enumerate(self.attn):
            self.attention_layer(a, seq=ai)

    def delta_layer(self, d):
        self.hot.delta(d['out'], d['state'], d['history'], d['qkv'], d['gate'], d['alpha'], d['beta'], d['conv'],
                       self.decay, self.bias, self.norm, self.T, HK, HV, DK)

    def run(self, events=None):
        ai = di = 0
        for layer in range(LAYERS):
            if layer % 4 == 3:
                if events is not None:
                    events[ai][0].record()
                self.attention_layer(self.attn[ai], seq=ai)
                if events is not None:
                    events[ai][1].record()
                ai += 1
            else:
                self.delta_layer(self.delta[di])
                di += 1

    # host-side (pinned) copies of the per-step inputs and outputs, for e2e
    def host_mirror(self):
        """Pinned host copies of the packed inputs (each rank feeds its own GPU) and outputs (read
        back by rank 0 only: the outputs are identical on every rank); returns the bytes a step
        copies each way."""
        torch = self.torch
        self.readback = self.rank == 0
        self.in_host = self.in_dev.cpu().pin_memory()
        self.out_host = torch.empty_like(self.out_dev, device='cpu').pin_memory()
        self.s_in, self.s_out = torch.cuda.Stream(), torch.cuda.Stream()
        h2d = self.in_dev.numel() * 4
        d2h = self.out_dev.numel() * 4 if self.readback else 0
        return h2d, d2h

    def run_e2e(self):
        """One step through the public API from pinned host buffers: the inputs of each group
        of four layers are copied host->device on a copy stream in layer order (a group's
        layers wait only for that group's copy), and each group's outputs are read back on a
        second copy stream as soon as its last layer is done; the step ends when the last
        read-back has landed."""
        torch = self.torch
        main = torch.cuda.current_stream()
        start = torch.cuda.Event()
        start.record(main)
        self.s_in.wait_event(start)
        self.s_out.wait_event(start)
        ready = []
        with torch.cuda.stream(self.s_in):
            for lo, hi in self.in_groups:
                self.in_dev[lo:hi].copy_(self.in_host[lo:hi], non_blocking=True)
                ev = torch.cuda.Event()
                ev.record(self.s_in)
                ready.append(ev)
        for layer, (is_attn, d) in enumerate(self.layers()):
            if layer % 4 == 0:
                main.wait_event(ready[layer // 4])
            if is_attn:
                self.attention_layer(d, seq=(layer - 3) // 4)
            else:
                self.delta_layer(d)
            if self.readback and layer % 4 == 3:
                done = torch.cuda.Event()
                done.record(main)
                self.s_out.wait_event(done)
                lo, hi = self.out_groups[layer // 4]
                with torch.cuda.stream(self.s_out):
                    self.out_host[lo:hi].copy_(self.out_dev[lo:hi], non_blocking=True)
        main.wait_stream(self.s_in)
        main.wait_stream(self.s_out)


def make_events(n, external):
    import torch
    return [(torch.cuda.Event(enable_timing=True, external=external),
             torch.cuda.Event(enable_timing=True, external=external)) for _ in range(n)]


def time_graph(torch, fn, reps, warmup, sync=None):
    """Mean device time (ms) of one replay of a CUDA graph of fn()."""
    graph = capture(torch, fn)
    for _ in range(warmup):
        graph.replay()
    torch.cuda.synchronize()
    if sync is not None:
        sync()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        graph.replay()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / reps
    graph.reset()
    return ms


def capture(torch, fn):
    """Capture fn() into a CUDA graph (after one eager call on the capture stream)."""
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        fn()
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        fn()
    torch.cuda.synchronize()
    return g


def bench_b200(args):
    import torch
    rank = int(os.environ.get('RANK', 0))
    world = int(os.environ.get('WORLD_SIZE', 1))
    local = int(os.environ.get('LOCAL_RANK', 0))
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group('nccl', timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device('cuda', local))
    from redshift_b200 import HotPath
    hot = HotPath()
    step = Step(hot, args.context, args.tokens, rank, world)
    exchange = 'none'
    if world > 1:
        exchange = 'nccl all-gather + merge kernel'
        if not args.nccl_merge:
            try:
                step.use_peer_exchange(dist)
                exchange = 'fused peer-memory exchange (P2P stores + flags, symmetric memory)'
            except Exception as exc:
                print(f'# peer exchange unavailable ({exc}); using NCCL all-gather', file=sys.stderr)
        if step.exchange is None:       # shard kernel + merge kernel per attention layer
            step.launches_per_step = len(step.attn) * 2 + len(step.delta)
    torch.cuda.synchronize()

    def barrier():
        if dist is not None:
            dist.barrier()

    def max_over_ranks(values):
        if dist is None:
            return values
        t = torch.tensor(values, device='cuda', dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return t.tolist()

    # One eager step creates the NCCL communicator and every lazy resource.
    step.run()
    torch.cuda.synchronize()
    events = make_events(len(step.attn), external=True)
    graph, mode = None, 'eager'
    if not args.no_graph:
        try:
            graph = capture(torch, lambda: step.run(events))
            mode = 'cuda-graph'
        except Exception as exc:  # capture is an optimisation; report and run eagerly
            print(f'# CUDA graph capture failed ({exc}); timing eager launches', file=sys.stderr)
            graph = None
            events = make_events(len(step.attn), external=False)
            torch.cuda.synchronize()
    graphs = [graph] if graph is not None else []      # every graph is reset before teardown

    def run_step():
        if graph is not None:
            graph.replay()
        else:
            step.run(events)

    for _ in range(args.warmup):
        run_step()
    torch.cuda.synchronize()
    if hot.status():
        raise RuntimeError('a kernel reported a timeout during warm-up')

    K = args.steps
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        barrier()
        torch.cuda.synchronize()
        t0.record()
        for _ in range(K):
            run_step()
        t1.record()
        torch.cuda.synchronize()
        barrier()
    ms = t0.elapsed_time(t1) / K
    # per-layer attention time of the last timed step (events inside the step)
    attn_ms = statistics.mean(s.elapsed_time(e) for s, e in events)
    ms, attn_ms = max_over_ranks([ms, attn_ms])
    if hot.status():
        raise RuntimeError('a kernel reported a timeout during the timed region')

    # end-to-end through the public entry points with host inputs/outputs
    e2e = None
    if not args.no_e2e:
        h2d, d2h = step.host_mirror()
        e2e_graph = None
        if graph is not None:
            try:
                e2e_graph = capture(torch, step.run_e2e)
                graphs.append(e2e_graph)
            except Exception as exc:
                print(f'# e2e graph capture failed ({exc}); eager e2e', file=sys.stderr)

        def run_e2e():
            if e2e_graph is not None:
                e2e_graph.replay()
            else:
                step.run_e2e()
        for _ in range(2):
            run_e2e()
        torch.cuda.synchronize()
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        e0.record()
        for _ in range(K):
            run_e2e()
        e1.record()
        torch.cuda.synchronize()
        barrier()
        e_ms = max_over_ranks([e0.elapsed_time(e1) / K])[0]
        e2e = {'value': round(e_ms * 1e3, 2), 'unit': UNIT, 'h2d_bytes_per_step': h2d,
               'd2h_bytes_per_step': d2h, 'launch': 'cuda-graph' if e2e_graph is not None else 'eager',
               'copies': 'every rank copies its own inputs, rank 0 reads back every layer\'s output, '
                         'one copy per group of four layers each way'}

    # The attention layers back to back (the sequence split's own figure, free of the replicated
    # DeltaNet layers): every rank times its shards; at N > 1 rank 0 also times the same 16 layers
    # at the full context on its one GPU, so that the scaling efficiency t1 / (N tN) comes from
    # one run on one box.
    attn_b2b = attn_1 = None
    if not args.no_extras:
        attn_b2b = max_over_ranks([time_graph(torch, step.attention_only, K, args.warmup, barrier)
                                   / len(step.attn)])[0]
        if world > 1:
            if rank == 0:
                full = Step(hot, args.context, args.tokens, 0, 1, seed=99, attention_only=True)
                attn_1 = time_graph(torch, full.attention_only, K, args.warmup) / len(full.attn)
                del full
                torch.cuda.empty_cache()
            barrier()

    hbm_peak, tc_peak, peak_kind = peaks()
    kv_rows = step.rows + (args.tokens if step.last else 0)
    attn_bytes = kv_rows * HKV * HD * 2 * 2
    achieved = attn_bytes / (attn_ms * 1e-3) / 1e9
    roofline = {'bound': 'hbm', 'achieved': round(achieved, 1), 'peak': hbm_peak, 'unit': 'GB/s',
                'frac': round(achieved / hbm_peak, 4),
                'traffic': FA_TRAFFIC_139K if (args.context == 139264 and world == 1) else None,
                'kernel': 'attention layer (one split-KV fa_kernel launch: prepare/append, attention, split '
                          'combine or peer exchange in its tail), per rank',
                'algorithmic_bytes_per_launch': attn_bytes, 'avg_layer_ms': round(attn_ms, 5),
                'peak_source': peak_kind}

    extras = {}
    if rank == 0 and world == 1 and not args.no_extras:
        extras = side_measurements(hot, torch, tc_peak, hbm_peak)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(args.context, args.tokens)

    per_layer = {'attention': round(attn_ms * 1e3, 2), 'delta_estimate': round((ms - 16 * attn_ms) * 1e3 / 48, 2)}
    if attn_b2b is not None:
        per_layer['attention_back_to_back'] = round(attn_b2b * 1e3, 2)
    if attn_1 is not None:
        per_layer['attention_back_to_back_1gpu'] = round(attn_1 * 1e3, 2)
        per_layer['attention_scaling_eff'] = round(attn_1 / (world * attn_b2b), 4)
    if rank == 0:
        line = {
            'metric': METRIC, 'value': round(ms * 1e3, 2), 'unit': UNIT, 'n_gpus': world, 'steps': K,
            'warmup': args.warmup, 'ms_per_step': round(ms, 5), 'higher_is_better': False,
            'scaling': 'strong', 'vs_baseline': None, 'dtype': 'f16 KV/operands, f32 accumulate and state',
            'data': 'synthetic (seeded N(0,1) fp16 KV, N(0,0.02) DeltaNet state)',
            'config': {'workload': f'verify-{args.tokens} hot-path step of the 64-layer model: 16 attention '
                                   f'layers at context {args.context} + 48 gated-DeltaNet layers',
                       'context': args.context, 'verify_tokens': args.tokens, 'attention_layers': 16,
                       'delta_layers': 48, 'attention': '24 q / 4 kv heads, d256, fp16 KV',
                       'deltanet': '16 k / 48 v heads, d128, fp32 state',
                       'l2': 'inputs larger than L2 (9.1 GB of KV + 151 MB of state per step)',
                       'launch': mode, 'exchange': exchange,
                       'parallelism': (f'sequence-split KV x{world} ({exchange}), DeltaNet replicated')
                                      if world > 1 else 'single GPU'},
            'clocks': clocks.summary(),
            'gpu_launches': step.launches_per_step * K,
            'e2e': e2e,
            'roofline': roofline,
            'cpu_baseline': cpu,
            'per_layer_us': per_layer,
            'extras': extras,
        }
        emit(line)
    # Graphs that captured NCCL calls must be released before the process group.
    torch.cuda.synchronize()
    for g in graphs:
        g.reset()
    graphs.clear()
    graph = e2e_graph = None
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


def side_measurements(hot, torch, tc_peak, hbm_peak):
    """Attention at 32k, causal prefill (config 3) and DeltaNet prefill core (config 4)."""
    res = {}
    # config 2 at 32,768: the 16 attention layers of a step back to back, replayed as a
    # CUDA graph (eager launches from Python would leave the GPU waiting on the host)
    step = Step(hot, 32768, 8, 0, 1, seed=77)
    graph = capture(torch, lambda: [step.attention_layer(a) for a in step.attn])
    for _ in range(3):
        graph.replay()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(10):
        graph.replay()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / (10 * len(step.attn))
    graph.reset()
    del graph
    res['attention_32k_us'] = round(ms * 1e3, 2)
    res['attention_32k_hbm_frac'] = round(32768 * 4096 / (ms * 1e-3) / 1e9 / hbm_peak, 4)
    del step
    torch.cuda.empty_cache()
    # config 3: causal prefill 4096 x 24/4 heads x 256
    L = 4096
    g = torch.Generator(device='cuda')
    g.manual_seed(3)
    q = torch.randn((L, H, HD), generator=g, device='cuda', dtype=torch.float16)
    k = torch.randn((L, HKV, HD), generator=g, device='cuda', dtype=torch.float16)
    v = torch.randn((L, HKV, HD), generator=g, device='cuda', dtype=torch.float16)
    out = torch.empty((L, H, HD), device='cuda', dtype=torch.float32)
    for _ in range(3):
        hot.prefill_attention(out, q, k, v, L)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(10):
        hot.prefill_attention(out, q, k, v, L)
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / 10
    flops = 4 * H * HD * (L * (L + 1) // 2)
    res['prefill_us'] = round(ms * 1e3, 2)
    res['prefill_tflops'] = round(flops / (ms * 1e-3) / 1e12, 1)
    res['prefill_tensor_frac'] = round(flops / (ms * 1e-3) / 1e12 / tc_peak, 4)
    # config 4: DeltaNet prefill core (4096 tokens)
    qd = torch.randn((L, HK, DK), generator=g, device='cuda', dtype=torch.float16)
    kd = torch.randn((L, HK, DK), generator=g, device='cuda', dtype=torch.float16)
    vd = torch.randn((L, HV, DK), generator=g, device='cuda', dtype=torch.float16)
    al = torch.randn((L, HV), generator=g, device='cuda')
    be = torch.randn((L, HV), generator=g, device='cuda')
    dec = torch.full((HV,), -1.0, device='cuda')
    bia = torch.zeros(HV, device='cuda')
    st = torch.zeros((HV, DK, DK), device='cuda')
    od = torch.empty((L, HV, DK), device='cuda')
    ws = torch.empty(hot.lib.qv_delta_chunked_workspace(L, HV), dtype=torch.uint8, device='cuda')
    for _ in range(3):
        st.zero_()
        hot.delta_chunked(od, st, qd, kd, vd, al, be, dec, bia, L, HK, HV, DK, workspace=ws)
    t_zero = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t_zero[0].record()
    for _ in range(10):
        st.zero_()
    t_zero[1].record()
    e0.record()
    for _ in range(10):
        st.zero_()
        hot.delta_chunked(od, st, qd, kd, vd, al, be, dec, bia, L, HK, HV, DK, workspace=ws)
    e1.record()
    torch.cuda.synchronize()
    ms = (e0.elapsed_time(e1) - t_zero[0].elapsed_time(t_zero[1])) / 10
    # chunked WY form per value head and chunk: 10 C^2 D + 6 C D^2 + 2/3 C^3 (C = 64, D = 128)
    C = 64
    gdn_flops = (10 * C * C * DK + 6 * C * DK * DK + 2 * C ** 3 / 3) * (L // C) * HV
    res['delta_prefill_4096_us'] = round(ms * 1e3, 2)
    res['delta_prefill_tflops'] = round(gdn_flops / (ms * 1e-3) / 1e12, 1)
    res['delta_prefill_tensor_frac'] = round(gdn_flops / (ms * 1e-3) / 1e12 / tc_peak, 4)
    e0.record()
    st.zero_()
    hot.delta_core(od, st, qd, kd, vd, al, be, dec, bia, L, HK, HV, DK)
    e1.record()
    torch.cuda.synchronize()
    res['delta_prefill_4096_recurrent_us'] = round(e0.elapsed_time(e1) * 1e3, 2)
    del ws, qd, kd, vd, od
    # the layer-level prefills with the reference's layer semantics at 4096 tokens: the DeltaNet layer
    # (conv + SiLU, norms, chunked recurrence, gated RMSNorm: qv_delta_prefill) and the attention layer
    # (RMSNorm + rotary + fp16 append, PRECISE causal attention, gate: qv_attention's prefill regime)
    C_ = (2 * HK + HV) * DK
    f32 = dict(device='cuda', dtype=torch.float32)
    lp = dict(state=torch.zeros((HV, DK, DK), **f32), history=torch.zeros((3, C_), **f32),
              qkv=torch.randn((L, C_), generator=g, **f32), gate=torch.randn((L, HV, DK), generator=g, **f32),
              alpha=torch.randn((L, HV), generator=g, **f32), beta=torch.randn((L, HV), generator=g, **f32),
              conv=torch.randn((C_, 4), generator=g, **f32) * 0.5, decay=dec, bias=bia, norm=torch.ones(DK, **f32))
    lout = torch.empty((L, HV, DK), **f32)
    lws = torch.empty(hot.lib.qv_delta_prefill_workspace(L, HK, HV), dtype=torch.uint8, device='cuda')
    for _ in range(2):
        hot.delta_prefill(lout, **lp, tokens=L, key_heads=HK, value_heads=HV, dim=DK, workspace=lws)
    e0.record()
    for _ in range(5):
        hot.delta_prefill(lout, **lp, tokens=L, key_heads=HK, value_heads=HV, dim=DK, workspace=lws)
    e1.record()
    torch.cuda.synchronize()
    res['delta_layer_prefill_4096_us'] = round(e0.elapsed_time(e1) / 5 * 1e3, 2)
    del lp, lout, lws
    kc = torch.zeros((L, HKV, HD), device='cuda', dtype=torch.float16)
    vc = torch.zeros_like(kc)
    qg = torch.randn((L, H, 2 * HD), generator=g, **f32)
    ky = torch.randn((L, HKV, HD), generator=g, **f32)
    vl = torch.randn((L, HKV, HD), generator=g, **f32)
    ao = torch.empty((L, H, HD), **f32)
    ones = torch.ones(HD, **f32)
    aws = torch.zeros(hot.lib.qv_attention_workspace(L, 0), dtype=torch.uint8, device='cuda')
    for _ in range(2):
        hot.attention(ao, kc, vc, qg, ky, vl, ones, ones, L, 0, workspace=aws)
    e0.record()
    for _ in range(5):
        hot.attention(ao, kc, vc, qg, ky, vl, ones, ones, L, 0, workspace=aws)
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / 5
    res['attention_layer_prefill_4096_us'] = round(ms * 1e3, 2)
    res['attention_layer_prefill_tflops'] = round(flops / (ms * 1e-3) / 1e12, 1)
    del kc, vc, qg, ky, vl, ao, aws
    # verify/commit transaction: 48 DeltaNet layers with distinct states,
    # plain layer vs recorded verify, and the commit of 3 of 8 tokens, each replayed as a graph
    T8, C_ = 8, (2 * HK + HV) * DK
    f32 = dict(device='cuda', dtype=torch.float32)
    layers = [dict(state=torch.randn((HV, DK, DK), generator=g, **f32) * 0.02, history=torch.zeros((3, C_), **f32),
                   saved_state=torch.empty((HV, DK, DK), **f32), saved_history=torch.empty((3, C_), **f32),
                   trace=torch.empty(int(hot.lib.qv_delta_trace_floats(HK, HV, DK)), **f32)) for _ in range(48)]
    conv = torch.zeros((C_, 4), **f32)
    conv[:, 3] = 1
    ins = (torch.randn((T8, C_), generator=g, **f32), torch.randn((T8, HV, DK), generator=g, **f32),
           torch.randn((T8, HV), generator=g, **f32), torch.randn((T8, HV), generator=g, **f32), conv,
           dec, bia, torch.ones(DK, **f32))
    outd = torch.empty((T8, HV, DK), **f32)

    def plain():
        for d in layers:
            hot.delta(outd, d['state'], d['history'], *ins, T8, HK, HV, DK)

    def verify():
        for d in layers:
            hot.delta_verify(outd, d['state'], d['history'], *ins, T8, HK, HV, DK,
                             d['saved_state'], d['saved_history'], d['trace'])

    def commit():
        for d in layers:
            hot.delta_commit(d['state'], d['history'], d['saved_state'], d['saved_history'], d['trace'], 3, T8,
                             HK, HV, DK)

    for name, fn in (('delta_layer_us', plain), ('delta_verify_record_us', verify), ('delta_commit_3of8_us', commit)):
        graph = capture(torch, fn)
        for _ in range(3):
            graph.replay()
        e0.record()
        for _ in range(5):
            graph.replay()
        e1.record()
        torch.cuda.synchronize()
        res[name] = round(e0.elapsed_time(e1) / (5 * 48) * 1e3, 2)
        graph.reset()
        del graph
    del layers
    # quantized projections: verify batch of 8 through a 17408 x 5120
    # matrix (the model's FFN shape), four distinct matrices in rotation (> L2)
    for kind, name in ((8, 'q8_0'), (12, 'q4_k'), (14, 'q6_k')):
        wbytes = int(hot.lib.qv_mm_weight_bytes(kind, 5120, 17408))
        mats = [torch.randint(0, 256, (wbytes,), generator=g, device='cuda', dtype=torch.uint8) for _ in range(4)]
        for m_ in mats:                     # finite fp16 block scales (first header bytes of each block)
            blk = 34 if kind == 8 else (144 if kind == 12 else 210)
            v = m_.view(-1, blk)
            scale = torch.tensor([0x00, 0x20] if kind != 14 else [0x00, 0x1c], dtype=torch.uint8, device='cuda')
            if kind == 14:
                v[:, 208:210] = scale
            else:
                v[:, 0:2] = scale
                if kind == 12:
                    v[:, 2:4] = scale
        xq = torch.randn((8, 5120), generator=g, device='cuda')
        oq = torch.empty((8, 17408), device='cuda')
        for _ in range(3):
            hot.mm(oq, mats[0], xq, kind, 8, 5120, 17408)
        e0.record()
        for i in range(20):
            hot.mm(oq, mats[i % 4], xq, kind, 8, 5120, 17408)
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / 20
        byt = wbytes + 8 * 5120 * 4 + 8 * 17408 * 4
        res[f'mm_{name}_17408x5120_t8_us'] = round(ms * 1e3, 2)
        res[f'mm_{name}_hbm_frac'] = round(byt / (ms * 1e-3) / 1e9 / hbm_peak, 4)
        del mats
    # checkpoint / restore: one attention layer's valid K and V prefix at
    # context 139,264 plus the 48 DeltaNet states and histories, as one span list
    P_ = 139264 - 8
    srcs = [torch.empty(P_ * HKV * HD * 2, dtype=torch.uint8, device='cuda') for _ in range(2)]
    srcs += [torch.empty(HV * DK * DK * 4 + 3 * C_ * 4, dtype=torch.uint8, device='cuda') for _ in range(48)]
    dsts = [torch.empty_like(t) for t in srcs]
    pairs = list(zip(dsts, srcs))
    for _ in range(3):
        hot.copy_spans(pairs)
    e0.record()
    for _ in range(10):
        hot.copy_spans(pairs)
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / 10
    nbytes = sum(t.numel() for t in srcs)
    res['checkpoint_spans'] = len(pairs)
    res['checkpoint_mb'] = round(nbytes / 1e6, 1)
    res['checkpoint_us'] = round(ms * 1e3, 2)
    res['checkpoint_hbm_frac'] = round(2 * nbytes / (ms * 1e-3) / 1e9 / hbm_peak, 4)
    del srcs, dsts, pairs
    return res


# ----------------------------------------------------------------------------- CPU
class CpuStep:
    """The same verify step on the host cores: the C restatement of the oracle (float64,
    oracle/c/qv_oracle.c, pinned to the reference's cpu_reference.py outputs by the tests),
    16 attention layers at the full context + 48 DeltaNet layers, every layer computed.

    The 16 attention layers share one prefix cache (570 MB of fp16 at context 139,264; every
    layer streams all of it, as a layer with its own cache would), each with its own inputs; the
    48 DeltaNet layers keep their own float64 states."""

    def __init__(self, context, tokens, threads, seed=4321):
        from oracle import inputs as I
        from oracle import native
        native.build()
        self.native, self.T, self.threads = native, tokens, threads
        self.position = context - tokens
        a = I.attention_layer(batch=tokens, position=self.position, seed=seed)
        n = context
        self.kc = np.zeros((n, HKV, HD), np.float16)
        self.vc = np.zeros_like(self.kc)
        self.kc[:self.position] = a['key_cache'][:self.position]
        self.vc[:self.position] = a['value_cache'][:self.position]
        rng = np.random.default_rng(seed)
        self.attn = [dict(q_gate=rng.standard_normal((tokens, H, 2 * HD), dtype=np.float32),
                          key=rng.standard_normal((tokens, HKV, HD), dtype=np.float32),
                          value=rng.standard_normal((tokens, HKV, HD), dtype=np.float32)) for _ in range(16)]
        self.ones = np.ones(HD, np.float32)
        self.delta = [I.delta_layer(batch=tokens, seed=seed + 1 + i) for i in range(48)]
        for d in self.delta:
            d['state'] = np.asarray(d['state'], np.float64).reshape(-1).copy()
            d['history'] = np.asarray(d['history'], np.float64).reshape(-1).copy()

    def run(self):
        """One step (the state and history of every DeltaNet layer advance, as on the GPU)."""
        nat, T = self.native, self.T
        for layer in range(LAYERS):
            if layer % 4 == 3:
                x = self.attn[layer // 4]
                nat.attention(self.kc, self.vc, x['q_gate'], x['key'], x['value'], self.ones, self.ones, T,
                              self.position, 1e-6, threads=self.threads, caches_in_place=True)
            else:
                d = self.delta[layer - layer // 4 - 1]
                _, d['state'], d['history'] = nat.delta(**d, threads=self.threads)

    def time_config(self, which):
        """Single-threaded time of BASELINE configuration 0 (attention, context 136) or 1 (DeltaNet)."""
        from oracle import inputs as I
        nat = self.native
        c = I.attention_layer(batch=8, position=128) if which == 0 else I.delta_layer(batch=8)
        fn = (lambda: nat.attention(**c, threads=1)) if which == 0 else (lambda: nat.delta(**c, threads=1))
        fn()
        t = time.perf_counter()
        reps = 20
        for _ in range(reps):
            fn()
        return (time.perf_counter() - t) / reps


def host_threads():
    return len(os.sched_getaffinity(0)) if hasattr(os, 'sched_getaffinity') else (os.cpu_count() or 1)


def cpu_baseline(context, tokens):
    """One full step of the C restatement on all host threads (no sampling, no scaling), and the
    single-threaded times of configurations 0 and 1."""
    threads = host_threads()
    step = CpuStep(context, tokens, threads)
    step.run()                                   # warm (page-in of the cache, thread start-up)
    t = time.perf_counter()
    step.run()
    seconds = time.perf_counter() - t
    return {'value': round(seconds * 1e6, 1), 'unit': UNIT, 'cores': threads, 'kind': 'port',
            'sample': f'one whole step: 16 attention layers at context {context} (verify-{tokens}) + 48 '
                      f'DeltaNet layers, float64 C restatement of cpu_reference.py on {threads} host threads '
                      f'(host has {os.cpu_count()} cpus)',
            'configs_single_thread_us': {'cfg0_attention_ctx136': round(step.time_config(0) * 1e6, 1),
                                         'cfg1_deltanet': round(step.time_config(1) * 1e6, 1)}}


def bench_reference(args):
    """The reference arm: the path's CPU implementation (the C restatement of the reference's
    cpu_reference.py; the reference's own is Python, which does not travel to the GPU box) timed
    on whole steps: args.warmup untimed steps, then args.steps timed ones, all on rank 0."""
    rank = int(os.environ.get('RANK', 0))
    if rank != 0:
        return
    threads = host_threads()
    step = CpuStep(args.context, args.tokens, threads)
    for _ in range(args.warmup):
        step.run()
    times = []
    for _ in range(args.steps):
        t = time.perf_counter()
        step.run()
        times.append(time.perf_counter() - t)
    value = statistics.mean(times) * 1e6
    line = {
        'metric': METRIC, 'value': round(value, 1), 'unit': UNIT, 'n_gpus': int(os.environ.get('WORLD_SIZE', 1)),
        'steps': args.steps, 'warmup': args.warmup, 'ms_per_step': round(value / 1e3, 3),
        'higher_is_better': False, 'scaling': 'strong', 'vs_baseline': None, 'dtype': 'f64',
        'data': 'synthetic (seeded N(0,1) fp16 KV, N(0,0.02) DeltaNet state)', 'impl': 'reference',
        'config': {'workload': f'verify-{args.tokens} hot-path step of the 64-layer model: 16 attention '
                               f'layers at context {args.context} + 48 gated-DeltaNet layers',
                   'context': args.context, 'verify_tokens': args.tokens},
        'cpu_baseline': {'value': round(value, 1), 'unit': UNIT, 'cores': threads, 'kind': 'port',
                         'sample': f'whole steps ({args.warmup} warm-up + {args.steps} timed, all run): the float64 '
                                   f'C restatement of the reference cpu_reference.py (oracle/c/qv_oracle.c) on '
                                   f'{threads} host threads; the reference itself is Python and does not travel'},
        'timed_seconds': round(sum(times), 2),
        'e2e': {'value': round(value, 1), 'unit': UNIT, 'h2d_bytes_per_step': 0, 'd2h_bytes_per_step': 0},
    }
    emit(line)


def main():
    args = parse()
    # Only the result line goes to stdout: anything libraries print there
    # (e.g. NCCL's version banner) is sent to stderr instead.
    global RESULT_OUT
    sys.stdout.flush()
    RESULT_OUT = os.fdopen(os.dup(1), 'w')
    os.dup2(2, 1)
    if args.impl == 'reference':
        bench_reference(args)
    else:
        bench_b200(args)


if __name__ == '__main__':
    main()
