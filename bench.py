#!/usr/bin/env python
"""Benchmark: routed-expert FFN prefill (2048-token chunk x 40 layers, W8A16).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One step = one 2048-token prefill chunk through 40 MoE expert layers
(256 experts top-8 + 1 shared expert, hidden 2048, intermediate 512, INT8
group-128 weights with FP32 scales, bf16 activations, Zipf(1.1)-biased
routing), every layer through ``gpu_routes.moe_block`` (routing metadata,
gate_up GEMM + SwiGLU, down GEMM + routing weight, ordered combine with the
gated shared expert and the residual add).  All 40 layers' weights (33.2 GB)
stay resident, so each step streams ~18 GB of distinct expert weights: the
inputs are larger than L2 and no L2 flush is needed.

Prints one JSON line (rank 0).  ``value`` = tokens/s over the whole job with
inputs resident in HBM; ``e2e`` = the same through the public API with the
step's inputs (hidden states, routing ids and weights for every layer) copied
from pinned host memory and the final hidden states copied back inside the
timed region.  ``--impl reference`` times the reference's CPU path (the HF
experts loop on fp32-dequantised weights) on the host cores instead.
"""
import argparse
import json
import os
import subprocess
import sys
import threading
import time

import numpy as np
import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

HIDDEN, INTER, EXPERTS, TOP = 2048, 512, 256, 8
EXPERT_BYTES = 3 * INTER * HIDDEN + 3 * INTER * HIDDEN // 128 * 4  # 3,244,032
METRIC = 'expert-FFN prefill tok/s (2048-chunk x 40 layers, W8A16)'
UNIT = 'tok/s'
# Kernels launched per layer of the step: meta_count_kernel, meta_scan_kernel,
# meta_place_kernel (routing metadata), permute_rows_kernel, grouped_ts_kernel<.., false>
# (gate_up + SwiGLU), grouped_ts_kernel<.., true> (down + routing weight), moe_combine_kernel.
LAUNCHES_PER_LAYER = 7
# expert-parallel layer: the owner's routed block (as above), the shared-only block (top 0:
# no per-chunk count or placement, 5 launches), the dispatch-row pack and unpack kernels
EP_LAUNCHES_PER_LAYER = LAUNCHES_PER_LAYER + 5 + 2
# DRAM bytes (read + write) of the two grouped-GEMM launches of one 2048-token layer, from one
# `ncu --set full` capture (`python bench.py --layers 2 --steps 1 --warmup 1 --no-cpu-baseline
# --no-extra`, -k regex:grouped_ts -s 2 -c 2): gate_up 404.2 MB + down 244.1 MB.  Per-layer
# work does not depend on the layer count, so no scaling is applied.
NCU_TRAFFIC_PER_LAYER = 648.3e6
NCU_TRAFFIC_SOURCE = ('ncu dram__bytes_read.sum + dram__bytes_write.sum, gate_up + down launches of one '
                      '2048-token layer; bytes per layer like alg_bytes_per_layer')


def parse(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument('--gpus', type=int, default=1)
    ap.add_argument('--steps', type=int, default=50)
    ap.add_argument('--warmup', type=int, default=5)
    ap.add_argument('--impl', choices=('ours', 'reference'), default='ours')
    ap.add_argument('--layers', type=int, default=40)
    ap.add_argument('--tokens', type=int, default=2048)
    ap.add_argument('--no-cpu-baseline', action='store_true')
    ap.add_argument('--seed', type=int, default=0)
    ap.add_argument('--no-extra', action='store_true', help='skip the decode (C3) and dense-sweep (C4) legs')
    ap.add_argument('--ep', action='store_true', help='with --gpus N > 1: expert parallelism (experts sharded, '
                                                      'all-to-all) instead of N data-parallel replicas')
    ap.add_argument('--ep-wire', choices=('bf16', 'int8'), default='bf16',
                    help='with --ep: format of the dispatched hidden rows (int8 = W8A8 activation '
                         'quantisation, 2112 instead of 4096 bytes per row)')
    return ap.parse_args(argv)


# ------------------------------------------------------------------ distributed
def dist_setup(n):
    rank = int(os.environ.get('RANK', '0'))
    world = int(os.environ.get('WORLD_SIZE', '1'))
    local = int(os.environ.get('LOCAL_RANK', '0'))
    if world != n:
        raise SystemExit(f'--gpus {n} but WORLD_SIZE={world}')
    if world > 1:
        import datetime
        torch.cuda.set_device(local)
        torch.distributed.init_process_group('nccl', timeout=datetime.timedelta(seconds=120))
    else:
        torch.cuda.set_device(0)
    return rank, world, local


def barrier(world):
    if world > 1:
        torch.distributed.barrier()


def max_over_ranks(v, world):
    if world == 1:
        return v
    t = torch.tensor([v], dtype=torch.float64, device='cuda')
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return float(t.item())


# ------------------------------------------------------------------ clocks
class ClockSampler:
    """nvidia-smi samples of this GPU while the timed region runs."""
    FIELDS = ('clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,'
              'clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,'
              'clocks_event_reasons.sw_power_cap')

    def __init__(self, index):
        self.index, self.rows, self.proc = index, [], None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ['nvidia-smi', '-i', str(self.index), f'--query-gpu={self.FIELDS}', '--format=csv,noheader,nounits',
                 '-lms', '100'], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
            time.sleep(0.25)
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(',')]
            if len(parts) == 7:
                self.rows.append(parts)

    def __exit__(self, *a):
        if self.proc is not None:
            time.sleep(0.15)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        if not self.rows:
            return {'sm_mhz': None, 'sm_max_mhz': None, 'reasons': ['no samples']}
        sm = np.array([float(r[0]) for r in self.rows])
        mx = float(self.rows[0][1])
        power = np.array([float(r[2]) for r in self.rows if r[2] not in ('[N/A]', '')] or [0.0])
        names = ('hw_slowdown', 'hw_thermal_slowdown', 'sw_thermal_slowdown', 'sw_power_cap')
        reasons = sorted({n for r in self.rows for n, v in zip(names, r[3:]) if v.lower() == 'active'})
        return {'sm_mhz': float(np.median(sm)), 'sm_max_mhz': mx, 'reasons': reasons,
                'samples': len(self.rows), 'power_w_max': float(power.max())}


# ------------------------------------------------------------------ workload
def quantize_gpu(w):
    """convert.quantize (convert.py:31-37) on the GPU: per-128 absmax / 127."""
    v = w.reshape(*w.shape[:-1], w.shape[-1] // 128, 128)
    s = v.abs().amax(-1).div(127).clamp_min(1e-30)
    q = (v / s.unsqueeze(-1)).round().clamp(-127, 127).to(torch.int8)
    return q.reshape(w.shape).contiguous(), s.contiguous()


def make_layers(layers, dev, seed, experts=EXPERTS):
    """Per layer: the routed bank (``experts`` experts: all 256, or this rank's shard
    under expert parallelism), the shared expert and its gate."""
    g = torch.Generator(device=dev).manual_seed(seed)
    out = []
    for _ in range(layers):
        qg, sg = quantize_gpu(torch.randn((experts, 2 * INTER, HIDDEN), generator=g, device=dev) * 0.02)
        qd, sd = quantize_gpu(torch.randn((experts, HIDDEN, INTER), generator=g, device=dev) * 0.02)
        shared = [quantize_gpu(torch.randn(s, generator=g, device=dev) * 0.02)
                  for s in ((INTER, HIDDEN), (INTER, HIDDEN), (HIDDEN, INTER))]
        gate = (torch.randn((1, HIDDEN), generator=g, device=dev) * 0.02).bfloat16()
        out.append(((qg, sg, qd, sd), shared, gate))
    return out


def make_routing(layers, tokens, dev, seed):
    g = torch.Generator(device=dev).manual_seed(seed + 1)
    ids, wts = [], []
    for _ in range(layers):
        ranks = torch.randperm(EXPERTS, generator=g, device=dev).float() + 1
        logits = torch.randn((tokens, EXPERTS), generator=g, device=dev) - 1.1 * torch.log(ranks)[None]
        p = torch.softmax(logits, dim=-1, dtype=torch.float32)
        w, i = torch.topk(p, TOP, dim=-1)
        w = w / w.sum(-1, keepdim=True)
        ids.append(i.contiguous())
        wts.append(w.contiguous())
    x = torch.randn((tokens, HIDDEN), generator=g, device=dev).bfloat16()
    return x, torch.stack(ids), torch.stack(wts)


def run_ours(a, rank, world, local):
    from localmoe35ba3b_b200 import _native
    from localmoe35ba3b_b200.runtime import ep, gpu_routes
    dev = torch.device('cuda', local)
    peaks = load_peaks()
    # N > 1: data-parallel replicas by default (all 40 layers' weights, 33.2 GB, fit on every
    # B200, and each GPU runs its own tokens); --ep shards the experts instead
    use_ep = world > 1 and a.ep
    e_loc = EXPERTS // world if use_ep else EXPERTS
    layers = make_layers(a.layers, dev, a.seed + 1000 * rank, e_loc)
    x0, ids, wts = make_routing(a.layers, a.tokens, dev, a.seed + 1000 * rank)
    active = [int(torch.unique(ids[l]).numel()) for l in range(a.layers)]
    if use_ep:
        fns = [(ep.gpu_local_moe(bank), ep.gpu_shared_part(bank, shared, gate)) for bank, shared, gate in layers]

    def step(x, ids, wts, events=None):
        if use_ep:
            # expert parallelism: this rank's experts serve every rank's routes to them
            for l in range(a.layers):
                x = ep.moe_forward(x, wts[l], ids[l], EXPERTS, fns[l][0], fns[l][1], residual=x, wire=a.ep_wire)
            return x
        for l, (bank, shared, gate) in enumerate(layers):
            x = gpu_routes.moe_block(x, wts[l], ids[l], bank, shared=shared, shared_gate_weight=gate,
                                     residual=x, stage_events=None if events is None else events[l])
        return x

    for _ in range(a.warmup):
        step(x0, ids, wts)
    torch.cuda.synchronize()
    _native.check_device_errors(dev)

    # ---- timed region: inputs resident in HBM
    timed_with_events = 0 if use_ep else min(a.steps, 10)
    evs = [[[torch.cuda.Event(enable_timing=True) for _ in range(5)] for _ in range(a.layers)]
           for _ in range(timed_with_events)]
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(world)
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        start.record()
        for k in range(a.steps):
            step(x0, ids, wts, evs[k] if k < timed_with_events else None)
        end.record()
        torch.cuda.synchronize()
    barrier(world)
    ms = max_over_ranks(start.elapsed_time(end), world)
    _native.check_device_errors(dev)
    ms_step = ms / a.steps
    value = world * a.tokens * a.steps / (ms / 1e3)

    # per-stage times from the events recorded inside the timed region
    st = np.zeros(4)
    for k in range(timed_with_events):
        for l in range(a.layers):
            e = evs[k][l]
            st += [e[i].elapsed_time(e[i + 1]) for i in range(4)]
    if timed_with_events:
        st /= timed_with_events * a.layers  # ms per layer
        gemm_ms = st[1] + st[2]
    else:
        # expert parallelism: no per-launch events across the exchange; the whole layer
        gemm_ms = ms_step / a.layers
    routes = a.tokens * TOP
    rows = routes + a.tokens
    flops = 2.0 * rows * 3 * INTER * HIDDEN  # gate_up + down, routed + shared
    act_bytes = a.tokens * HIDDEN * 2 + 2 * rows * INTER * 2 + rows * HIDDEN * 2
    wbytes = (float(np.mean(active)) / (world if use_ep else 1) + 1) * EXPERT_BYTES
    gemm_bytes = wbytes + act_bytes
    tflops = flops / (gemm_ms / 1e3) / 1e12
    gbs = gemm_bytes / (gemm_ms / 1e3) / 1e9
    pk_tc, pk_tc_src = peaks['tc_sustained'], peaks['src']
    pk_hbm = peaks['hbm']
    t_tc, t_hbm = flops / (pk_tc * 1e12), gemm_bytes / (pk_hbm * 1e9)
    bound = 'tensor' if t_tc >= t_hbm else 'hbm'
    if bound == 'tensor':
        roof = {'bound': 'tensor', 'achieved': round(tflops, 1), 'peak': pk_tc, 'unit': 'TFLOP/s',
                'frac': round(tflops / pk_tc, 4)}
    else:
        roof = {'bound': 'hbm', 'achieved': round(gbs, 1), 'peak': pk_hbm, 'unit': 'GB/s',
                'frac': round(gbs / pk_hbm, 4)}
    roof.update({'traffic': None if use_ep else NCU_TRAFFIC_PER_LAYER,
                 'traffic_source': 'not captured for the expert-parallel step' if use_ep else NCU_TRAFFIC_SOURCE,
                 'kernel': ('whole expert-parallel layer (all-to-all + local experts + shared + combine), per rank'
                            if use_ep else 'grouped GEMMs (gate_up+SwiGLU, down+weight) per layer'),
                 'peak_source': pk_tc_src, 'flops_per_layer': flops, 'alg_bytes_per_layer': round(gemm_bytes),
                 'tensor_frac': round(tflops / pk_tc, 4), 'hbm_frac': round(gbs / pk_hbm, 4),
                 'gemm_us_per_layer': round(gemm_ms * 1e3, 2),
                 'stage_us_per_layer': {'route_meta': round(st[0] * 1e3, 2), 'gate_up': round(st[1] * 1e3, 2),
                                        'down': round(st[2] * 1e3, 2), 'combine': round(st[3] * 1e3, 2)}})

    # ---- end to end through the public API with host buffers
    xh = x0.cpu().pin_memory()
    idh = ids.cpu().pin_memory()
    wh = wts.cpu().pin_memory()
    outh = torch.empty_like(xh).pin_memory()
    xd, idd, wd = torch.empty_like(x0), torch.empty_like(ids), torch.empty_like(wts)

    def e2e_step():
        xd.copy_(xh, non_blocking=True)
        idd.copy_(idh, non_blocking=True)
        wd.copy_(wh, non_blocking=True)
        y = step(xd, idd, wd)
        outh.copy_(y, non_blocking=True)

    e2e_step()
    torch.cuda.synchronize()
    e_steps = max(3, a.steps // 2)
    barrier(world)
    torch.cuda.synchronize()
    s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s2.record()
    for _ in range(e_steps):
        e2e_step()
    e2.record()
    torch.cuda.synchronize()
    barrier(world)
    ms_e2e = max_over_ranks(s2.elapsed_time(e2), world)
    e2e = {'value': round(world * a.tokens * e_steps / (ms_e2e / 1e3), 1), 'unit': UNIT,
           'h2d_bytes_per_step': int(xh.numel() * 2 + idh.numel() * 8 + wh.numel() * 4),
           'd2h_bytes_per_step': int(outh.numel() * 2)}

    cpu = None
    if rank == 0 and world == 1 and not a.no_cpu_baseline:
        cpu = cpu_baseline_leg()
    extra = {}
    if not a.no_extra and world == 1:
        extra['c3_decode'] = decode_leg(layers, dev, peaks, max(3, a.steps), a.warmup, a.seed + 1000 * rank)
        extra['c4_dense'] = dense_leg(dev, peaks)

    line = {
        'metric': METRIC, 'value': round(value, 1), 'unit': UNIT, 'n_gpus': world, 'steps': a.steps,
        'warmup': a.warmup, 'ms_per_step': round(ms_step, 4), 'higher_is_better': True, 'scaling': 'weak',
        'vs_baseline': None, 'dtype': 'bf16', 'data': 'synthetic (seeded random-init INT8 weights, N(0,1) inputs)',
        'config': {'workload': workload(a),
                   'tokens_per_gpu': a.tokens, 'layers': a.layers,
                   'parallelism': (f'ep{world} (experts {e_loc} per GPU, all-to-all over NCCL, '
                                   f'{a.ep_wire} dispatch rows)' if use_ep
                                   else (f'dp{world} replicas (full weights per GPU; --ep for expert parallelism)'
                                         if world > 1 else 'single')),
                   'active_experts_mean': round(float(np.mean(active)), 1),
                   'l2': 'inputs larger than L2 (33.2 GB of resident expert weights per GPU)'},
        'roofline': roof, 'cpu_baseline': cpu, 'e2e': e2e,
        'gpu_launches': (EP_LAUNCHES_PER_LAYER if use_ep else LAUNCHES_PER_LAYER) * a.layers * a.steps,
        'clocks': clk.summary(),
    }
    if extra:
        line['extra'] = extra
    if rank == 0:
        print(json.dumps(line), flush=True)


def decode_leg(layers, dev, peaks, steps, warmup, seed):
    """C3: one-token decode through all layers (W8A8 routed experts + W8A16 shared
    expert + gate + residual), captured once in a CUDA graph and replayed; per-layer
    time and the HBM roofline of its 9 x 3,244,032 weight bytes."""
    from localmoe35ba3b_b200.runtime import decode
    g = torch.Generator(device=dev).manual_seed(seed + 7)
    L = len(layers)
    ids, wts = [], []
    for _ in range(L):
        ranks = torch.randperm(EXPERTS, generator=g, device=dev).float() + 1
        logits = torch.randn((1, EXPERTS), generator=g, device=dev) - 1.1 * torch.log(ranks)[None]
        p = torch.softmax(logits, dim=-1, dtype=torch.float32)
        w, i = torch.topk(p, TOP, dim=-1)
        ids.append(i.contiguous())
        wts.append((w / w.sum(-1, keepdim=True)).contiguous())
    x0 = torch.randn((1, HIDDEN), generator=g, device=dev).bfloat16()

    def step():
        x = x0
        for l, (bank, shared, gate) in enumerate(layers):
            x = decode.decode_block(x, wts[l], ids[l], bank, shared=shared, shared_gate_weight=gate, residual=x)
        return x

    s = torch.cuda.Stream(dev)
    s.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(s):
        for _ in range(2):
            step()
    torch.cuda.current_stream(dev).wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step()
    for _ in range(warmup):
        graph.replay()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record()
    for _ in range(steps):
        graph.replay()
    e1.record()
    torch.cuda.synchronize()
    us_layer = e0.elapsed_time(e1) * 1e3 / (steps * L)
    del graph
    wbytes = 9 * EXPERT_BYTES
    gbs = wbytes / (us_layer * 1e-6) / 1e9
    return {'us_per_layer': round(us_layer, 2), 'tok_per_s': round(1e6 / (us_layer * L), 1),
            'weight_bytes_per_layer': wbytes, 'achieved_gbs': round(gbs, 1), 'peak_gbs': peaks['hbm'],
            'hbm_frac': round(gbs / peaks['hbm'], 4), 'launches_per_layer': 2,
            'workload': f'1 token x {L} layers, 8 routed (W8A8) + shared (W8A16) experts, one CUDA graph',
            'l2': f'{L} layers of weights ({L * 9 * EXPERT_BYTES / 1e9:.2f} GB touched per step) exceed L2'}


def _graph_time(fn, iters, dev):
    """Device time per call of fn(i), i = 0..iters-1, captured in one CUDA graph (so
    host launch overhead between the calls is not timed) and replayed after warm-up."""
    s = torch.cuda.Stream(dev)
    s.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(s):
        for i in range(3):
            fn(i)
    torch.cuda.current_stream(dev).wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for i in range(iters):
            fn(i)
    g.replay()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record()
    g.replay()
    e1.record()
    torch.cuda.synchronize()
    del g
    return e0.elapsed_time(e1) * 1e3 / iters


def dense_leg(dev, peaks, iters=20):
    """C4: W8A16 dense linear sweep K=2048, N in {512,2048,4096,8192}, M in {1,16,256,2048}
    (and the W8A8 table GEMV at M=1).  Weight copies rotate so each iteration reads
    weights from HBM (the pool of copies exceeds L2)."""
    from localmoe35ba3b_b200.operators import int8 as I8
    from localmoe35ba3b_b200.operators import w8a8 as W8
    K = 2048
    out = []
    for n in (512, 2048, 4096, 8192):
        wb = n * K + n * (K // 128) * 4
        copies = max(2, -(-256 * 2 ** 20 // wb))
        qs = [torch.randint(-127, 128, (n, K), dtype=torch.int8, device=dev) for _ in range(copies)]
        ss = [torch.rand((n, K // 128), device=dev) * 1e-3 for _ in range(copies)]
        for m in (1, 16, 256, 2048):
            x = torch.randn((m, K), device=dev).bfloat16()
            us = _graph_time(lambda i: I8.linear(x, qs[i % copies], ss[i % copies]), iters, dev)
            flops = 2.0 * m * n * K
            bytes_ = wb + 2 * m * K + 2 * m * n
            tf, gbs = flops / (us * 1e-6) / 1e12, bytes_ / (us * 1e-6) / 1e9
            bound = 'tensor' if flops / (peaks['tc'] * 1e12) > bytes_ / (peaks['hbm'] * 1e9) else 'hbm'
            frac = tf / peaks['tc'] if bound == 'tensor' else gbs / peaks['hbm']
            out.append({'op': 'w8a16', 'M': m, 'N': n, 'K': K, 'us': round(us, 2), 'tflops': round(tf, 2),
                        'gbs': round(gbs, 1), 'bound': bound, 'frac': round(frac, 4)})
        # W8A8 at M=1: the table-driven GEMV over one descriptor row (the weight itself)
        x = torch.randn((1, K), device=dev).bfloat16()
        tabs = [torch.tensor([[q.data_ptr(), s.data_ptr(), q.data_ptr(), s.data_ptr(), 0]], dtype=torch.int64,
                             device=dev) for q, s in zip(qs, ss)]
        us = _graph_time(lambda i: W8.grouped_linear(x, tabs[i % copies], 1, n, 0, True), iters, dev)
        gbs = (wb + 2 * K + 2 * n) / (us * 1e-6) / 1e9
        out.append({'op': 'w8a8', 'M': 1, 'N': n, 'K': K, 'us': round(us, 2), 'gbs': round(gbs, 1), 'bound': 'hbm',
                    'frac': round(gbs / peaks['hbm'], 4)})
        del qs, ss, tabs
    return out


def load_peaks():
    p = os.path.join(ROOT, 'MEASURED_PEAKS.json')
    if os.path.exists(p):
        d = json.load(open(p))
        return {'hbm': float(d['hbm_gbs']), 'tc': float(d['bf16_tflops']),
                'tc_sustained': float(d.get('bf16_tflops_sustained', d['bf16_tflops'])),
                'src': 'measured (MEASURED_PEAKS.json, sustained bf16)'}
    return {'hbm': 6650.0, 'tc': 1590.0, 'tc_sustained': 1400.0, 'src': 'fallback'}


# ------------------------------------------------------------------ CPU legs
def cpu_baseline_leg(repeats=3):
    from oracle import cpu_baseline as C
    case = C.make_case(tokens=256)
    t, threads = C.time_layer(case, repeats=repeats)
    return {'value': round(256 / (t * 40), 2), 'unit': UNIT, 'cores': threads, 'kind': 'port',
            'sample': f'1 MoE layer (256 experts top-8 + shared), 256 tokens, torch fp32 dequantise-then-matmul '
                      f'(HF experts loop), median of {repeats}, scaled to 40 layers; CPU: {C.cpu_model()}'}


def workload(a):
    """The workload name both arms report in ``config``."""
    return (f'prefill chunk: {a.tokens} tokens x {a.layers} layers, 256 experts top-8 + shared, '
            'hidden 2048, moe_intermediate 512, INT8 g128 FP32 scales, Zipf(1.1) routing')


def run_reference(a, rank, world):
    if rank != 0:
        return
    from oracle import cpu_baseline as C
    case = C.make_case(tokens=256)
    for _ in range(a.warmup):
        C.time_layer(case, repeats=1)
    t0 = time.perf_counter()
    for _ in range(a.steps):
        t, threads = C.time_layer(case, repeats=1)
    wall = time.perf_counter() - t0
    # each step times one layer of 256 tokens; tok/s of the whole workload = 256 tokens
    # per (layer time x layers), and a workload step (a.tokens through a.layers) is
    # a.tokens / value seconds
    value = 256 * a.steps / (wall * a.layers)
    print(json.dumps({
        'impl': 'reference', 'metric': METRIC, 'value': round(value, 2), 'unit': UNIT, 'n_gpus': world,
        'steps': a.steps, 'warmup': a.warmup, 'ms_per_step': round(a.tokens / value * 1e3, 2),
        'higher_is_better': True, 'scaling': 'weak', 'vs_baseline': None, 'dtype': 'f32',
        'data': 'synthetic (seeded random-init INT8 weights, N(0,1) inputs)',
        'config': {'workload': workload(a), 'tokens_per_gpu': a.tokens, 'layers': a.layers,
                   'parallelism': 'host CPU (the oracle port of the reference path)',
                   'l2': 'not applicable (host CPU)'},
        'cpu_baseline': {'value': round(value, 2), 'unit': UNIT, 'cores': threads, 'kind': 'port',
                         'sample': f'256 tokens x 1 MoE layer per step, scaled to {a.layers} layers (HF experts '
                                   f'loop, fp32 dequantised weights, torch on {threads} host threads; CPU: '
                                   f'{C.cpu_model()})'},
        'e2e': {'value': round(value, 2), 'unit': UNIT, 'h2d_bytes_per_step': 0, 'd2h_bytes_per_step': 0},
    }), flush=True)


def main():
    a = parse()
    if a.impl == 'reference':
        rank = int(os.environ.get('RANK', '0'))
        run_reference(a, rank, a.gpus)
        return
    rank, world, local = dist_setup(a.gpus)
    try:
        run_ours(a, rank, world, local)
    finally:
        if world > 1:
            torch.distributed.destroy_process_group()


if __name__ == '__main__':
    main()
