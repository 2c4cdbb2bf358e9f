#!/usr/bin/env python
"""Benchmark: routed-expert FFN prefill through 40 MoE layers (W8A16).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

N = 1: one step = one 2048-token prefill chunk through 40 MoE
layers (256 experts top-8 + 1 shared expert, hidden 2048, intermediate 512, INT8
group-128 weights with FP32 scales, bf16 activations, Zipf(1.1)-biased routing),
every layer through ``gpu_routes.moe_block`` (routing metadata, gate_up GEMM +
SwiGLU, down GEMM + routing weight, ordered combine with the gated shared expert
and the residual add).  All 40 layers' weights (33.2 GB) stay resident, so each
step streams ~18 GB of distinct expert weights: the inputs are larger than L2 and
no L2 flush is needed.

N > 1 (torchrun): expert parallelism.  One step = 16,384 tokens
in total (``--total-tokens``; 16384 / N per GPU) through 40 layers whose 256
experts are sharded 256 / N per GPU; each layer is ``ep.GpuLayer.forward``
(dispatch kernels, an all-to-all over NCCL, the owner's experts + the shared
expert, the return all-to-all, the fold).  The total work is fixed as N grows
(strong scaling).  ``--dp`` runs N independent data-parallel replicas instead.

Prints one JSON line (rank 0).  ``value`` = tokens/s over the whole job with the
inputs resident in HBM (no per-stage events inside the timed region); the
per-stage times come from separate instrumented steps after it.  ``e2e`` = the
same through the public API with the step's inputs (hidden states, routing ids
and weights of all layers) copied from pinned host memory and the final hidden
states copied back inside the timed region.  ``--impl reference`` times the
reference's CPU path (the HF experts loop on fp32-dequantised weights) on the
host cores instead.
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
# Kernels launched per layer of the single-GPU step: meta_count_kernel, meta_scan_kernel,
# meta_place_kernel (routing metadata), permute_rows_kernel, grouped_ts_kernel<.., false>
# (gate_up + SwiGLU), grouped_ts_kernel<.., true> (down + routing weight), moe_combine_kernel.
LAUNCHES_PER_LAYER = 7
# expert-parallel layer: meta_count_kernel, meta_scan_kernel, meta_place_kernel (this rank's
# routes sorted by expert), ep_slots_kernel, ep_pack_kernel (dispatch), ep_owner_meta_kernel,
# ep_owner_scatter_kernel, the two grouped_ts_kernel launches, ep_owner_combine_kernel,
# ep_fold_kernel (+ two NCCL all-to-all kernels, not counted)
EP_LAUNCHES_PER_LAYER = 11
# DRAM bytes (read + write) of the two grouped-GEMM launches of one 2048-token layer, from one
# `ncu --set full` capture (`python bench.py --layers 2 --steps 1 --warmup 1 --no-cpu-baseline
# --no-extra`, -k regex:grouped_ts -s 2 -c 2): gate_up 404.2 MB + down 244.9 MB.  Per-layer
# work does not depend on the layer count, so no scaling is applied.
NCU_TRAFFIC_PER_LAYER = 649.1e6
NCU_TRAFFIC_SOURCE = ('ncu dram__bytes_read.sum + dram__bytes_write.sum, gate_up + down launches of one '
                      '2048-token layer; bytes per layer like alg_bytes_per_layer')


def parse(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument('--gpus', type=int, default=1)
    ap.add_argument('--steps', type=int, default=20)
    ap.add_argument('--warmup', type=int, default=5)
    ap.add_argument('--impl', choices=('ours', 'reference'), default='ours')
    ap.add_argument('--layers', type=int, default=40)
    ap.add_argument('--tokens', type=int, default=2048, help='tokens per GPU (single GPU, --dp)')
    ap.add_argument('--total-tokens', type=int, default=16384, help='tokens of the whole job (expert parallelism)')
    ap.add_argument('--stage-steps', type=int, default=3, help='instrumented steps after the timed region')
    ap.add_argument('--no-cpu-baseline', action='store_true')
    ap.add_argument('--seed', type=int, default=0)
    ap.add_argument('--no-extra', action='store_true', help='skip the decode (C3), dense (C4) and C5 1-GPU legs')
    ap.add_argument('--only', choices=('c3', 'c4', 'c5'), default=None,
                    help='run one extra leg alone (1 GPU; for profiling) and print its JSON')
    ap.add_argument('--dp', action='store_true', help='with --gpus N > 1: N data-parallel replicas (full weights '
                                                      'per GPU) instead of expert parallelism')
    ap.add_argument('--ep-transport', choices=('p2p', 'nccl'), default='p2p',
                    help='expert parallelism: rows stored straight into the peers\' buffers over NVLink (p2p) or '
                         'moved by NCCL all_to_all between the kernels')
    ap.add_argument('--ep-wire', choices=('bf16', 'int8'), default='bf16',
                    help='expert parallelism: format of the dispatched hidden rows (int8 = W8A8 activation '
                         'quantisation, 2112 instead of 4096 payload bytes per row)')
    return ap.parse_args(argv)


def use_ep(a, world):
    return world > 1 and not a.dp


def job_tokens(a, world):
    """(tokens of the whole job per step, tokens per GPU)."""
    if use_ep(a, world):
        if a.total_tokens % world:
            raise SystemExit(f'--total-tokens {a.total_tokens} is not divisible by {world} GPUs')
        return a.total_tokens, a.total_tokens // world
    return a.tokens * world, a.tokens


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
        torch.distributed.init_process_group('nccl', timeout=datetime.timedelta(seconds=120),
                                             device_id=torch.device('cuda', local))
    else:
        torch.cuda.set_device(0)
    return rank, world, local


def barrier(world):
    if world > 1:
        torch.distributed.barrier()


def max_over_ranks(v, world):
    if world == 1:
        return v
    t = torch.tensor(np.atleast_1d(np.asarray(v, dtype=np.float64)), device='cuda')
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    r = t.cpu().numpy()
    return float(r[0]) if np.ndim(v) == 0 else r


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


def make_layers(layers, dev, seed, experts=EXPERTS, shard=0):
    """Per layer: the routed bank (``experts`` experts: all 256, or shard ``shard`` of
    them under expert parallelism), the shared expert and its gate (the same on
    every rank)."""
    g = torch.Generator(device=dev).manual_seed(seed + 7919 * shard)
    gs = torch.Generator(device=dev).manual_seed(seed + 104729)
    out = []
    for _ in range(layers):
        qg, sg = quantize_gpu(torch.randn((experts, 2 * INTER, HIDDEN), generator=g, device=dev) * 0.02)
        qd, sd = quantize_gpu(torch.randn((experts, HIDDEN, INTER), generator=g, device=dev) * 0.02)
        shared = [quantize_gpu(torch.randn(s, generator=gs, device=dev) * 0.02)
                  for s in ((INTER, HIDDEN), (INTER, HIDDEN), (HIDDEN, INTER))]
        gate = (torch.randn((1, HIDDEN), generator=gs, device=dev) * 0.02).bfloat16()
        out.append(((qg, sg, qd, sd), shared, gate))
    return out


def make_routing(layers, tokens, dev, seed):
    """Per layer: router logits ~N(0,1) plus a Zipf(1.1) bias over a seeded permutation of
    the experts, softmax top-8 renormalised (HF's router tail); and the layer-0 input."""
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


def load_peaks():
    p = os.path.join(ROOT, 'MEASURED_PEAKS.json')
    if os.path.exists(p):
        d = json.load(open(p))
        return {'hbm': float(d['hbm_gbs']), 'tc': float(d['bf16_tflops']),
                'tc_sustained': float(d.get('bf16_tflops_sustained', d['bf16_tflops'])),
                'src': 'measured (MEASURED_PEAKS.json, sustained bf16)'}
    return {'hbm': 6650.0, 'tc': 1590.0, 'tc_sustained': 1400.0, 'src': 'fallback'}


def workload(a, world=1):
    """The workload name both arms report in ``config``."""
    total, per = job_tokens(a, world)
    if use_ep(a, world):
        return (f'expert-parallel prefill: {total} tokens x {a.layers} layers over {world} GPUs ({per} per GPU), '
                '256 experts top-8 + shared, hidden 2048, moe_intermediate 512, INT8 g128 FP32 scales, '
                'Zipf(1.1) routing')
    return (f'prefill chunk: {per} tokens x {a.layers} layers{f" per GPU x {world} replicas" if world > 1 else ""}'
            ', 256 experts top-8 + shared, hidden 2048, moe_intermediate 512, INT8 g128 FP32 scales, '
            'Zipf(1.1) routing')


def config(a, world):
    """``config`` of the JSON line, the same for both arms."""
    total, per = job_tokens(a, world)
    if use_ep(a, world):
        how = ('rows stored into the peers\' buffers over NVLink by the pack and combine kernels'
               if a.ep_transport == 'p2p' else 'all-to-all over NCCL')
        par = f'ep{world} (experts {EXPERTS // world} per GPU, {how}, {a.ep_wire} dispatch rows, fixed-size exchanges)'

    else:
        par = f'dp{world} replicas (full weights per GPU)' if world > 1 else 'single'
    return {'workload': workload(a, world), 'tokens': total, 'tokens_per_gpu': per, 'layers': a.layers,
            'parallelism': par, 'l2': 'inputs larger than L2 (every layer\'s expert weights resident in HBM, '
                                      'streamed once per step)'}


def scaling(a, world):
    return 'strong' if use_ep(a, world) else 'weak'


# ------------------------------------------------------------------ our arm
def run_ours(a, rank, world, local):
    from localmoe35ba3b_b200 import _native
    from localmoe35ba3b_b200.runtime import ep, gpu_routes
    dev = torch.device('cuda', local)
    peaks = load_peaks()
    ep_mode = use_ep(a, world)
    total, tokens = job_tokens(a, world)
    e_loc = EXPERTS // world if ep_mode else EXPERTS
    layers = make_layers(a.layers, dev, a.seed, e_loc, shard=rank if ep_mode else 0)
    x0, ids, wts = make_routing(a.layers, tokens, dev, a.seed + 1000 * rank)
    active = [int(torch.unique(ids[l]).numel()) for l in range(a.layers)]
    layer_ep = ep.GpuLayer(tokens, TOP, EXPERTS, world, HIDDEN, INTER, torch.bfloat16, dev, a.ep_wire,
                           transport=a.ep_transport) if ep_mode else None

    def step(x, ids, wts, events=None):
        for l, (bank, shared, gate) in enumerate(layers):
            ev = None if events is None else events[l]
            if ep_mode:
                x = layer_ep.forward(x, wts[l], ids[l], bank, shared, gate, residual=x, events=ev)
            else:
                x = gpu_routes.moe_block(x, wts[l], ids[l], bank, shared=shared, shared_gate_weight=gate,
                                         residual=x, stage_events=ev)
        return x

    for _ in range(a.warmup):
        step(x0, ids, wts)
    torch.cuda.synchronize()
    _native.check_device_errors(dev)

    # ---- timed region: inputs resident in HBM, no per-stage events
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(world)
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        start.record()
        for _ in range(a.steps):
            step(x0, ids, wts)
        end.record()
        torch.cuda.synchronize()
    barrier(world)
    ms = max_over_ranks(start.elapsed_time(end), world)
    _native.check_device_errors(dev)
    ms_step = ms / a.steps
    value = total * a.steps / (ms / 1e3)

    # ---- stage times: separate instrumented steps (events between the launches stop the
    #      programmatic-dependent-launch overlap, so they stay out of the timed region)
    nev = 6 if ep_mode else 5
    S = max(1, a.stage_steps)
    evs = [[[torch.cuda.Event(enable_timing=True) for _ in range(nev)] for _ in range(a.layers)] for _ in range(S)]
    barrier(world)
    for k in range(S):
        step(x0, ids, wts, evs[k])
    torch.cuda.synchronize()
    barrier(world)
    st = np.zeros(nev - 1)
    for k in range(S):
        for l in range(a.layers):
            e = evs[k][l]
            st += [e[i].elapsed_time(e[i + 1]) for i in range(nev - 1)]
    st /= S * a.layers  # ms per layer
    st_max = max_over_ranks(st, world)
    if ep_mode:
        # the owner's own stages (metadata + scatter, gate_up, down, combine) from one more step
        oev = [[torch.cuda.Event(enable_timing=True) for _ in range(5)] for _ in range(a.layers)]
        x = x0
        for l, (bank, shared, gate) in enumerate(layers):
            layer_ep.dispatch(x, wts[l], ids[l])
            layer_ep.exchange(layer_ep.recv, layer_ep.send)
            layer_ep.owner(x, bank, shared, stage_events=oev[l])
            layer_ep.exchange(layer_ep.back, layer_ep.partial)
            x = layer_ep.fold(x, gate, residual=x)
        torch.cuda.synchronize()
        ost = np.mean([[oev[l][i].elapsed_time(oev[l][i + 1]) for i in range(4)] for l in range(a.layers)], 0)
        ost_max = max_over_ranks(ost, world)
        gemm_ms = float(ost_max[1] + ost_max[2])
    else:
        gemm_ms = float(st[1] + st[2])

    routes = tokens * TOP
    rows = routes + tokens
    flops = 2.0 * rows * 3 * INTER * HIDDEN  # gate_up + down, routed + shared
    act_bytes = tokens * HIDDEN * 2 + 2 * rows * INTER * 2 + rows * HIDDEN * 2
    if ep_mode:
        # experts of this rank with at least one route from any rank: measured on the device
        wbytes = (e_loc + 1) * EXPERT_BYTES
    else:
        wbytes = (float(np.mean(active)) + 1) * EXPERT_BYTES
    gemm_bytes = wbytes + act_bytes
    tflops = flops / (gemm_ms / 1e3) / 1e12
    gbs = gemm_bytes / (gemm_ms / 1e3) / 1e9
    pk_tc, pk_hbm = peaks['tc_sustained'], peaks['hbm']
    bound = 'tensor' if flops / (pk_tc * 1e12) >= gemm_bytes / (pk_hbm * 1e9) else 'hbm'
    if bound == 'tensor':
        roof = {'bound': 'tensor', 'achieved': round(tflops, 1), 'peak': pk_tc, 'unit': 'TFLOP/s',
                'frac': round(tflops / pk_tc, 4)}
    else:
        roof = {'bound': 'hbm', 'achieved': round(gbs, 1), 'peak': pk_hbm, 'unit': 'GB/s',
                'frac': round(gbs / pk_hbm, 4)}
    roof.update({'traffic': None if ep_mode else NCU_TRAFFIC_PER_LAYER,
                 'traffic_source': ('not captured for the expert-parallel owner' if ep_mode else NCU_TRAFFIC_SOURCE),
                 'kernel': ('grouped GEMMs (gate_up+SwiGLU, down+weight) per layer' +
                            (', on each rank\'s received routes + its own tokens\' shared expert (max over ranks)'
                             if ep_mode else '')),
                 'timing': f'CUDA events between the launches, {S} instrumented steps after the timed region',
                 'peak_source': peaks['src'], 'flops_per_layer': flops, 'alg_bytes_per_layer': round(gemm_bytes),
                 'tensor_frac': round(tflops / pk_tc, 4), 'hbm_frac': round(gbs / pk_hbm, 4),
                 'gemm_us_per_layer': round(gemm_ms * 1e3, 2)})
    if ep_mode:
        names = ('dispatch', 'all_to_all_dispatch', 'owner', 'all_to_all_return', 'fold')
        phases = {n: round(float(v) * 1e3, 2) for n, v in zip(names, st_max)}
        phases.update({f'owner_{n}': round(float(v) * 1e3, 2)
                       for n, v in zip(('meta_scatter', 'gate_up', 'down', 'combine'), ost_max)})
        seg = (layer_ep.cap + 1) * layer_ep.row_bytes
        cross = (world - 1) * seg
        # with the direct transport the rows cross NVLink inside the dispatch (and the owner's
        # combine) kernels: their phase time bounds the transfer rate from below
        xfer_us = phases['all_to_all_dispatch'] if a.ep_transport == 'nccl' else phases['dispatch']
        roof['phase_us_per_layer_max_over_ranks'] = phases
        roof['limiting_phase'] = max(names, key=lambda n: phases[n])
        roof['nvlink'] = {'dispatch_bytes_per_rank': cross, 'return_bytes_per_rank': (world - 1) * layer_ep.cap *
                          HIDDEN * 2, 'dispatch_gbs': round(cross / (xfer_us * 1e-6) / 1e9, 1) if xfer_us > 0 else None,
                          'dispatch_gbs_timing': ('the all_to_all phase' if a.ep_transport == 'nccl' else
                                                  'the whole dispatch phase (metadata, slots, pack + NVLink stores)'),
                          'peer_copy_ref_gbs': 770.0}
    else:
        roof['stage_us_per_layer'] = {'route_meta': round(st[0] * 1e3, 2), 'gate_up': round(st[1] * 1e3, 2),
                                      'down': round(st[2] * 1e3, 2), 'combine': round(st[3] * 1e3, 2)}

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
    e2e = {'value': round(total * e_steps / (ms_e2e / 1e3), 1), 'unit': UNIT,
           'h2d_bytes_per_step': int(xh.numel() * 2 + idh.numel() * 8 + wh.numel() * 4),
           'd2h_bytes_per_step': int(outh.numel() * 2),
           'api': 'ep.GpuLayer.forward per layer' if ep_mode else 'gpu_routes.moe_block per layer'}

    cpu = check = None
    if rank == 0 and world == 1 and not a.no_cpu_baseline:
        cpu, check = cpu_baseline_leg(layers[0], x0, ids[0], wts[0], dev)
    extra = {}
    if not a.no_extra and world == 1:
        extra['c3_decode'] = decode_leg(layers, dev, peaks, max(3, a.steps), a.warmup, a.seed)
        extra['c4_dense'] = dense_leg(dev, peaks)
        extra['c5_ep_1gpu'] = ep_single_gpu_leg(a, layers, dev)

    gpu_launches = (EP_LAUNCHES_PER_LAYER if ep_mode else LAUNCHES_PER_LAYER) * a.layers * a.steps
    line = {
        'metric': METRIC, 'value': round(value, 1), 'unit': UNIT, 'n_gpus': world, 'steps': a.steps,
        'warmup': a.warmup, 'ms_per_step': round(ms_step, 4), 'higher_is_better': True,
        'scaling': scaling(a, world), 'vs_baseline': None, 'dtype': 'bf16',
        'data': 'synthetic (seeded random-init INT8 weights, N(0,1) inputs)',
        'config': config(a, world),
        'workload_stats': {'active_experts_mean_per_layer': round(float(np.mean(active)), 1)},
        'roofline': roof, 'cpu_baseline': cpu, 'e2e': e2e,
        'gpu_launches': gpu_launches,
        'clocks': clk.summary(),
    }
    if check is not None:
        line['check'] = check
    if extra:
        line['extra'] = extra
    if rank == 0:
        print(json.dumps(line), flush=True)
    if layer_ep is not None:
        layer_ep.close()


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
            'hbm_frac': round(gbs / peaks['hbm'], 4), 'launches_per_layer': 1,
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
    """C4: dense linear sweep K=2048, N in {512,2048,4096,8192}, M in {1,16,256,2048}, W8A16
    and W8A8 (the table GEMV at M=1, the int8 tensor-core GEMM above).  Weight copies rotate
    so each iteration reads weights from HBM (the pool of copies exceeds L2)."""
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
        # W8A8 at M > 1: activation quantisation + the int8 tensor-core GEMM (int32 group dots);
        # the tensor peak is taken as twice the measured bf16 one (int8 runs at twice the rate)
        for m in (16, 256, 2048):
            x = torch.randn((m, K), device=dev).bfloat16()
            us = _graph_time(lambda i: W8.linear(x, qs[i % copies], ss[i % copies]), iters, dev)
            flops = 2.0 * m * n * K
            bytes_ = wb + 2 * m * K + 2 * m * n
            tops, gbs = flops / (us * 1e-6) / 1e12, bytes_ / (us * 1e-6) / 1e9
            pk_i8 = 2 * peaks['tc']
            bound = 'tensor' if flops / (pk_i8 * 1e12) > bytes_ / (peaks['hbm'] * 1e9) else 'hbm'
            frac = tops / pk_i8 if bound == 'tensor' else gbs / peaks['hbm']
            out.append({'op': 'w8a8', 'M': m, 'N': n, 'K': K, 'us': round(us, 2), 'tops': round(tops, 2),
                        'gbs': round(gbs, 1), 'bound': bound, 'frac': round(frac, 4),
                        'peak': 'int8 = 2 x measured bf16' if bound == 'tensor' else 'measured HBM'})
        del qs, ss, tabs
    return out


def ep_single_gpu_leg(a, layers, dev, steps=3, warmup=2):
    """C5 at one GPU: the expert-parallel benchmark's whole job (``--total-tokens``
    through the same layers) on this GPU through ``gpu_routes.moe_block`` -- the t1 of
    the scaling efficiency t1 / (N * tN) of the N-GPU expert-parallel runs."""
    from localmoe35ba3b_b200.runtime import gpu_routes
    tokens = a.total_tokens
    x0, ids, wts = make_routing(a.layers, tokens, dev, a.seed + 555)

    def step():
        x = x0
        for l, (bank, shared, gate) in enumerate(layers):
            x = gpu_routes.moe_block(x, wts[l], ids[l], bank, shared=shared, shared_gate_weight=gate, residual=x)
        return x

    for _ in range(warmup):
        step()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record()
    for _ in range(steps):
        step()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    del x0, ids, wts
    return {'tokens': tokens, 'layers': a.layers, 'ms_per_step': round(ms, 3),
            'tok_per_s': round(tokens / (ms / 1e3), 1), 'us_per_layer': round(ms * 1e3 / a.layers, 2),
            'workload': f'{tokens} tokens x {a.layers} layers on 1 GPU (moe_block; all 256 experts), the '
                        'expert-parallel job at N = 1'}


# ------------------------------------------------------------------ CPU legs
def _bf16_np(t):
    return t.float().cpu().numpy()


def cpu_baseline_leg(layer, x, ids, wts, dev, repeats=3):
    """The reference's CPU path (HF experts loop, fp32 dequantise-then-matmul, plus the
    gated shared expert) on layer 0 of this run's own weights and all of its tokens,
    timed on the host cores; its output is also the fp32 check of the GPU block on the
    same inputs (max-abs-normalised error, the north-star's 1e-2 bar)."""
    from localmoe35ba3b_b200.runtime import gpu_routes
    from oracle import cpu_baseline as C
    (qg, sg, qd, sd), shared, gate = layer
    gpu = gpu_routes.moe_block(x, wts, ids, [qg, sg, qd, sd], shared=shared, shared_gate_weight=gate)
    torch.cuda.synchronize()
    case = (x.float().cpu(), ids.cpu(), wts.cpu(), tuple(t.cpu() for t in (qg, sg, qd, sd)),
            [(q.cpu(), s.cpu()) for q, s in shared], gate.float().cpu())
    t, threads = C.time_layer(case, repeats=repeats)
    with torch.no_grad():
        ref = C.moe_block(*case).numpy()
    got = _bf16_np(gpu)
    err = float(np.abs(got - ref).max() / np.abs(ref).max())
    tokens = x.shape[0]
    cpu = {'value': round(tokens / (t * 40), 2), 'unit': UNIT, 'cores': threads, 'kind': 'port',
           'sample': f'all {tokens} tokens through layer 0 (1 of the 40 layers) of this run\'s weights per repeat, '
                     f'median of {repeats} after 1 warm-up, tok/s = tokens / (40 x layer time); torch fp32 '
                     f'dequantise-then-matmul (HF experts loop + shared expert); CPU: {C.cpu_model()}',
           'layer_s': round(t, 4)}
    check = {'what': 'GPU moe_block vs the CPU fp32 dequantise-then-matmul block, layer 0, all tokens',
             'max_abs_norm_err': err, 'tol': 1e-2, 'ok': err < 1e-2}
    return cpu, check


def run_reference(a, rank, world):
    """The reference arm: the reference's CPU path (HF experts loop on fp32-dequantised
    INT8 weights + the shared expert; the oracle port, oracle/cpu_baseline.py) on all the
    host cores.  Each step is one MoE layer over ALL the job's tokens (2048, or the
    expert-parallel job's total): a sample of 1 of the job's layers, every layer being
    the same work; tok/s = tokens / (layers x layer time)."""
    if rank != 0:
        return
    from oracle import cpu_baseline as C
    total, _ = job_tokens(a, world)
    case = C.make_case(tokens=total, seed=a.seed)
    threads = os.cpu_count()
    for _ in range(a.warmup):
        C.time_layer(case, repeats=1, threads=threads, warmup=False)
    times = []
    for _ in range(a.steps):
        t, threads = C.time_layer(case, repeats=1, threads=threads, warmup=False)
        times.append(t)
    t_layer = float(np.mean(times))
    value = total / (a.layers * t_layer)
    print(json.dumps({
        'impl': 'reference', 'metric': METRIC, 'value': round(value, 2), 'unit': UNIT, 'n_gpus': world,
        'steps': a.steps, 'warmup': a.warmup, 'ms_per_step': round(t_layer * 1e3, 2),
        'higher_is_better': True, 'scaling': scaling(a, world), 'vs_baseline': None, 'dtype': 'f32',
        'data': 'synthetic (seeded random-init INT8 weights, N(0,1) inputs)',
        'config': config(a, world),
        'cpu_baseline': {'value': round(value, 2), 'unit': UNIT, 'cores': threads, 'kind': 'port',
                         'sample': f'each step = all {total} tokens through 1 MoE layer (1 of the {a.layers}; '
                                   f'ms_per_step is that layer), tok/s = tokens / ({a.layers} x mean layer time); '
                                   f'HF experts loop, fp32 dequantised weights, torch on {threads} host threads; '
                                   f'CPU: {C.cpu_model()}'},
        'e2e': {'value': round(value, 2), 'unit': UNIT, 'h2d_bytes_per_step': 0, 'd2h_bytes_per_step': 0},
    }), flush=True)


def run_only(a):
    """One extra leg on its own (no prefill timing): the profiling entry point."""
    torch.cuda.set_device(0)
    dev = torch.device('cuda', 0)
    peaks = load_peaks()
    if a.only == 'c4':
        out = dense_leg(dev, peaks)
    else:
        layers = make_layers(a.layers, dev, a.seed)
        out = (decode_leg(layers, dev, peaks, max(3, a.steps), a.warmup, a.seed) if a.only == 'c3'
               else ep_single_gpu_leg(a, layers, dev))
    print(json.dumps({'only': a.only, 'layers': a.layers, a.only: out}), flush=True)


def main():
    a = parse()
    if a.only is not None and a.impl == 'ours':
        run_only(a)
        return
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
