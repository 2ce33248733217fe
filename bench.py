#!/usr/bin/env python
"""Benchmark of the hybrid block at T = 32760 tokens.

One step = the GDN mixer chain followed by the FP8-attention mixer chain of
``kairos_sensenova_b200.hybrid.HybridBlock`` over the whole sequence, Ulysses
sequence-parallel over N GPUs (one process per GPU, NCCL).  Metric: hybrid
block Mtokens/s = T / step time.  Synthetic seeded N(0,1) hidden states
[32760, 3072] bf16, random-init N(0,0.02) weights (no checkpoints exist here).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--dit-steps K2]

After the hybrid block the same run times BASELINE config 4, the full DiT
denoise step (``kairos_sensenova_b200.dit``), and adds it to the JSON line as
``dit_step`` (ms per step, max over ranks; ``--dit-steps 0`` skips it).

For N > 1 launch with torch.distributed.run (127.0.0.1 rendezvous).
``--impl reference`` times the reference path's CPU restatement (the oracle
port of the reference's torch code) on this host's cores, rank 0 only.
"""
from __future__ import annotations

import argparse
import datetime
import gc
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

import torch
import torch.distributed as dist

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

T_FULL, HIDDEN, HEADS, HEAD_DIM = 32760, 3072, 24, 128
METRIC = 'hybrid-block Mtokens/s @T=32760 bf16'


def _peaks():
    p = ROOT / 'MEASURED_PEAKS.json'
    if p.exists():
        d = json.loads(p.read_text())
        return d['bf16_tflops'], d['hbm_gbs'], 'measured'
    return 1590.0, 6650.0, 'fallback'


def _cpu_model():
    try:
        for line in subprocess.run(['lscpu'], capture_output=True, text=True, timeout=10).stdout.splitlines():
            if line.startswith('Model name:'):
                return line.split(':', 1)[1].strip()
    except (OSError, subprocess.SubprocessError):
        pass
    return None


def _cpu_step_seconds(runs, warmup=1):
    """Time the FULL config-3 hybrid step (both chains, all 24 heads, T = 32760,
    every projection) on the host cores with the oracle restatement of the
    reference's torch path (fp32, all threads): ``warmup`` untimed runs, then
    ``runs`` timed ones.  Returns the list of seconds per run."""
    from oracle.hybrid import attn_chain, freqs_cis_3d, gdn_chain
    torch.set_num_threads(os.cpu_count())
    w, x = _cpu_inputs()
    fr = freqs_cis_3d(HEAD_DIM, 21, 30, 52)
    times = []
    with torch.no_grad():
        for i in range(warmup + runs):
            t0 = time.perf_counter()
            y = gdn_chain(w, x, HEADS, HEAD_DIM)
            attn_chain(w, y, HEADS, HEAD_DIM, freqs=fr)
            if i >= warmup:
                times.append(time.perf_counter() - t0)
    return times


def _cpu_inputs():
    g = torch.Generator().manual_seed(0)
    w = {n: torch.randn(HEADS * HEAD_DIM, HIDDEN, generator=g) * 0.02 for n in ('Wq', 'Wk', 'Wv', 'Wg', 'Aq', 'Ak', 'Av')}
    w['Wo'] = torch.randn(HIDDEN, HEADS * HEAD_DIM, generator=g) * 0.02
    w['Ao'] = torch.randn(HIDDEN, HEADS * HEAD_DIM, generator=g) * 0.02
    w['Wa'] = torch.randn(HEADS, HIDDEN, generator=g) * 0.02
    w['Wb'] = torch.randn(HEADS, HIDDEN, generator=g) * 0.02
    for n in ('cq', 'ck', 'cv'):
        w[n] = torch.rand(HEADS * HEAD_DIM, 4, generator=g) - 0.5
    w['A_log'] = torch.log(torch.rand(HEADS, generator=g) * 16)
    w['dt_bias'] = torch.randn(HEADS, generator=g) * 0.1 - 3
    w['o_norm_w'] = torch.ones(HEAD_DIM)
    x = torch.randn(T_FULL, HIDDEN, generator=g).bfloat16().float()
    return w, x


class ClockSampler:
    """nvidia-smi clock / throttle sampling during the timed region."""

    def __init__(self, gpu_index):
        self.proc = None
        self.path = Path('/tmp') / f'kb200_clocks_{os.getpid()}.csv'
        try:
            self.proc = subprocess.Popen(
                ['nvidia-smi', f'--id={gpu_index}',
                 '--query-gpu=clocks.sm,clocks.max.sm,clocks_event_reasons.active,'
                 'clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,'
                 'clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap',
                 '--format=csv,noheader,nounits', '-lms', '200'],
                stdout=open(self.path, 'w'), stderr=subprocess.DEVNULL)
        except (FileNotFoundError, OSError):
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = [r.split(',') for r in self.path.read_text().strip().splitlines() if r.strip()]
        sm, mx, reasons = [], 0.0, set()
        names = ['hw_slowdown', 'hw_thermal_slowdown', 'sw_thermal_slowdown', 'sw_power_cap']
        for r in rows:
            try:
                sm.append(float(r[0]))
                mx = max(mx, float(r[1]))
                for n, v in zip(names, r[3:7]):
                    if v.strip().lower() == 'active':
                        reasons.add(n)
            except (ValueError, IndexError):
                continue
        return {'sm_mhz': statistics.median(sm) if sm else None, 'sm_max_mhz': mx or None,
                'reasons': sorted(reasons), 'samples': len(sm)}


def _config(world):
    return {'workload': 'config3 hybrid block: GDN chain + FP8-attention chain, T=32760, '
                        'hidden 3072, 24x128 heads, Ulysses over ranks',
            'global_batch': 1, 'seq_len': T_FULL, 'parallelism': f'ulysses{world}'}


def run_reference(args, rank):
    """The reference arm: the reference's CPU torch path for the whole config-3
    step (the oracle port: the reference's path is Python/Triton and cannot run
    on the GPU box), rank 0 only.  Each timed run is one FULL step -- nothing is
    sampled or extrapolated; one untimed warm-up, then min(steps, 3) timed runs
    (a full step takes tens of seconds on the host), reported as their median."""
    if rank != 0:
        return
    runs = max(1, min(args.steps, 3))
    times = _cpu_step_seconds(runs, warmup=1)
    step_s = statistics.median(times)
    v = T_FULL / step_s / 1e6
    cores = torch.get_num_threads()
    cpu = {'value': v, 'unit': 'Mtokens/s', 'cores': cores, 'kind': 'port', 'cpu_model': _cpu_model(),
           'sample': f'the full config-3 step (all 24 heads, T=32760), fp32 oracle port of the reference torch '
                     f'path; 1 warm-up + median of {runs} timed full steps; not extrapolated'}
    line = {
        'impl': 'reference', 'metric': METRIC, 'value': v, 'unit': 'Mtokens/s',
        'n_gpus': args.gpus, 'steps': runs, 'steps_requested': args.steps, 'warmup': 1,
        'warmup_requested': args.warmup, 'ms_per_step': step_s * 1e3, 'run_ms': [t * 1e3 for t in times],
        'higher_is_better': True, 'scaling': 'strong', 'vs_baseline': None, 'dtype': 'f32', 'data': 'synthetic',
        'extrapolated': False, 'config': _config(args.gpus), 'cpu_baseline': cpu,
        'e2e': {'value': v, 'unit': 'Mtokens/s', 'h2d_bytes_per_step': 0, 'd2h_bytes_per_step': 0},
    }
    print(json.dumps(line), flush=True)


def _bind_host_cpus(local_rank):
    """Pin this rank's host threads to the CPUs NVML lists as close to its GPU,
    so the pinned staging buffers of the e2e loop are first touched on that
    GPU's NUMA node.  Returns the CPU count bound to, or None (NVML missing)."""
    try:
        import pynvml
        pynvml.nvmlInit()
        pr = torch.cuda.get_device_properties(local_rank)
        bus = f'{pr.pci_domain_id:08x}:{pr.pci_bus_id:02x}:{pr.pci_device_id:02x}.0'
        h = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
        words = pynvml.nvmlDeviceGetCpuAffinity(h, (os.cpu_count() + 63) // 64)
        cpus = {64 * i + b for i, wd in enumerate(words) for b in range(64) if (wd >> b) & 1}
        cpus &= set(range(os.cpu_count()))
        if cpus:
            os.sched_setaffinity(0, cpus)
            return len(cpus)
    except Exception:
        return None
    return None


GDN_BYTES = 811.0e6          # config 1 compulsory HBM bytes: q,k,v,o bf16, g fp32, beta bf16, final state fp32
GDN_FLOPS = 1.438e11         # config 1 algorithmic flops (182,955 per token-head x 786,240 token-heads)


def time_gdn_op(flush, steps):
    """the GDN chunk forward alone, B1 T32760 H24 d128, bf16
    q/k/v/beta, fp32 g, fp32 final state, inputs resident in HBM (q, k already
    L2-normalised as the config says).  CUDA events on the launch stream per
    call, L2 flushed before each; returns the mean ms."""
    from kairos_sensenova_b200 import chunk_gated_delta_rule
    gen = torch.Generator(device='cuda')
    gen.manual_seed(0)
    B, T, H, K = 1, T_FULL, HEADS, HEAD_DIM
    nrm = torch.nn.functional.normalize
    q = nrm(torch.randn(B, T, H, K, generator=gen, device='cuda'), dim=-1).bfloat16()
    k = nrm(torch.randn(B, T, H, K, generator=gen, device='cuda'), dim=-1).bfloat16()
    v = torch.randn(B, T, H, K, generator=gen, device='cuda').bfloat16()
    beta = torch.randn(B, T, H, generator=gen, device='cuda').sigmoid().bfloat16()
    g = -torch.nn.functional.softplus(torch.randn(B, T, H, generator=gen, device='cuda'))
    run = lambda: chunk_gated_delta_rule(q, k, v, g, beta, output_final_state=True)  # noqa: E731
    for _ in range(3):
        run()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    for e0, e1 in ev:
        flush.zero_()
        e0.record()
        run()
        e1.record()
    torch.cuda.synchronize()
    return statistics.mean(e0.elapsed_time(e1) for e0, e1 in ev), chunk_gated_delta_rule.launches


def time_sdpa_bf16(flush, steps):
    """torch's bf16 SDPA (the library flash kernel) on config 2's shape
    (B1 H24 S32760 d128, non-causal): the attention kernel's library baseline,
    timed like it (CUDA events, L2 flushed)."""
    gen = torch.Generator(device='cuda')
    gen.manual_seed(1)
    q, k, v = (torch.randn(1, HEADS, T_FULL, HEAD_DIM, generator=gen, device='cuda').bfloat16() for _ in range(3))
    F = torch.nn.functional
    for _ in range(2):
        F.scaled_dot_product_attention(q, k, v)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    for e0, e1 in ev:
        flush.zero_()
        e0.record()
        F.scaled_dot_product_attention(q, k, v)
        e1.record()
    torch.cuda.synchronize()
    return statistics.mean(e0.elapsed_time(e1) for e0, e1 in ev)


def time_dit(args, world, rank, sync_all, flush):
    """one full DiT denoise step (30 blocks, hidden 3072, 24x128
    heads, FFN 8192, GDN in 3 of every 4 blocks, FP8 attention in every 4th,
    cross-attention to 512 text tokens of dim 4096; latent 16x21x60x104 -> 32760
    tokens), sequence-parallel over the ranks.  Random-init weights (seed 2),
    N(0,1) latent and text, t = 500.  Device time with CUDA events per step,
    L2 flushed between steps; the caller takes the max over ranks."""
    from kairos_sensenova_b200.dit import DiTConfig, KairosDiT
    cfg = DiTConfig()
    model = KairosDiT(cfg, world=world, rank=rank)
    gen = torch.Generator(device='cuda')
    gen.manual_seed(2)
    latent = torch.randn(cfg.in_dim, *cfg.latent, generator=gen, device='cuda')
    ctx = torch.randn(cfg.text_len, cfg.text_dim, generator=gen, device='cuda')
    ts = torch.tensor([500.0], device='cuda')
    warm = max(3, args.warmup)
    step = model
    if not args.eager_dit:
        from kairos_sensenova_b200.graphs import GraphedStep
        step = GraphedStep(model, latent, ts, ctx)
    with torch.no_grad():
        for _ in range(warm):
            step(latent, ts, ctx)
        sync_all()
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
              for _ in range(args.dit_steps)]
        for s0, s1 in ev:
            flush.zero_()
            s0.record()
            out = step(latent, ts, ctx)
            s1.record()
        sync_all()
    ms = statistics.mean(s0.elapsed_time(s1) for s0, s1 in ev)
    ok = bool(torch.isfinite(out.float()).all())
    n = model.launches_per_step()
    del model, step, out
    gc.collect()
    sync_all()
    torch.cuda.empty_cache()
    return {'metric': 'DiT denoise-step ms', 'ms_per_step': ms, 'higher_is_better': False,
            'steps': args.dit_steps, 'warmup': warm, 'n_gpus': world, 'finite_output': ok,
            'gpu_launches': n * args.dit_steps,
            'config': {'workload': 'config4 DiT step: 30 blocks, hidden 3072, 24x128 heads, FFN 8192 tanh-GELU, '
                                   'GDN in 3 of 4 blocks + FP8 attention every 4th, cross-attn 512x4096, '
                                   'latent 16x21x60x104 (32760 tokens), t=500',
                       'parallelism': f'sequence/ulysses{world}', 'data': 'synthetic, random-init weights',
                       'launch': 'eager' if args.eager_dit else 'one CUDA graph per step',
                       'l2': 'flushed (256 MB write) between timed steps'}}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument('--gpus', type=int, default=1)
    ap.add_argument('--steps', type=int, default=10)
    ap.add_argument('--warmup', type=int, default=3)
    ap.add_argument('--impl', default='ours', choices=['ours', 'reference'])
    ap.add_argument('--no-cpu-baseline', action='store_true')
    ap.add_argument('--eager', action='store_true',
                    help='issue the hybrid step op by op instead of replaying it as one captured CUDA graph (always so with more than one GPU)')
    ap.add_argument('--eager-dit', action='store_true',
                    help='time the DiT step issued op by op instead of as one captured CUDA graph')
    ap.add_argument('--nccl-timeout', type=int, default=300,
                    help='seconds before a collective that a peer never joins fails (NCCL process group timeout)')
    ap.add_argument('--dit-steps', type=int, default=3,
                    help='timed DiT denoise steps (BASELINE config 4) after the hybrid block; 0 skips')
    args = ap.parse_args()
    world = int(os.environ.get('WORLD_SIZE', '1'))
    rank = int(os.environ.get('RANK', '0'))
    local = int(os.environ.get('LOCAL_RANK', '0'))
    if args.impl == 'reference':
        run_reference(args, rank)
        return
    torch.cuda.set_device(local)
    host_cpus = _bind_host_cpus(local)
    if world > 1:
        # a bounded communicator timeout: a rank that never joins a collective ends the
        # others' wait with an error instead of a hang
        dist.init_process_group('nccl', device_id=torch.device('cuda', local),
                                timeout=datetime.timedelta(seconds=args.nccl_timeout))
    from kairos_sensenova_b200.hybrid import HybridBlock
    assert T_FULL % world == 0 and HEADS % world == 0
    Tl = T_FULL // world
    blk = HybridBlock(HIDDEN, HEADS, HEAD_DIM, world=world, rank=rank, group=None)
    gen = torch.Generator(device='cuda')
    gen.manual_seed(2)
    x_full = torch.randn(T_FULL, HIDDEN, generator=gen, device='cuda').to(torch.bfloat16)
    x = x_full[rank * Tl:(rank + 1) * Tl].contiguous()
    del x_full
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device='cuda')   # > 126 MB L2

    def sync_all():
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    with torch.no_grad():
        for _ in range(args.warmup):
            blk.forward(x)
        sync_all()
        # the attention kernel's own duration (roofline), CUDA events on its launch
        # stream around the kernel, eager steps with the L2 flushed before each
        aev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
               for _ in range(args.steps)]
        for a0, a1 in aev:
            flush.zero_()
            blk.forward(x, events=(a0, a1))
        sync_all()
        attn_ms = statistics.mean(a0.elapsed_time(a1) for a0, a1 in aev)
        launches = blk.launches_per_step()
        # per-phase device time (eager steps, CUDA events at the phase boundaries on the
        # compute stream): where a multi-GPU step spends its time
        phase_runs = []
        for _ in range(min(args.steps, 5)):
            flush.zero_()
            marks = []
            blk.forward(x, phases=marks)
            phase_runs.append(marks)
        sync_all()
        phase_ms = {}
        for marks in phase_runs:
            for (_, e0), (name, e1) in zip(marks[:-1], marks[1:]):
                if name.endswith('.start'):
                    continue
                phase_ms[name] = phase_ms.get(name, 0.0) + e0.elapsed_time(e1) / len(phase_runs)
        # the step: one CUDA graph per input buffer (two, ping-ponged by the e2e loop),
        # at every GPU count.  A graph that captured NCCL sends/receives holds on to the
        # communicator's resources: the graphs are destroyed (and the device idle) on
        # every rank before the process group is torn down.
        xd = [x.clone(), x.clone()]
        eager = args.eager
        if eager:
            steps = [lambda b=b: blk.forward(xd[b]) for b in range(2)]
        else:
            from kairos_sensenova_b200.graphs import GraphedStep
            steps = [GraphedStep(blk.forward, xd[b], static_inputs=True) for b in range(2)]
        for _ in range(args.warmup):
            steps[0]()
        sync_all()
        sampler = ClockSampler(local) if rank == 0 else None
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
              for _ in range(args.steps)]
        sync_all()
        for s0, s1 in ev:
            flush.zero_()                       # L2 flush between timed steps (outside the events)
            s0.record()
            steps[0]()
            s1.record()
        sync_all()
        step_ms = statistics.mean(s0.elapsed_time(s1) for s0, s1 in ev)
        # end to end through the public API with host buffers: every step copies its
        # input from pinned host memory and its result back; the two directions run on
        # their own streams (separate copy engines, full duplex), double-buffered, so
        # step i's transfers overlap step i+-1's compute
        xh = [x.cpu().pin_memory() for _ in range(2)]
        yh = [torch.empty(Tl, HIDDEN, dtype=torch.bfloat16).pin_memory() for _ in range(2)]
        comp = torch.cuda.current_stream()
        copy = torch.cuda.Stream()          # host -> device
        back = torch.cuda.Stream()          # device -> host
        ev_in = [torch.cuda.Event() for _ in range(2)]
        ev_out = [torch.cuda.Event() for _ in range(2)]
        ev_free = [torch.cuda.Event() for _ in range(2)]
        ev_read = [torch.cuda.Event() for _ in range(2)]
        sync_all()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(comp)
        copy.wait_event(e0)
        back.wait_event(e0)
        with torch.cuda.stream(copy):
            xd[0].copy_(xh[0], non_blocking=True)
            ev_in[0].record(copy)
        for i in range(args.steps):
            b_ = i % 2
            if i + 1 < args.steps:          # prefetch the next step's input
                with torch.cuda.stream(copy):
                    if i >= 1:
                        copy.wait_event(ev_free[(i + 1) % 2])
                    xd[(i + 1) % 2].copy_(xh[(i + 1) % 2], non_blocking=True)
                    ev_in[(i + 1) % 2].record(copy)
            comp.wait_event(ev_in[b_])
            if i >= 2:                      # step i-2's result has left this buffer's output
                comp.wait_event(ev_read[b_])
            y = steps[b_]()
            ev_free[b_].record(comp)
            ev_out[b_].record(comp)
            with torch.cuda.stream(back):
                back.wait_event(ev_out[b_])
                yh[b_].copy_(y, non_blocking=True)
                ev_read[b_].record(back)
            if eager:
                y.record_stream(back)
        comp.wait_stream(copy)
        comp.wait_stream(back)
        e1.record(comp)
        sync_all()
        e2e_ms = e0.elapsed_time(e1) / args.steps
        clocks = sampler.stop() if sampler else None
        del steps, y
        gc.collect()
        sync_all()

    del blk
    gdn_ms = sdpa_ms = gdn_launches = None
    if rank == 0:
        torch.cuda.empty_cache()
        gdn_ms, gdn_launches = time_gdn_op(flush, args.steps)
        sdpa_ms = time_sdpa_bf16(flush, args.steps)
        torch.cuda.empty_cache()
    sync_all()
    dit = time_dit(args, world, rank, sync_all, flush) if args.dit_steps > 0 else None
    names = sorted(phase_ms)
    t = torch.tensor([step_ms, attn_ms, e2e_ms, dit['ms_per_step'] if dit else 0.0] + [phase_ms[n] for n in names],
                     device='cuda')
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    vals = t.tolist()
    step_ms, attn_ms, e2e_ms, dit_ms = vals[:4]
    phase_ms = dict(zip(names, vals[4:]))
    if rank == 0:
        bf16_tf, hbm, kind = _peaks()
        # QK^T (half the FLOPs) runs at the e4m3 rate, 2x bf16; P.V at the bf16 rate
        # (bf16 P and V): the peak is the harmonic blend of the two halves
        fp8_peak = 1.0 / (0.5 / (2 * bf16_tf) + 0.5 / bf16_tf)
        flops = 4.0 * T_FULL * T_FULL * HEAD_DIM * (HEADS // world)
        units = T_FULL * (HEADS // world)
        traffic = 33.86e6 * units / (8192 * 8) + 2.0 * units * HEAD_DIM
        achieved = flops / (attn_ms * 1e-3) / 1e12
        gdn_gbs = GDN_BYTES / (gdn_ms * 1e-3) / 1e9
        gdn_tf = GDN_FLOPS / (gdn_ms * 1e-3) / 1e12
        line = {
            'metric': METRIC, 'value': T_FULL / (step_ms * 1e-3) / 1e6, 'unit': 'Mtokens/s',
            'n_gpus': world, 'steps': args.steps, 'warmup': args.warmup, 'ms_per_step': step_ms,
            'higher_is_better': True, 'scaling': 'strong', 'vs_baseline': None, 'dtype': 'bf16/e4m3',
            'data': 'synthetic',
            'config': {**_config(world),
                       'l2': 'flushed (256 MB write) between timed steps',
                       'launch': 'eager' if eager else 'one CUDA graph per step',
                       'host_cpus_near_gpu': host_cpus},
            'e2e': {'value': T_FULL / (e2e_ms * 1e-3) / 1e6, 'unit': 'Mtokens/s',
                    'h2d_bytes_per_step': Tl * HIDDEN * 2, 'd2h_bytes_per_step': Tl * HIDDEN * 2},
            'gpu_launches': launches * args.steps,
            'roofline': {'kernel': 'attention (e4m3 QK, bf16 PV)',
                         'bound': 'tensor', 'achieved': achieved,
                         'peak': fp8_peak, 'unit': 'TFLOP/s', 'frac': achieved / fp8_peak,
                         'traffic': traffic, 'attn_ms': attn_ms, 'sdpa_bf16_ms': sdpa_ms,
                         'traffic_source': 'ESTIMATE: ncu dram read bytes of a B1 S8192 H8 capture (33.86 MB) '
                                           'scaled linearly by tokens x heads, plus the bf16 output bytes',
                         'sdpa_source': 'torch bf16 scaled_dot_product_attention, config-2 shape, same run',
                         'peak_source': f'{kind} bf16 dense ({bf16_tf} TFLOP/s) x 4/3: QK at 2x (e4m3), PV at 1x (bf16)'},
            'roofline_gdn': {'kernel': 'GDN chunk forward (config 1: B1 T32760 H24 d128)', 'bound': 'hbm',
                             'gdn_ms': gdn_ms, 'launches': gdn_launches,
                             'achieved': gdn_gbs, 'peak': hbm, 'unit': 'GB/s', 'frac': gdn_gbs / hbm,
                             'algorithmic_bytes': GDN_BYTES, 'tflops': gdn_tf,
                             'tensor_frac': gdn_tf / bf16_tf,
                             'peak_source': f'{kind} HBM copy bandwidth; tensor_frac against {kind} bf16 dense'},
            'clocks': clocks,
            'phases_ms': {'values': phase_ms, 'how': 'eager steps, CUDA events at phase boundaries on the '
                                                      'compute stream, mean over steps, max over ranks'},
        }
        if dit:
            dit['ms_per_step'] = dit_ms
            line['dit_step'] = dit
        if world == 1 and not args.no_cpu_baseline:
            ts = _cpu_step_seconds(1, warmup=0)
            line['cpu_baseline'] = {'value': T_FULL / ts[0] / 1e6, 'unit': 'Mtokens/s',
                                    'cores': torch.get_num_threads(), 'kind': 'port', 'cpu_model': _cpu_model(),
                                    'ms_per_step': ts[0] * 1e3,
                                    'sample': 'one full config-3 step (all 24 heads, T=32760), fp32 oracle port '
                                              'of the reference torch path, no warm-up; not extrapolated'}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


if __name__ == '__main__':
    main()
