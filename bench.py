"""Committed voxels/s of StreamVoxel's column-generation step on B200 (BASELINE.json `metric`, config 2 workload).

One step = one slot-batched bf16 forward of DiT-B/4 + 12-layer ControlNet over 8 slots with cached packed K/V,
followed by the EASE step of every slot (entropy, 4^3 block-quota selection, low-entropy-last deferral, counter-based
categorical draw, token commit), all in one CUDA graph. Windows run their whole schedule (1 marking + up to 32 solid
forwards, cap 32, quartercos) and are re-armed when they finish; committed voxels count every voxel a window commits,
the deferred ones at its finish (`streamvoxel/stream/slot.py:166-176`).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

N > 1: one process per GPU (torchrun), each with its own 8 slots and no collective on the data path (windows shard
by dependency-safe admission); rank 0 prints the whole-job line with the time = max over ranks. `--impl reference`
times the reference algorithm's CPU path (the oracle port: fp32 torch forward + numpy EASE step) on the host cores.
"""
from __future__ import annotations

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

METRIC = 'committed voxels/s per B200 (8 slots)'
UNIT = 'voxels/s'
L1_CAP, L2_CAP, CAP = 8, 81, 32
WORKLOADS = {
    'config2': (8, 'dit_b4_control',
                'config2: DiT-B/4 (d=768, 8x96 heads, 12 layers, V=256) + 12-layer ControlNet, 8 slots, bf16, cached K/V'),
    'config4': (8, 'dit_b4_control',
                'config4: streaming expansion 32^2 -> 64^2 columns (3072 windows), DiT-B/4 + 12-layer ControlNet, '
                '8 slots per GPU, cap 32, Chebyshev >= 2 admission, whole step in one CUDA graph'),
    'config5': (16, 'dit_l4_control',
                'config5: DiT-L/4-class (d=1152, 12x96 heads, 24 layers, MLP 4608, V=256) + 24-layer ControlNet, '
                '16 slots, bf16, cached K/V'),
}
SLOTS, MODEL, WORKLOAD = WORKLOADS['config2']


def model_config():
    from streamvoxel_b200 import model as sm
    return getattr(sm, MODEL)()
BYTE_KERNELS = ('ease_scores', 'patch_embed')   # memory-bound: rates in GB/s, left out of the step's FLOPs


def parse():
    p = argparse.ArgumentParser()
    p.add_argument('--gpus', type=int, default=1)
    p.add_argument('--steps', type=int, default=66)
    p.add_argument('--warmup', type=int, default=5)
    p.add_argument('--impl', default='ours', choices=['ours', 'reference'])
    p.add_argument('--cpu-sample', type=int, default=1, help='slot-forwards in the CPU baseline sample')
    p.add_argument('--workload', default='config2', choices=sorted(WORKLOADS),
                   help='config2 (default, the metric\'s configuration), config4 (the streaming expansion) or '
                        'config5 (the larger model, 16 slots)')
    p.add_argument('--side0', type=int, default=32, help='config4: side of the committed start square (columns)')
    p.add_argument('--side1', type=int, default=64, help='config4: side of the target region (columns)')
    args = p.parse_args()
    global SLOTS, MODEL, WORKLOAD
    SLOTS, MODEL, WORKLOAD = WORKLOADS[args.workload]
    return args


def dist_env():
    rank = int(os.environ.get('RANK', 0))
    world = int(os.environ.get('WORLD_SIZE', 1))
    local = int(os.environ.get('LOCAL_RANK', 0))
    return rank, world, local


# ------------------------------------------------------------------------------------------------- clocks

class Clocks:
    """SM clocks and throttle reasons sampled during the timed region: NVML in a thread every 20 ms (read-only
    queries, the device found by its UUID), else `nvidia-smi -lms 200`. One sample is also taken on entry and exit,
    so a short timed region still has a record."""
    QUERY = ('index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,'
             'clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,'
             'clocks_event_reasons.sw_power_cap')
    # NVML clocks-event reason bits (nvml.h): the ones that reject or annotate a measurement.
    REASONS = {0x8: 'hw_slowdown', 0x40: 'hw_thermal_slowdown', 0x20: 'sw_thermal_slowdown', 0x4: 'sw_power_cap'}

    def __init__(self, index):
        self.index, self.rows, self.proc, self.nvml, self.stop = index, [], None, None, threading.Event()

    def _nvml_handle(self):
        try:
            import pynvml
            pynvml.nvmlInit()
            uuid = str(torch.cuda.get_device_properties(self.index).uuid)
            return pynvml, pynvml.nvmlDeviceGetHandleByUUID(uuid if uuid.startswith('GPU-') else 'GPU-' + uuid)
        except Exception:
            return None

    def _sample(self):
        nv, h = self.nvml
        sm = nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)
        mx = nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)
        bits = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
        self.rows.append(dict(sm=float(sm), max=float(mx), reasons={n for b, n in self.REASONS.items() if bits & b}))

    def _poll(self):
        while not self.stop.wait(0.02):
            try:
                self._sample()
            except Exception:
                return

    def __enter__(self):
        self.nvml = self._nvml_handle()
        if self.nvml is not None:
            try:
                self._sample()
                self.thread = threading.Thread(target=self._poll, daemon=True)
                self.thread.start()
                return self
            except Exception:
                self.nvml = None
        try:
            self.proc = subprocess.Popen(['nvidia-smi', f'--id={self.index}', f'--query-gpu={self.QUERY}',
                                          '--format=csv,noheader,nounits', '-lms', '200'],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        names = ['hw_slowdown', 'hw_thermal_slowdown', 'sw_thermal_slowdown', 'sw_power_cap']
        for line in self.proc.stdout:
            r = [v.strip() for v in line.split(',')]
            if len(r) >= 9 and r[1].replace('.', '').isdigit():
                self.rows.append(dict(sm=float(r[1]), max=float(r[2]) if r[2].replace('.', '').isdigit() else None,
                                      reasons={n for n, v in zip(names, r[5:9]) if v.lower() == 'active'}))

    def __exit__(self, *exc):
        if self.nvml is not None:
            self.stop.set()
            self.thread.join(timeout=5)
            try:
                self._sample()
            except Exception:
                pass
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        if not self.rows:
            return dict(sm_mhz=None, sm_max_mhz=None, reasons=['no clock samples (NVML and nvidia-smi unavailable)'],
                        samples=0)
        sm = [r['sm'] for r in self.rows]
        mx = [r['max'] for r in self.rows if r['max']]
        return dict(sm_mhz=float(np.median(sm)), sm_max_mhz=max(mx) if mx else None,
                    reasons=sorted(set().union(*(r['reasons'] for r in self.rows))), samples=len(self.rows),
                    source='nvml' if self.nvml is not None else 'nvidia-smi')


# ------------------------------------------------------------------------------------------------ ours

def bench_items(cfg, seed=0):
    """The slots' synthetic windows (`synth.item`: k ~ U{0..8} L1 tiles, 80 L2 columns, the biome window) and their
    packed key lengths (prefix L2 tokens + L1 tokens + biome tokens), the one length rule of both arms."""
    from streamvoxel_b200 import synth
    from streamvoxel_b200.stream.condition import ModelSpec
    spec = ModelSpec.of(cfg)
    l1, l2, biome = cfg.condition_widths()
    rng = np.random.default_rng(seed)
    items = [synth.item(int(rng.integers(1 << 30)), spec) for _ in range(SLOTS)]
    lengths = [len(it.l2_blocks) * l2 + len(it.l1_blocks) * l1 + biome for it in items]
    return spec, items, lengths


def bench_config(lengths, world):
    """The workload description both arms print (the same dict, so the two lines name the same configuration)."""
    return dict(workload=WORKLOAD, slots_per_gpu=SLOTS, cap=CAP, l1_cap=L1_CAP, l2_cap=L2_CAP,
                packed_keys=[int(v) for v in lengths], mean_packed_keys=float(np.mean(lengths)),
                committed_accounting=('each forward of a window credited with an equal share of the window\'s '
                                      '65536 voxels (exact for whole windows; steady-state rate otherwise)'),
                l2_policy='inputs larger than L2 (the step reads all weights and writes all logits: >= 1 GB)',
                parallelism=f'dp{world}: one engine per GPU, no collective on the data path')


def build(device, seed=0):
    from streamvoxel_b200 import model as sm
    from streamvoxel_b200.stream.batch import SlotBatch
    from streamvoxel_b200.stream.fast_ops import FastSlotForward
    cfg = model_config()
    sd = sm.synthetic_state_dict(cfg, seed=seed)
    spec, items, lengths = bench_items(cfg, seed)
    forward = FastSlotForward((cfg, sd), spec, device, SLOTS, L1_CAP, L2_CAP)
    for i, item in enumerate(items):
        forward.load_slot(i, item)
    forward.wait_loads()
    assert forward.packed.lengths.tolist() == lengths
    batch = SlotBatch(forward)
    return cfg, sd, forward, batch, lengths


def run_device_steps(batch, steps, seeds):
    """Exactly `steps` forwards, device-resident inside each window (see `SlotBatch.run_cycles`). Returns
    (committed voxels, kernel launches, marking forwards). Each forward of a window is credited with an equal share of
    the window's voxels (its column commits them all: solid steps plus the deferred low-entropy-last voxels at finish):
    exact for whole windows, and the steady-state rate when the timed region ends inside a window."""
    committed = launches = markings = 0
    per_step = batch.launches()
    done = 0
    it = iter(seeds)
    while done < steps:
        for i in range(batch.slots):
            batch.arm(i, next(it), CAP)
        batch.params.zero_()
        batch.graph.replay()
        batch._mark(range(batch.slots))
        counts = batch.last_count.tolist()
        batch._after_mark(range(batch.slots), counts)
        launches += per_step + 2   # one marking launch (all slots) and its column-run launch
        markings += 1
        done += 1
        staged = []
        while done + len(staged) < steps and any(st['solid_calls'] < len(st['quotas']) for st in batch.state):
            rows = batch._rows()
            staged.append(batch._pack(rows))
            for st in batch.state:
                if st['solid_calls'] < len(st['quotas']):
                    st['solid_calls'] += 1
                    st['nfe'] += 1
        if staged:
            table = torch.stack(staged).to(batch.device)
            for s in range(len(staged)):
                batch.params.copy_(table[s])
                batch.graph.replay()
            launches += len(staged) * per_step
            done += len(staged)
        for st in batch.state:   # the forwards each window ran in this cycle (marking + solid steps)
            committed += batch.total * (1 + st['solid_calls']) / (1 + len(st['quotas']))
        if all(st['solid_calls'] >= len(st['quotas']) for st in batch.state):
            for i in range(batch.slots):
                batch._finish(i)
    return committed, launches, markings


def run_api_steps(batch, steps, seeds):
    """Exactly `steps` forwards through the SlotBatch API as a caller that overlaps its host work with the device
    drives it: up to `SlotBatch.depth` steps in flight (`launch` queues a step with the H2D copy of its scalars from
    pinned memory and the D2H copies of its commits; `collect` waits for the oldest and books them), finished windows
    re-armed after their step is collected. The same per-forward share of each window's voxels as
    `run_device_steps`."""
    committed = h2d = d2h = 0
    it = iter(seeds)
    for i in range(batch.slots):
        if batch.state[i]['phase'] == 'idle':
            batch.arm(i, next(it), CAP)
    launched = collected = 0
    while collected < steps:
        while launched < steps and batch.in_flight < batch.depth and batch.runnable():
            batch.launch()
            rows = batch._queue[-1]['rows']
            kmax = max([r[0] for r in rows] + [0])
            h2d += batch.params_host.numel()
            d2h += (2 * batch.slots) * 4 + (batch.slots * kmax * (4 + 2) if kmax else 0)
            launched += 1
        if not batch.in_flight:
            raise RuntimeError('no slot can take a forward')   # every finished window is re-armed, so it cannot happen
        results = batch.collect()
        collected += 1
        for i, (record, commit) in results.items():
            if record is not None:
                committed += batch.total   # a finished window committed its whole column
                batch.arm(i, next(it), CAP)
    for st in batch.state:   # windows still running: their share for the forwards they had
        if st['phase'] == 'solid' and st['quotas']:
            committed += batch.total * st['nfe'] / (1 + len(st['quotas']))
    return committed, h2d, d2h


# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) per launch from one ncu capture of the kernel on the
# profile_case input (`python -m streamvoxel_b200.profile_case <case>`), with that case's algorithmic bytes: the
# roofline's `traffic` scales the measurement to the timed launch by its algorithmic bytes (traffic grows with the
# valid keys / rows processed).
MEASURED_TRAFFIC = {
    # cross (8 slots x 8 heads, keys 1344 + 1024 i: K/V 121.1 MB + Q 12.6 MB + O 12.6 MB) + self (Q/K/V 37.7 MB +
    # O 12.6 MB) in one launch
    'attention_joint': (222.1e6, 196.6e6),
    # A 12.6 MB + W 4.7 MB + out 50.3 MB (the output mostly stays in L2 at kernel end)
    'gemm_fc1_gelu': (20.5e6, 67.6e6),
}


def algorithmic_bytes(name, cfg, lengths):
    """Bytes a launch must move at least once (inputs read + outputs written), for the traffic scaling."""
    rows = SLOTS * cfg.patches
    if name == 'attention_joint':   # cross K/V + Q + O, self Q/K/V + O
        return float(np.sum(lengths)) * cfg.heads * 96 * 2 * 2 + 2 * rows * cfg.d * 2 + 4 * rows * cfg.d * 2
    if name == 'gemm_fc1_gelu':
        return (rows * cfg.d + cfg.mlp * cfg.d + rows * cfg.mlp) * 2.0
    return None


def time_kernels(cfg, forward, batch, lengths):
    """Average launch duration of each kernel class of the step at the step's shapes (CUDA events around a replayed
    CUDA graph of 20 launches)."""
    from streamvoxel_b200 import ops, _lib
    dev = forward.device
    rows, d, heads = SLOTS * cfg.patches, cfg.d, cfg.heads
    ws = forward.engine.ws
    m = forward.model
    bw, cw = m.backbone[0], m.cross[0]
    k0, v0 = forward.engine.kv[0]
    stats = forward.engine.stats['b']
    tables = m.rope_sin, m.rope_cos
    ones = torch.ones(d, device=dev, dtype=torch.bfloat16)

    def clock(fn, reps=20):
        """Device time per launch: `reps` launches captured in one CUDA graph and replayed (as the step runs them), so
        that host-side launch cost (ctypes, tensor-map encoding) does not set a floor under short kernels."""
        side = torch.cuda.Stream(device=dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            fn()
            fn()
        torch.cuda.current_stream(dev).wait_stream(side)
        torch.cuda.synchronize(dev)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for _ in range(reps):
                fn()
        graph.replay()
        torch.cuda.synchronize(dev)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        graph.replay()
        b.record()
        b.synchronize()
        del graph
        return a.elapsed_time(b) / reps * 1e-3

    mean_len = float(np.mean(lengths))
    # The engine's joint plan (cross-attention over these lengths + backbone self-attention), as svx_engine_set_lengths
    # builds it.
    cap = k0.shape[2]
    plan = ops.attention_multi_plan([(lengths, cap), (None, cfg.patches)], SLOTS, heads, cfg.patches,
                                    torch.cuda.get_device_properties(dev).multi_processor_count, dev)
    cross = dict(q=ws['qx'], k=k0, v=v0, keys=cap, q_row_stride=d, kv_slot_stride=heads * cap * 96,
                 kv_head_stride=cap * 96, kv_row_stride=96, lengths=forward.engine.lengths, out=ws['ax'])
    self_ = dict(q=ws['qkv'], k=ws['qkv'][:, d:], v=ws['qkv'][:, 2 * d:], keys=cfg.patches, q_row_stride=3 * d,
                 kv_slot_stride=cfg.patches * 3 * d, kv_head_stride=96, kv_row_stride=3 * d, out=ws['attn'])
    self_flops = 4.0 * SLOTS * heads * cfg.patches * cfg.patches * 96
    nc = len(cfg.layer_indices)   # control layers: each has a cross-attention, a joint launch and a projection group
    kernels = {
        # as the engine runs them: the LayerNorm folded into qkv / fc1 / head, row statistics from fc2 / proj / zero
        'gemm_qkv_rope': (lambda: ops.gemm(ws['xb'], bw['qkv_fold'][0], bw['attn.qkv.bias'], _lib.EPI_ROPE,
                                           out=ws['qkv'], rope=tables, rope_cols=2 * d, rows_per_slot=cfg.patches,
                                           ln=(stats, *bw['qkv_fold'][1:], 1e-6)),
                          2.0 * rows * d * 3 * d, 2 * cfg.depth),
        'gemm_fc1_gelu': (lambda: ops.gemm(ws['xb'], bw['fc1_fold'][0], bw['mlp.0.bias'], _lib.EPI_BIAS_GELU,
                                           out=ws['mlp'], ln=(stats, *bw['fc1_fold'][1:], 1e-6)),
                          2.0 * rows * d * cfg.mlp, 2 * cfg.depth),
        'gemm_fc2_gate': (lambda: ops.gemm(ws['mlp'], bw['mlp.2.weight'], bw['mlp.2.bias'], _lib.EPI_GATE_RESIDUAL,
                                           out=ws['xb'], gate=bw['gate2'], residual=ws['xb'], stats_out=stats),
                          2.0 * rows * cfg.mlp * d, 2 * cfg.depth),
        'gemm_dxd': (lambda: ops.gemm(ws['attn'], bw['attn.proj.weight'], bw['attn.proj.bias'],
                                      _lib.EPI_GATE_RESIDUAL, out=ws['xb'], gate=bw['gate1'], residual=ws['xb'],
                                      stats_out=stats),
                     2.0 * rows * d * d, 3 * nc),   # control proj, cross query, zero
        # a control layer's cross projection (gate of ones: the plain residual) with its backbone block's attention
        # projection in one launch, as the engine runs them
        'gemm_dxd_group': (lambda: ops.gemm_group([
            dict(a=ws['ax'], w=cw['proj.weight'], bias=cw['proj.bias'], gate=ones, residual=ws['xc'],
                 stats_out=forward.engine.stats['c'], out=ws['xc']),
            dict(a=ws['attn'], w=bw['attn.proj.weight'], bias=bw['attn.proj.bias'], gate=bw['gate1'], residual=ws['xb'],
                 stats_out=stats, out=ws['xb'])]), 2 * 2.0 * rows * d * d, nc),
        'gemm_head': (lambda: ops.gemm(ws['xb'], m.head_fold[0], m.head_b, _lib.EPI_CLASS_MAJOR, out=forward.logits,
                                       rows_per_slot=cfg.patches, classes=cfg.classes, geometry=cfg.voxel_shape,
                                       ln=(stats, *m.head_fold[1:], 1e-6)),
                      2.0 * rows * d * 64 * cfg.classes, 1),
        # the control branch's self-attention (alone: the cross-attention that follows depends on it)
        'attention_self': (lambda: ops.attention(ws['qkv'], ws['qkv'][:, d:], ws['qkv'][:, 2 * d:], SLOTS, heads,
                                                 cfg.patches, cfg.patches, q_row_stride=3 * d,
                                                 kv_slot_stride=cfg.patches * 3 * d, kv_head_stride=96,
                                                 kv_row_stride=3 * d, out=ws['attn']), self_flops, nc),
        # the cross-attention with the backbone's self-attention in one launch
        'attention_joint': (lambda: ops.attention_multi([cross, self_], SLOTS, heads, cfg.patches, plan),
                            4.0 * SLOTS * heads * cfg.patches * mean_len * 96 + self_flops, nc),
        'ease_scores': (lambda: ops.ease_scores(forward.logits, batch.status, out=batch.scores),
                        float(forward.logits.numel() * 2 + batch.scores.numel() * 4), 1),
        # both branches' embed of the slots' current tokens with the first LayerNorms' chunk statistics; bytes: tokens
        # in, y-embeddings in, rows and statistics out (the 2 x 25 MB tables are gathered from L2)
        'patch_embed': (lambda: ops.patch_embed(forward.tokens, cfg.classes, m.table_b, m.bias_b, m.yadd_b, m.table_c,
                                                m.bias_c, m.yadd_c, out_b=ws['xb'], out_c=ws['xc'], stats_b=stats,
                                                stats_c=forward.engine.stats['c']),
                        float(forward.tokens.numel() * 2 + 2 * cfg.patches * d * 2 + 2 * rows * d * 2
                              + 2 * (d // 32) * rows * 8), 1),
    }
    out = {}
    for name, (fn, work, count) in kernels.items():
        t = clock(fn)
        out[name] = dict(seconds=t, work=work, per_step=count, share_seconds=t * count)
    return out


def cpu_baseline(cfg, sd, lengths, sample=1, warmup=1):
    """The reference's CPU path (oracle port: fp32 torch forward + numpy EASE step) on the host cores for `sample`
    slot-forwards of the same workload (one slot at the mean packed K/V length of the bench's slots), after `warmup`
    untimed ones, in committed voxels/s. Runs with no other process of the job alive (the GPU ranks have returned), on
    every core the process may use."""
    from oracle import model as om
    from oracle import sampler as osm
    threads = len(os.sched_getaffinity(0)) if hasattr(os, 'sched_getaffinity') else (os.cpu_count() or 1)
    torch.set_num_threads(threads)
    cfgd = dict(num_classes=cfg.classes, voxel_shape=cfg.voxel_shape, patch_size=4, depth=cfg.depth,
                num_heads=cfg.heads, y_range=cfg.y_range, layer_indices=list(cfg.layer_indices))
    rng = np.random.default_rng(1)
    length = int(round(float(np.mean(lengths))))
    kv = [(torch.randn(1, cfg.heads, length, 96), torch.randn(1, cfg.heads, length, 96)) for _ in cfg.layer_indices]
    tokens = torch.full((1, *cfg.voxel_shape), cfg.classes, dtype=torch.long)
    total = int(np.prod(cfg.voxel_shape))
    quotas = osm.low_entropy_last_quotas(total, CAP, 0)

    def one(s):
        logits = om.control_forward(sd, tokens, kv, cfgd)[0].numpy()
        slot = osm.Slot(cfg.voxel_shape, cfg.classes, (0,), 0, 1e-4, 4)
        slot.arm(s, CAP, (), rng.permutation(total // 64))
        slot.phase, slot.quotas, slot.last = 'solid', quotas, np.zeros(cfg.voxel_shape, bool)
        slot.solid_calls = 0
        slot.consume(logits, tokens[0].numpy().copy(), native=True)

    with torch.no_grad():
        for s in range(warmup):
            one(sample + s)
        began = time.perf_counter()
        for s in range(sample):
            one(s)
    seconds = (time.perf_counter() - began) / sample
    per_forward = total / (1 + len(quotas))   # voxels a slot commits per forward, averaged over its window
    return dict(value=per_forward / seconds, unit=UNIT, cores=threads, kind='port',
                warmup=warmup, sample=f'{sample} slot-forward(s) of the bench model (d={cfg.d}, {cfg.depth} + '
                       f'{len(cfg.layer_indices)} layers; fp32, K/V length {length}) + one EASE solid step on '
                       f'[{cfg.classes}, 65536]; {seconds:.2f} s each; voxels/s = 65536/33 per slot-forward')


def main_ours(args):
    """Time the step on this rank's GPU; returns (the JSON line without its CPU baseline, cfg, sd, lengths) on rank 0
    and None elsewhere. Every rank takes the same collective steps in the same order."""
    rank, world, local = dist_env()
    if world > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group('nccl', timeout=datetime.timedelta(seconds=300))
    device = torch.device('cuda', local)
    torch.cuda.set_device(device)
    from streamvoxel_b200 import _lib
    _lib.require_device(device)
    # Weak scaling: every rank runs the same per-GPU workload (the same weights and the same eight windows'
    # conditions, so the same packed key lengths as at N = 1); only the sampled windows' seeds differ by rank. With
    # per-rank conditions the slowest rank's longer keys, not the GPUs, set the max-over-ranks time.
    cfg, sd, forward, batch, lengths = build(device, seed=0)
    seeds = list(range(rank * 1_000_000, rank * 1_000_000 + 100_000))
    # warm-up: W forwards through the public step path
    run_api_steps(batch, max(3, args.warmup), iter(seeds[50_000:]))
    for i in range(batch.slots):
        batch.state[i] = dict(phase='idle')

    def barrier():
        torch.cuda.synchronize(device)
        if world > 1:
            import torch.distributed as dist
            dist.barrier()
        torch.cuda.synchronize(device)

    def gather(obj):
        if world == 1:
            return [obj]
        import torch.distributed as dist
        out = [None] * world
        dist.all_gather_object(out, obj)
        return out

    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(local) as clocks:
        barrier()
        start.record()
        committed, launches, markings = run_device_steps(batch, args.steps, iter(seeds))
        stop.record()
        barrier()
    own_seconds = start.elapsed_time(stop) * 1e-3
    # end to end through the public step API (host scalars in, commits out, host bookkeeping), same step count
    for i in range(batch.slots):
        batch.state[i] = dict(phase='idle')
    barrier()
    start.record()
    e2e_committed, h2d, d2h = run_api_steps(batch, args.steps, iter(seeds[10_000:]))
    stop.record()
    barrier()
    own_e2e = start.elapsed_time(stop) * 1e-3
    kernels = time_kernels(cfg, forward, batch, lengths)
    ranks = gather(dict(rank=rank, ms_per_step=own_seconds / args.steps * 1e3,
                        e2e_ms_per_step=own_e2e / args.steps * 1e3, committed=committed, e2e_committed=e2e_committed,
                        mean_packed_keys=float(np.mean(lengths)), clocks=clocks.summary()))
    if rank != 0:
        return None
    seconds = max(r['ms_per_step'] for r in ranks) * args.steps * 1e-3   # max over ranks
    e2e_seconds = max(r['e2e_ms_per_step'] for r in ranks) * args.steps * 1e-3
    value = sum(r['committed'] for r in ranks) / seconds
    e2e_value = sum(r['e2e_committed'] for r in ranks) / e2e_seconds
    peaks = json.load(open(os.path.join(ROOT, 'MEASURED_PEAKS.json'))) if os.path.exists(
        os.path.join(ROOT, 'MEASURED_PEAKS.json')) else {}
    dominant = max(kernels, key=lambda k: kernels[k]['share_seconds'])
    kd = kernels[dominant]
    if dominant in BYTE_KERNELS:
        peak, unit, bound, src = peaks.get('hbm_gbs', 6650.0), 'GB/s', 'hbm', 'measured' if peaks else 'fallback'
        achieved = kd['work'] / kd['seconds'] / 1e9
    else:
        peak, unit, bound = peaks.get('bf16_tflops', 1590.0), 'TFLOP/s', 'tensor'
        src = 'measured (burst; kernel timed alone)' if peaks else 'fallback'
        achieved = kd['work'] / kd['seconds'] / 1e12
    traffic = None
    if dominant in MEASURED_TRAFFIC:
        measured, captured_alg = MEASURED_TRAFFIC[dominant]
        traffic = measured * algorithmic_bytes(dominant, cfg, lengths) / captured_alg
    step_flops = sum(k['work'] * k['per_step'] for n, k in kernels.items() if n not in BYTE_KERNELS)
    steps_per_s = args.steps / seconds
    line = dict(
        metric=METRIC, value=value, unit=UNIT, n_gpus=world, steps=args.steps, warmup=args.warmup,
        ms_per_step=seconds / args.steps * 1e3, higher_is_better=True, scaling='weak', vs_baseline=None,
        dtype='bf16', data='synthetic (seeded world generator, random-init N(0,0.02) weights)',
        config=bench_config(lengths, world),
        sampler='EASE, native Gumbel-max Philox draw (bit-exact with its host restatement)',
        forwards_per_s=steps_per_s * world, marking_forwards=markings,
        e2e=dict(value=e2e_value, unit=UNIT, h2d_bytes_per_step=h2d / args.steps, d2h_bytes_per_step=d2h / args.steps),
        gpu_launches=launches,
        roofline=dict(kernel=dominant, bound=bound, achieved=achieved, peak=peak, unit=unit, frac=achieved / peak,
                      peak_source=src, traffic=traffic, traffic_unit='bytes per launch (ncu, scaled)',
                      algorithmic=f"{kd['work']:.4g} {'bytes' if bound == 'hbm' else 'FLOP'} per launch"),
        step_tflops=step_flops / (seconds / args.steps) / 1e12,
        kernels={k: dict(us=v['seconds'] * 1e6, per_step=v['per_step'],
                         rate=(v['work'] / v['seconds'] / (1e9 if k in BYTE_KERNELS else 1e12)))
                 for k, v in kernels.items()},
        clocks=clocks.summary(),
        per_rank=[dict(rank=r['rank'], ms_per_step=r['ms_per_step'], e2e_ms_per_step=r['e2e_ms_per_step'],
                       mean_packed_keys=r['mean_packed_keys'], sm_mhz=r['clocks'].get('sm_mhz'),
                       reasons=r['clocks'].get('reasons')) for r in ranks])
    return line, cfg, sd, lengths


def main_reference(args):
    """The reference's CPU path on the host cores (rank 0 only), on this arm's config, metric and unit: each step is one
    bounded sample (one slot-forward of the workload's model at the bench's mean packed key length + one EASE solid
    step), at most 3 timed samples after 3 untimed ones."""
    rank, world, _ = dist_env()
    if rank != 0:
        return
    from streamvoxel_b200 import model as sm
    cfg = model_config()
    sd = sm.synthetic_state_dict(cfg, seed=0)
    _, _, lengths = bench_items(cfg, 0)
    steps = min(max(1, args.steps), 3)
    warmup = 3   # untimed samples first (thread pool, allocator, first-touch), as many as the rules ask of any arm
    began = time.perf_counter()
    result = cpu_baseline(cfg, sd, lengths, steps, warmup=warmup)
    seconds = time.perf_counter() - began
    line = dict(metric=METRIC, value=result['value'], unit=UNIT, n_gpus=world, steps=steps, warmup=warmup,
                higher_is_better=True, scaling='weak', vs_baseline=None, dtype='f32', data='synthetic', impl='reference',
                config=bench_config(lengths, world), cpu_baseline=result,
                e2e=dict(value=result['value'], unit=UNIT, h2d_bytes_per_step=0, d2h_bytes_per_step=0),
                seconds=seconds)
    print(json.dumps(line), flush=True)


def main_expand(args):
    """a committed side0^2 start region grown to side1^2 columns through the public engine API
    (`SlotBatch`, window admission, per-window condition encoding, commits), one engine per GPU; the ranks exchange
    finished columns on the host (a gloo group). The timed region is the whole expansion (CUDA events on each rank,
    max over ranks); `value` = committed voxels of all ranks / that time. Returns the JSON line on rank 0."""
    rank, world, local = dist_env()
    group = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group('nccl', timeout=datetime.timedelta(seconds=600))
        group = dist.new_group(backend='gloo', timeout=datetime.timedelta(seconds=600))
    device = torch.device('cuda', local)
    torch.cuda.set_device(device)
    from streamvoxel_b200 import _lib
    from streamvoxel_b200.stream import expand
    _lib.require_device(device)
    cfg, sd, forward, batch, lengths = build(device, seed=0)
    run_api_steps(batch, max(3, args.warmup), iter(range(10_000, 20_000)))   # warm-up through the step API
    for i in range(batch.slots):
        batch.state[i] = dict(phase='idle')
    committed, region, biomes, player = expand.start_region(11, args.side0, args.side1, forward.spec,
                                                            classes=cfg.classes)
    exp = expand.Expansion(committed, biomes, forward.spec, player, region, ranks=world, slots=SLOTS, l2_cap=L2_CAP)
    exchange = None   # one rank: nothing to exchange
    if world > 1:     # finished columns and free slots over NCCL, on a stream of their own
        import torch.distributed as dist
        exchange = expand.DeviceExchange(dist.group.WORLD, SLOTS, forward.shape, device)

    def barrier():
        torch.cuda.synchronize(device)
        if world > 1:
            import torch.distributed as dist
            dist.barrier()
        torch.cuda.synchronize(device)

    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    batch.timing, batch.device_seconds = True, 0.0
    with Clocks(local) as clocks:
        barrier()
        start.record()
        stats = expand.run(batch, exp, rank, group=group, exchange=exchange)
        stop.record()
        barrier()
    seconds = start.elapsed_time(stop) * 1e-3
    stats['step_device_seconds'] = batch.device_seconds   # the step graphs' own device time (the rest: gaps)
    ranks = expand.host_exchange(dict(rank=rank, seconds=seconds, stats=stats, digest=exp.digest(),
                                      clocks=clocks.summary()), group)
    if rank != 0:
        return None
    wall = max(r['seconds'] for r in ranks)
    voxels = sum(r['stats']['committed_voxels'] for r in ranks)
    forwards = sum(r['stats']['forwards'] for r in ranks)
    windows = sum(r['stats']['windows'] for r in ranks)
    config = dict(workload=WORKLOAD, slots_per_gpu=SLOTS, cap=CAP, l1_cap=L1_CAP, l2_cap=L2_CAP, side0=args.side0,
                  side1=args.side1, admission='pick_window order around the player at the region centre, Chebyshev >= 2',
                  l2_policy='inputs larger than L2 (the step reads all weights and writes all logits: >= 1 GB)',
                  parallelism=f'dp{world}: one engine per GPU, finished columns all-gathered over NCCL each round')
    per_step_h2d = batch.params_host.numel()
    line = dict(metric=METRIC, value=voxels / wall, unit=UNIT, n_gpus=world, steps=forwards, warmup=args.warmup,
                ms_per_step=wall / max(1, forwards / world) * 1e3, higher_is_better=True, scaling='strong',
                vs_baseline=None, dtype='bf16', data='synthetic (seeded world generator, random-init N(0,0.02) weights)',
                config=config, windows=windows, committed_voxels=voxels, seconds=wall,
                replicas_agree=len({r['digest'] for r in ranks}) == 1,
                e2e=dict(value=voxels / wall, unit=UNIT, h2d_bytes_per_step=per_step_h2d,
                         d2h_bytes_per_step=None,
                         note='the expansion is timed end to end through the public API (item building, encoding, '
                              'steps, commits, host exchange): value and e2e are the same measurement'),
                gpu_launches=forwards * batch.launches(),
                clocks=clocks.summary(),
                per_rank=[dict(rank=r['rank'], seconds=r['seconds'], sm_mhz=r['clocks'].get('sm_mhz'),
                               reasons=r['clocks'].get('reasons'),
                               **{k: (round(v, 3) if isinstance(v, float) else v) for k, v in r['stats'].items()})
                          for r in ranks])
    return line


def main():
    args = parse()
    if args.impl == 'reference':
        main_reference(args)
        return
    result = None
    try:
        result = main_expand(args) if args.workload == 'config4' else main_ours(args)
    finally:
        import torch.distributed as dist
        if dist.is_available() and dist.is_initialized():
            dist.barrier()
            dist.destroy_process_group()
    if result is None:
        return
    if args.workload == 'config4':
        print(json.dumps(result), flush=True)
        return
    line, cfg, sd, lengths = result
    # The CPU baseline runs after the process group is gone and the other ranks have returned, so no waiting rank
    # spins on a host core while it is timed.
    if line['n_gpus'] > 1:
        time.sleep(2.0)
    line['cpu_baseline'] = cpu_baseline(cfg, sd, lengths, args.cpu_sample)
    print(json.dumps(line), flush=True)


if __name__ == '__main__':
    main()
