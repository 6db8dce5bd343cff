"""All slots of one engine stepping together: the worker's engine step (`streamvoxel/stream/worker.py:378-399`) as one
CUDA graph per step -- the slot-batched forward, then entropy, block-quota selection, the categorical draw and the
token commit for every slot in the same graph, with no host read inside.

Per-window work stays outside the graph, as in the reference: the block order (`torch.randperm` on the device with the
window seed + 9173, `streamvoxel/stream/slot.py:97-99`), the marking forward's last mask and its count (one host read,
`slot.py:130`) and the quartercos quota list. Slots that are marking, finished or idle take k = 0 in the step graph.

Two draws (`sampling`):
* 'native' -- the Gumbel-max draw on counter-based Philox keyed by (slot seed, step, voxel, class): nothing outside
  the graph, reproducible bit for bit by a host restatement;
* 'parity' -- the reference's draw: each solid step's exponential noise is drawn from the slot's own torch generator
  (seeded with the window seed, the call `torch.multinomial(p, 1, generator)` makes, `streamvoxel/stream/slot.py:150`)
  into a static device buffer before the graph replays, and the graph's draw takes argmax(softmax(x) / q) with torch's
  row-softmax order, so every commit equals the reference slot's given the same logits. The noise fill is a device
  kernel per solid slot, enqueued before the replay; the host does not wait for it.

Two drivers:
* `step()` -- one forward for every armed slot with the host bookkeeping of `consume_batch`: per-step scalars copied
  H2D from pinned memory, commits copied D2H and returned (the worker-facing path, one host wait per forward);
* `run_cycles(n)` -- n whole windows per slot back to back on the device: the scalars of every step are staged once per
  window, so the host never waits inside a window (device-resident throughput).
"""
from __future__ import annotations

from collections import deque

import numpy as np
import torch

from streamvoxel_b200 import ops
from streamvoxel_b200.sampling import counts, low_entropy_last_quotas

EASE_LAUNCHES = 5   # scores, quota, block select, fix-up/compaction, sample


class SlotBatch:
    def __init__(self, forward, *, air_ids=(0,), air_token=0, last_eps=1e-4, block_size=4, sampling='native',
                 min_cap=32):
        """`min_cap`: the smallest window cap `arm` accepts in parity mode; it sizes the static noise buffer (the
        largest quota of a cap-step quartercos schedule, times the classes, per slot)."""
        if sampling not in ('native', 'parity'):
            raise ValueError('sampling must be native or parity')
        if block_size != 4:
            raise ValueError('the selection kernel implements 4^3 blocks')
        self.sampling = sampling
        self.forward = forward
        self.device = forward.device
        self.slots = forward.batch
        self.shape = forward.shape
        self.total = int(np.prod(self.shape))
        self.classes = forward.classes
        self.air_ids, self.air_token, self.last_eps = tuple(air_ids), int(air_token), float(last_eps)
        dev, b = self.device, self.slots
        self.blocks = self.total // 64
        self.air_dev = torch.as_tensor(self.air_ids, dtype=torch.int32, device=dev)
        self.params = torch.zeros(b * ops.STEP_DTYPE.itemsize, dtype=torch.uint8, device=dev)
        self.params_host = torch.zeros(b * ops.STEP_DTYPE.itemsize, dtype=torch.uint8, pin_memory=True)
        self.params_host_sets = [torch.zeros_like(self.params_host).pin_memory() for _ in range(2)]
        self.pos = torch.zeros((b, self.blocks), dtype=torch.int32, device=dev)
        self.last = torch.zeros((b, *self.shape), dtype=torch.uint8, device=dev)
        self.last_count = torch.zeros(b, dtype=torch.int32, device=dev)
        self.scores = torch.zeros((b, *self.shape), dtype=torch.float32, device=dev)
        self.chosen = torch.zeros((b, *self.shape), dtype=torch.uint8, device=dev)
        self.index = torch.zeros((b, self.total), dtype=torch.int32, device=dev)
        self.count = torch.zeros(b, dtype=torch.int32, device=dev)
        self.status = torch.zeros(b, dtype=torch.int32, device=dev)
        self.values = torch.zeros((b, self.total), dtype=torch.int16, device=dev)
        self.workspace = ops.select_workspace(b, self.total, dev)
        # Flat pinned staging for the commits, one set per step that may be in flight: a step's [slots, kmax] copy
        # lands in the first slots * kmax entries as one contiguous block (a strided pinned destination would make the
        # copy wait on the host).
        self.host_index_flat = [torch.zeros(b * self.total, dtype=torch.int32, pin_memory=True) for _ in range(2)]
        self.host_values_flat = [torch.zeros(b * self.total, dtype=torch.int16, pin_memory=True) for _ in range(2)]
        self.host_small_sets = [torch.zeros(2 * b, dtype=torch.int32, pin_memory=True) for _ in range(2)]
        self.state = [dict(phase='idle') for _ in range(b)]
        self.noise = None
        self.generators = [None] * b
        self._queue = deque()   # launched, uncollected steps, oldest first (at most `depth`)
        # a finishing window's tokens and its deferred-voxel mask, copied to the host by the step that finishes it and
        # by its marking step, so its committed column is ready when that step is collected
        self._final_tokens = torch.zeros((b, *self.shape), dtype=torch.int16, pin_memory=True)
        self._final_last = torch.zeros((b, *self.shape), dtype=torch.uint8, pin_memory=True)
        self._launches = 0
        # device time of the steps (step graph + marking), accumulated by `collect` when `timing` is on
        self.timing, self.device_seconds, self._timing_events = False, 0.0, None
        if sampling == 'parity':
            self.min_cap = int(min_cap)
            self.noise_capacity = max(counts(self.total, self.min_cap, 'quartercos'))
            self.noise = torch.ones((b, self.noise_capacity, self.classes), dtype=torch.float32, device=dev)
        self.graph = None
        self._capture()

    # -- device work of one step
    def _ease(self):
        logits = self.forward.logits
        ops.ease_scores(logits, self.status, out=self.scores)
        ops.ease_select(self.scores, self.forward.tokens, self.last, self.pos, self.params, self.classes, self.total,
                        chosen=self.chosen, index=self.index, count=self.count, status=self.status,
                        workspace=self.workspace)
        ops.ease_sample(logits, self.index, self.params, self.forward.tokens, noise=self.noise, values=self.values,
                        status=self.status)

    def _device_step(self):
        self.forward._call(self.slots)
        self._ease()

    def _capture(self):
        self.params.zero_()
        current = torch.cuda.current_stream(self.device)
        warm = torch.cuda.Stream(device=self.device)
        warm.wait_stream(current)
        with torch.cuda.stream(warm):
            for _ in range(3):
                self._device_step()
        current.wait_stream(warm)
        torch.cuda.synchronize(self.device)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=torch.cuda.Stream(device=self.device), capture_error_mode='thread_local'):
            self._device_step()
        self.graph = graph

    def launches(self):
        """Kernel launches in one step graph."""
        return self.forward.engine.launches(self.slots) + EASE_LAUNCHES

    # -- windows
    def arm(self, slot, seed, cap, item=None, target=(), *, order=None, wait=True):
        """Start a window in `slot` (`LowEntropyLastSlot.arm`, `slot.py:86-103`); `item` loads its conditions.
        `order` replaces the block permutation drawn from Generator(seed + 9173). With `wait=False` the condition
        encode stays on the engine's side stream, joined by the next `launch` (the reference's `load_slot` then
        `wait_loads` before the replay, `streamvoxel/stream/fast_ops.py:252-264`): a slot may be armed while another
        step is in flight, since the side stream first waits for the work already enqueued."""
        if self.sampling == 'parity' and int(cap) < self.min_cap:
            raise ValueError(f'cap {cap} is below min_cap {self.min_cap}, which sized the parity noise buffer')
        if any(slot in entry['slots'] for entry in self._queue):
            raise ValueError(f'slot {slot} takes part in a step in flight; collect it first')
        if item is not None:
            self.forward.load_slot(slot, item)
            if wait:
                self.forward.wait_loads()
        else:
            self.forward.tokens[slot].fill_(self.classes)
        if order is None:
            g = torch.Generator(device=self.device).manual_seed(int(seed) + 9173)
            order = torch.randperm(self.blocks, device=self.device, generator=g)
        else:
            order = torch.as_tensor(order, dtype=torch.long, device=self.device)
        self.pos[slot, order] = torch.arange(self.blocks, device=self.device, dtype=torch.int32)
        if self.sampling == 'parity':
            self.generators[slot] = torch.Generator(device=self.device).manual_seed(int(seed))
        self.last[slot].zero_()
        self.state[slot] = dict(phase='marking', seed=int(seed), cap=int(cap), target=tuple(target), nfe=0,
                                solid_calls=0, quotas=None, last_count=0, launched=0, nfe_launched=0)

    def _rows(self):
        rows = []
        for st in self.state:
            if st['phase'] == 'solid' and st['solid_calls'] < len(st['quotas']):
                k = st['quotas'][st['solid_calls']]
                committed = sum(st['quotas'][:st['solid_calls']])
                frac = (committed + k) / (self.total - st['last_count'])
                rows.append((k, st['nfe'] + 1, committed, frac, st['seed']))
            else:
                rows.append((0, 0, 0, 0.0, 0))
        return rows

    def _pack(self, rows):
        arr = np.zeros(len(rows), ops.STEP_DTYPE)
        for i, row in enumerate(rows):
            arr[i] = (row[0], row[1], row[2], row[3], row[4] & 0xFFFFFFFFFFFFFFFF)
        return torch.from_numpy(arr.view(np.uint8))

    def _mark(self, marking):
        """One marking launch per run of consecutive slots."""
        logits = self.forward.logits
        slots = sorted(marking)
        while slots:
            n = 1
            while n < len(slots) and slots[n] == slots[0] + n:
                n += 1
            lo, hi = slots[0], slots[0] + n
            ops.ease_mark(logits[lo:hi], self.air_dev, self.last_eps, last=self.last[lo:hi],
                          last_count=self.last_count[lo:hi])
            slots = slots[n:]

    def _after_mark(self, marking, counts):
        finished = []
        for i in marking:
            st = self.state[i]
            st['nfe'] += 1
            st['nfe_launched'] = max(st.get('nfe_launched', 0), st['nfe'])
            st['last_count'] = int(counts[i])
            st['quotas'] = low_entropy_last_quotas(self.total, st['cap'], st['last_count'], 'quartercos')
            st['phase'] = 'solid'
            if not st['quotas']:
                finished.append(i)
        return finished

    def column(self, slot):
        """The slot's tokens as a host int16 array [Y, Z, X] (a finished window's committed column)."""
        return self.forward.tokens[slot].cpu().numpy().astype(np.int16, copy=True)

    def column_async(self, slot):
        """Enqueue the copy of the slot's tokens to pinned host memory; returns a callable that waits for that copy
        only (not for work enqueued after it) and returns the column as `column` does."""
        if not hasattr(self, '_column_host'):
            self._column_host = torch.empty((self.slots, *self.shape), dtype=torch.int16, pin_memory=True)
        host = self._column_host[slot]
        host.copy_(self.forward.tokens[slot], non_blocking=True)
        event = torch.cuda.Event()
        event.record(torch.cuda.current_stream(self.device))

        def result():
            event.synchronize()
            return host.numpy().astype(np.int16, copy=True)
        return result

    def _finish(self, i):
        """`_finish` (`slot.py:166-176`): deferred voxels take air_token; returns the window record."""
        st = self.state[i]
        self.forward.tokens[i].masked_fill_(self.last[i].bool(), self.air_token)
        st['phase'] = 'idle'
        return dict(target=st['target'], seed=st['seed'], cap=st['cap'], nfe=st['nfe'], actual=st['solid_calls'],
                    last_count=st['last_count'], last_frac=st['last_count'] / self.total)

    def _draw_noise(self, rows):
        """Parity mode: each solid slot's exponential draws for this step, from its generator, into the static
        buffer (the same generator call and shape as `torch.multinomial(p[k, C], 1, generator)`)."""
        if self.sampling != 'parity':
            return
        for i, row in enumerate(rows):
            k = row[0]
            if k > self.noise_capacity:
                raise ValueError(f'quota {k} exceeds the parity noise capacity {self.noise_capacity}')
            if k:
                self.noise[i, :k].exponential_(generator=self.generators[i])

    def step(self):
        """One forward for every armed slot with its EASE step; returns {slot: (record|None, commit|None)}."""
        self.launch()
        return self.collect()

    depth = 2   # steps that may be in flight at once

    @property
    def in_flight(self):
        return len(self._queue)

    def runnable(self):
        """Whether a step launched now would give some slot a forward (a marking or a solid step)."""
        return any(st['phase'] == 'marking' or (st['phase'] == 'solid' and st['launched'] < len(st['quotas']))
                   for st in self.state)

    def _rows_ahead(self):
        """Per-slot scalars of the next step to launch: solid steps are counted when launched, so a step can be
        launched while the previous one is still in flight (the schedule of a window is known once it is marked)."""
        rows = []
        for st in self.state:
            if st['phase'] == 'solid' and st['launched'] < len(st['quotas']):
                k = st['quotas'][st['launched']]
                committed = sum(st['quotas'][:st['launched']])
                frac = (committed + k) / (self.total - st['last_count'])
                rows.append((k, st['nfe_launched'] + 1, committed, frac, st['seed']))
            else:
                rows.append((0, 0, 0, 0.0, 0))
        return rows

    def launch(self):
        """Enqueue one step (the step graph, the marking launches and the D2H copies of its results) without waiting
        for it; `collect` waits for the oldest step and does its host bookkeeping. Up to `depth` steps may be in flight:
        a slot whose window was marked in a step still in flight takes no forward in later steps until that step is
        collected (its quotas come from the marking), and a window whose last solid step is in flight takes none."""
        if len(self._queue) >= self.depth:
            raise RuntimeError(f'{self.depth} steps are already in flight; collect one first')
        self.forward.wait_loads()
        marking = [i for i, st in enumerate(self.state) if st['phase'] == 'marking']
        rows = self._rows_ahead()
        solid = [i for i, r in enumerate(rows) if r[0] > 0]
        for i in marking:
            self.state[i]['phase'] = 'marking_sent'
            self.state[i]['nfe_launched'] += 1
        for i in solid:
            self.state[i]['launched'] += 1
            self.state[i]['nfe_launched'] += 1
        buf = self._launches % 2
        self._launches += 1
        # one pinned source per step in flight: the H2D copy reads it when the stream reaches it
        params_host = self.params_host_sets[buf]
        params_host.copy_(self._pack(rows))
        self.params.copy_(params_host, non_blocking=True)
        self.status.zero_()
        self._draw_noise(rows)
        timing = None
        if self.timing:
            timing = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
            timing[0].record()
        self.graph.replay()
        self._mark(marking)
        if self.timing:
            timing[1].record()
        for i in marking:
            self._final_last[i].copy_(self.last[i], non_blocking=True)
        finishing = [i for i in solid if self.state[i]['launched'] == len(self.state[i]['quotas'])]
        for i in finishing:
            self._final_tokens[i].copy_(self.forward.tokens[i], non_blocking=True)
        kmax = max([r[0] for r in rows] + [0])
        host_index = host_values = None
        if kmax:
            host_index = self.host_index_flat[buf][:self.slots * kmax].view(self.slots, kmax)
            host_values = self.host_values_flat[buf][:self.slots * kmax].view(self.slots, kmax)
            host_index.copy_(self.index[:, :kmax], non_blocking=True)
            host_values.copy_(self.values[:, :kmax], non_blocking=True)
        host_small = self.host_small_sets[buf]
        host_small[:self.slots].copy_(self.status, non_blocking=True)
        host_small[self.slots:].copy_(self.last_count, non_blocking=True)
        event = torch.cuda.Event()
        event.record(torch.cuda.current_stream(self.device))
        self._queue.append(dict(marking=marking, rows=rows, solid=solid, slots=set(marking) | set(solid), event=event,
                                index=host_index, values=host_values, small=host_small, timing=timing,
                                finishing=set(finishing)))
        # the params buffer is read by this step's graph; the next launch's H2D copy is queued after it

    def collect(self):
        """Wait for the oldest launched step and book its commits; returns {slot: (record|None, commit|None)}."""
        if not self._queue:
            raise RuntimeError('no step in flight')
        entry = self._queue.popleft()
        marking, rows, solid = entry['marking'], entry['rows'], entry['solid']
        entry['event'].synchronize()
        if entry['timing'] is not None:
            self.device_seconds += entry['timing'][0].elapsed_time(entry['timing'][1]) * 1e-3
        small = entry['small']
        results = {}
        for i in self._after_mark(marking, small[self.slots:].tolist()):
            record = self._finish(i)   # every voxel deferred: the column is all air
            record['column'] = np.full(self.shape, self.air_token, np.int16)
            results[i] = (record, None)
        for i in marking:
            results.setdefault(i, (None, None))
        for i in solid:
            if int(small[i]) & 1:
                raise AssertionError('low-entropy-last solid step did not meet its quota')
            st = self.state[i]
            k = rows[i][0]
            st['solid_calls'] += 1
            st['nfe'] += 1
            commit = dict(positions=entry['index'][i, :k].numpy().copy(), values=entry['values'][i, :k].numpy().copy(),
                          step=st['nfe'])
            record = None
            if st['solid_calls'] >= len(st['quotas']):
                record = self._finish(i)
                if i in entry['finishing']:   # the committed column, deferred voxels as air, without a device wait
                    column = self._final_tokens[i].numpy().copy()
                    column[self._final_last[i].numpy().astype(bool)] = self.air_token
                    record['column'] = column
            results[i] = (record, commit)
        return dict(sorted(results.items()))

    def run_cycles(self, cycles, seeds):
        """`cycles` whole windows in every slot, device-resident: per window one marking forward, one host read of the
        last counts, then every solid step's scalars staged in one H2D copy and replayed back to back. Returns the
        committed voxel count (every window commits all its voxels, the deferred ones at finish)."""
        committed = 0
        dev = self.device
        for c in range(cycles):
            for i in range(self.slots):
                self.arm(i, seeds[c * self.slots + i], 32)
            # marking forward for every slot (params all k = 0)
            self.params.zero_()
            self.graph.replay()
            self._mark(range(self.slots))
            counts = self.last_count.tolist()
            self._after_mark(range(self.slots), counts)
            steps = max(len(st['quotas']) for st in self.state)
            staged, row_list = [], []
            for s in range(steps):
                rows = self._rows()
                staged.append(self._pack(rows))
                row_list.append(rows)
                for st in self.state:
                    if st['solid_calls'] < len(st['quotas']):
                        st['solid_calls'] += 1
                        st['nfe'] += 1
            table = torch.stack(staged).to(dev, non_blocking=False)
            for s in range(steps):
                self.params.copy_(table[s])
                self._draw_noise(row_list[s])
                self.graph.replay()
            for i in range(self.slots):
                self._finish(i)
            committed += self.slots * self.total
        return committed
