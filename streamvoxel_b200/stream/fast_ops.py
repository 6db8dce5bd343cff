"""Drop-in for the reference's live slot path (`streamvoxel/stream/fast_ops.py`) on libsvx.

* `FastSlotForward` (`fast_ops.py:164-376`): same attributes and methods the worker uses (tokens, shape, batch, sizes,
  graphs, graph, outputs, packed.lengths, load_slot, wait_loads, clear_tokens, bucket, replay, eager, _call,
  numerical_gate). The forward is one `svx_engine_forward` (tcgen05 GEMMs, fused epilogues, varlen attention over the
  packed K/V) captured in one CUDA graph per slot bucket. Tokens are int16 (the mask id V does not fit uint8).
* `FastLowEntropyLastSlot` (`fast_ops.py:481-581`): the reference slot whose marking, selection, draw and commit run
  in libsvx. `sampling='parity'` takes the categorical draw's exponential noise from the slot's torch generator (the
  same call `torch.multinomial` makes), so commits equal the reference's given the same logits; `sampling='native'`
  draws with counter-based Philox on the device (Gumbel-max, no generator, fully graph-capturable, reproduced bit for
  bit by the host restatement in the oracle).
* `SelectGraphs` (`fast_ops.py:584-623`) and `consume_batch` (`fast_ops.py:626-642`): per-(bucket, slot) captured
  selection and one host wait per forward.
"""
from __future__ import annotations

import json

import numpy as np
import torch

from streamvoxel_b200 import _lib, ops
from streamvoxel_b200.model import Engine
from streamvoxel_b200.modules import prepared_model
from streamvoxel_b200.sampling import actual_time, low_entropy_last_quotas
from streamvoxel_b200.stream.condition import largest_item, probe_item

KEY_BLOCK = 128
RECOMMENDED = dict(patchify='gather', attention='flex', compile='emulate')


class PackedKeys:
    """The view of the engine's packed keys the worker reads (`fast_ops.py:122-147`): lengths per slot."""

    def __init__(self, engine):
        self.engine = engine
        self.lengths = engine.lengths
        self.keys = engine.key_capacity
        self.kv = engine.kv


class FastSlotForward:
    """Slot-batched forward over cached packed K/V (`streamvoxel/stream/fast_ops.py:164-376`)."""

    def __init__(self, model, spec, device, batch, l1_cap, l2_cap, *, patchify='gather', attention='flex',
                 compile=False, capture=True):
        if patchify not in ('gather', 'conv') or attention not in ('flex', 'sdpa'):
            raise ValueError('patchify must be gather|conv and attention flex|sdpa')
        if compile not in (False, True, 'emulate'):
            raise ValueError("compile must be False, True or 'emulate'")
        self.device = torch.device(device)
        _lib.require_device(self.device)
        # a reference CompactStreamingControlNet (as `worker.py:272` passes it), a (ModelConfig, state dict) pair or a
        # PreparedModel
        model = prepared_model(model, self.device)
        self.model, self.spec = model, spec
        self.l2_cache = None   # created on the first item that names its L2 columns (`Item.l2_keys`)
        cfg = model.cfg
        self.cfg = cfg
        self.batch, self.l1_cap, self.l2_cap = int(batch), int(l1_cap), int(l2_cap)
        self.classes = spec.num_classes
        if self.classes != cfg.classes or (spec.height, spec.tile, spec.tile) != tuple(cfg.voxel_shape):
            raise ValueError('ModelSpec does not match the model configuration')
        self.shape = (spec.height, spec.tile, spec.tile)
        self.options = dict(patchify=patchify, attention=attention, compile=compile)
        l1, l2, biome = cfg.condition_widths()
        self.l1_tokens, self.l2_tokens, self.biome_tokens = l1, l2, biome
        self.prefix_len = l2_cap * l2
        self.local_len = l1_cap * l1 + biome
        keys = self.prefix_len + self.local_len
        keys += (-keys) % KEY_BLOCK
        self.engine = Engine(model, self.batch, keys)
        self.packed = PackedKeys(self.engine)
        self.tokens = torch.full((self.batch, *self.shape), self.classes, dtype=torch.int16, device=self.device)
        self.timestep = torch.ones(self.batch, device=self.device)
        self.logits = torch.zeros((self.batch, self.classes, *self.shape), dtype=torch.bfloat16, device=self.device)
        probe = self.encode(probe_item(spec))
        for slot in range(self.batch):
            self.engine.write_slot(slot, probe)
        self.side = torch.cuda.Stream(device=self.device)          # slot writes: ordered after the queued steps
        self.encoder = torch.cuda.Stream(device=self.device)       # condition encodes: never wait for a step
        # One encode of the largest condition the slots hold (l1_cap L1 tiles, l2_cap L2 columns), on the encoder
        # stream, so that the memory pool already holds blocks of every size later encodes ask for: a device
        # allocation while steps are queued would stall the device (it synchronises).
        with torch.cuda.stream(self.encoder):
            self.encode(largest_item(spec, self.l1_cap, self.l2_cap))
        torch.cuda.synchronize(self.device)
        self.sizes = sorted({min(self.batch, 2 ** k) for k in range(self.batch.bit_length() + 1)})
        self.graphs, self.outputs = {}, {}
        self.graph_ok = False
        if capture:
            self._capture()
        self.graph = self.graphs.get(self.batch)

    # -- conditions
    def encode(self, item):
        """Per-layer packed (K, V) [H, P+L, 96] of one item (`fast_ops.py:228-239`)."""
        keys = getattr(item, 'l2_keys', None)
        if keys is not None and self.l2_cache is None:
            from streamvoxel_b200.model import L2TokenCache
            self.l2_cache = L2TokenCache()
        layers = self.model.encode_item(item.l1_blocks, item.l1_xz, item.l2_blocks, item.l2_xz, item.biomes,
                                        l2_keys=keys, cache=self.l2_cache)
        prefix = len(item.l2_blocks) * self.l2_tokens
        if prefix > self.prefix_len or layers[0][0].shape[1] - prefix > self.local_len:
            raise ValueError('Condition exceeds the slot capacity')
        return layers

    def load_slot(self, index, item):
        """Encode + copy off the caller's stream; `wait_loads` joins it before the next replay
        (`fast_ops.py:252-260`). The encode reads only the item and the weights, so it runs on its own stream that
        never waits for a step (its host inputs go through pinned memory: the host never waits either); the copy into
        the slot's K/V rows and tokens runs on the side stream after the encode and after the work already queued on
        the caller's stream, and the slot's key length is applied by `wait_loads`. Encodes of several slots therefore
        queue back to back, not each behind the previous slot's copy."""
        with torch.cuda.stream(self.encoder):
            layers = self.encode(item)
        self.side.wait_stream(self.encoder)
        self.side.wait_stream(torch.cuda.current_stream(self.device))
        for k, v in layers:   # made on the encoder stream, read on the side stream
            k.record_stream(self.side)
            v.record_stream(self.side)
        with torch.cuda.stream(self.side):
            self.engine.write_slot(index, layers, defer=True)
            self.tokens[index].fill_(self.classes)

    def wait_loads(self):
        torch.cuda.current_stream(self.device).wait_stream(self.side)
        self.engine.apply_lengths()

    def clear_tokens(self):
        self.wait_loads()
        self.tokens.fill_(self.classes)

    def bucket(self, count):
        return next(size for size in self.sizes if size >= max(1, count))

    # -- forward
    def _call(self, size=None):
        n = self.batch if size is None else size
        self.engine.forward(n, self.tokens, self.logits)
        return self.logits[:n]

    def _capture(self):
        current = torch.cuda.current_stream(self.device)
        warm = torch.cuda.Stream(device=self.device)
        warm.wait_stream(current)
        with torch.cuda.stream(warm):
            for size in self.sizes:
                for _ in range(3):
                    self._call(size)
        current.wait_stream(warm)
        torch.cuda.synchronize(self.device)
        stream = torch.cuda.Stream(device=self.device)
        try:
            for size in reversed(self.sizes):
                graph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(graph, stream=stream, capture_error_mode='thread_local'):
                    self.outputs[size] = self._call(size)
                self.graphs[size] = graph
            self.graph_ok = True
        except Exception as error:  # same fallback event as the reference (`fast_ops.py:334-337`)
            self.graphs, self.outputs = {}, {}
            self.graph_ok = False
            print(json.dumps(dict(event='cuda_graph_fallback', device=str(self.device),
                                  error=f'{type(error).__name__}: {error}')), flush=True)

    def replay(self, timestep, count=None):
        """Logits [bucket, V, Y, Z, X] of the first bucket(count) slots (`fast_ops.py:339-345`). The time-free model
        ignores the timestep; it is stored for API parity."""
        self.timestep.copy_(torch.as_tensor(timestep, dtype=self.timestep.dtype, device=self.device))
        size = self.batch if count is None else self.bucket(count)
        if size not in self.graphs:
            return self._call(size)
        self.graphs[size].replay()
        return self.outputs[size]

    def eager(self, timestep):
        self.timestep.copy_(torch.as_tensor(timestep, dtype=self.timestep.dtype, device=self.device))
        return self._call()

    def launches(self, count=None):
        """Kernel launches in one replay of bucket(count)."""
        return self.engine.launches(self.batch if count is None else self.bucket(count))

    @torch.inference_mode()
    def numerical_gate(self, item, other=None):
        """`FastSlotForward.numerical_gate` (`fast_ops.py:352-375`) with the same report keys. The packed-vs-unpadded
        check compares slot 0 of the batched forward with a single-slot forward of the same item (packing and
        batching invariance); the reference-model comparison lives in the test suite."""
        self.load_slot(0, item)
        if other is not None and self.batch > 1:
            self.load_slot(1, other)
        self.wait_loads()
        time = torch.ones(self.batch, device=self.device)
        eager = self.eager(time).clone()
        replayed = self.replay(time).clone() if self.graph is not None else eager
        equal = self.graph is not None and bool(torch.equal(eager, replayed))
        single = self._call(1)[:1].clone()
        gap = (eager[0].float() - single[0].float()).abs()
        match = float((eager[0].argmax(0) == single[0].argmax(0)).float().mean())
        mean_abs = float(gap.mean())
        lead = min(2, self.batch)
        small = self.replay(time, lead)[:lead].float()
        bucket_match = float((small.argmax(1) == eager[:lead].argmax(1)).float().mean())
        bucket_close = bucket_match >= 0.999 and float((small - eager[:lead].float()).abs().mean()) <= 0.05
        return dict(graph_equal=equal, graph_used=self.graph is not None,
                    padded_close=bool(match >= 0.999 and mean_abs <= 0.05), bucket_close=bool(bucket_close),
                    bucket_match=bucket_match, buckets=sorted(self.graphs) or [], max_abs=float(gap.max()),
                    mean_abs=mean_abs, argmax_match=match, batch=self.batch, prefix_len=self.prefix_len,
                    local_len=self.local_len, options=self.options)


class LowEntropyLastSlot:
    """Host state of one window (`streamvoxel/stream/slot.py:50-176`); the device work is in the subclass."""

    def __init__(self, shape, classes, air_ids, air_token, last_eps, block_size, device):
        self.shape = tuple(shape)
        self.total = int(np.prod(self.shape))
        self.classes = int(classes)
        self.air_ids = tuple(air_ids)
        self.air_token = int(air_token)
        self.last_eps = float(last_eps)
        self.block_size = int(block_size)
        self.device = torch.device(device)
        self.phase = 'idle'
        self.target = self.seed = self.cap = self.quotas = self.order = self.generator = None
        self.solid_calls = self.actual = self.nfe = self.last_count = 0
        self.step_map = torch.zeros(self.shape, dtype=torch.int16)
        self.values = torch.full(self.shape, -1, dtype=torch.int16)

    @property
    def idle(self):
        return self.phase == 'idle'

    def arm(self, seed, cap, target, *, order=None):
        """`slot.py:86-103`: block order from Generator(seed + 9173), sample generator on seed. `order` replaces the
        block permutation (for a caller that replays a window whose order another device drew: `torch.randperm`
        gives different permutations on the CPU and on CUDA for the same seed)."""
        self.phase = 'marking'
        self.seed, self.cap, self.target = int(seed), int(cap), tuple(target)
        self.nfe = self.actual = self.solid_calls = 0
        self.quotas = None
        self.last_count = 0
        blocks = self.total // self.block_size ** 3
        if order is None:
            order_rng = torch.Generator(device=self.device).manual_seed(self.seed + 9173)
            self.order = torch.randperm(blocks, device=self.device, generator=order_rng)
        else:
            self.order = torch.as_tensor(order, dtype=torch.long, device=self.device)
            if sorted(self.order.tolist()) != list(range(blocks)):
                raise ValueError(f'order must be a permutation of the {blocks} blocks')
        self.generator = torch.Generator(device=self.device).manual_seed(self.seed)
        self.step_map = torch.zeros(self.shape, dtype=torch.int16)
        self.values = torch.full(self.shape, -1, dtype=torch.int16)

    def drop(self):
        self.phase = 'idle'
        self.target = None
        self.quotas = None

    def time(self, tokens=None):
        """`slot.py:110-115`."""
        if self.phase == 'idle':
            return 1.0
        committed = sum(self.quotas[:self.solid_calls]) if self.quotas else 0
        return actual_time((self.total - committed) / self.total)


class FastLowEntropyLastSlot(LowEntropyLastSlot):
    """`FastLowEntropyLastSlot` (`fast_ops.py:481-581`) on libsvx: marking, entropy, block-quota selection, the draw
    and the token commit run on the device; one D2H copy and one host wait per solid step."""

    def __init__(self, *args, entropy='torch', sampling='parity', **kwargs):
        super().__init__(*args, **kwargs)
        # Parity mode: a callable (k, classes) -> fp32 device tensor [k, classes] that replaces the exponential draws
        # from the slot generator (a replay of draws recorded elsewhere); None draws them from the generator.
        self.noise_source = None
        if entropy not in ('torch', 'triton'):
            raise ValueError('entropy must be torch or triton')
        if sampling not in ('parity', 'native'):
            raise ValueError('sampling must be parity or native')
        if self.block_size != 4:
            raise ValueError('the selection kernel implements 4^3 blocks')
        _lib.require_device(self.device)
        self.entropy_name, self.sampling = entropy, sampling
        dev = self.device
        blocks = self.total // 64
        self.air_dev = torch.as_tensor(self.air_ids, dtype=torch.int32, device=dev)
        self.last_static = torch.zeros((1, *self.shape), dtype=torch.uint8, device=dev)
        self.last_count_dev = torch.zeros(1, dtype=torch.int32, device=dev)
        self.pos = torch.zeros((1, blocks), dtype=torch.int32, device=dev)
        self.params = torch.zeros(32, dtype=torch.uint8, device=dev)
        self._params_host = torch.zeros(32, dtype=torch.uint8, pin_memory=True)
        self.scores = torch.zeros((1, *self.shape), dtype=torch.float32, device=dev)
        self.chosen = torch.zeros((1, *self.shape), dtype=torch.uint8, device=dev)
        self.index = torch.zeros((1, self.total), dtype=torch.int32, device=dev)
        self.count = torch.zeros(1, dtype=torch.int32, device=dev)
        self.status = torch.zeros(1, dtype=torch.int32, device=dev)
        self.values_dev = torch.zeros((1, self.total), dtype=torch.int16, device=dev)
        self.workspace = ops.select_workspace(1, self.total, dev)
        self._host = torch.empty(2 * self.total + 1, dtype=torch.int32, pin_memory=True)

    def arm(self, seed, cap, target, *, order=None):
        super().arm(seed, cap, target, order=order)
        self.last_static.zero_()
        self.pos[0, self.order] = torch.arange(len(self.order), device=self.device, dtype=torch.int32)

    @property
    def last(self):
        """The deferred-voxel mask [Y, Z, X] bool on the device (the reference slot's `last`)."""
        return self.last_static[0].bool()

    def stageable(self):
        return self.phase == 'solid' and self.quotas is not None and self.solid_calls < len(self.quotas)

    def mark(self, logits):
        """Marking forward (`slot.py:124-136`): the last mask on the device, one host read of its count."""
        self.nfe += 1
        ops.ease_mark(logits[None], self.air_dev, self.last_eps, last=self.last_static, last_count=self.last_count_dev)
        self.last_count = int(self.last_count_dev.item())
        self.quotas = low_entropy_last_quotas(self.total, self.cap, self.last_count, 'quartercos')
        self.phase = 'solid'
        self.solid_calls = 0

    def prepare(self):
        """Per-step scalars into the static params buffer (`fast_ops.py:519-532`)."""
        k = self.quotas[self.solid_calls]
        committed = sum(self.quotas[:self.solid_calls])
        frac = (committed + k) / (self.total - self.last_count)
        arr = np.zeros(1, ops.STEP_DTYPE)
        arr[0] = (k, self.nfe + 1, committed, frac, self.seed & 0xFFFFFFFFFFFFFFFF)
        self._params_host.copy_(torch.from_numpy(arr.view(np.uint8)))
        self.params.copy_(self._params_host, non_blocking=True)
        self.status.zero_()
        return k

    def select(self, logits, tokens):
        """Graph-capturable: entropy + block-quota selection into the static buffers (`fast_ops.py:534-540`)."""
        ops.ease_scores(logits[None], self.status, out=self.scores)
        ops.ease_select(self.scores, tokens[None], self.last_static, self.pos, self.params, self.classes, self.total,
                        chosen=self.chosen, index=self.index, count=self.count, status=self.status,
                        workspace=self.workspace)

    def stage(self, logits, tokens, graph=None):
        """Select, draw and commit on the device, then one async D2H of (index, values, status) (`fast_ops.py:542-558`)."""
        if tokens.dtype != torch.int16:
            raise ValueError('slot tokens must be int16 (FastSlotForward.tokens rows)')
        k = self.prepare()
        if graph is None:
            self.select(logits, tokens)
        else:
            graph.replay()
        noise = None
        if self.sampling == 'parity' and self.noise_source is not None:
            noise = torch.as_tensor(self.noise_source(k, self.classes), dtype=torch.float32,
                                    device=self.device).reshape(1, k, self.classes).contiguous()
        elif self.sampling == 'parity':
            # The exponential draws torch.multinomial(probabilities, 1, generator) makes (`slot.py:150`).
            noise = torch.empty((1, k, self.classes), device=self.device).exponential_(generator=self.generator)
        ops.ease_sample(logits[None], self.index, self.params, tokens[None], noise=noise, values=self.values_dev,
                        status=self.status)
        host = self._host
        host[:k].copy_(self.index[0, :k], non_blocking=True)
        host[k:2 * k].copy_(self.values_dev[0, :k], non_blocking=True)
        host[2 * k:2 * k + 1].copy_(self.status, non_blocking=True)
        event = torch.cuda.Event()
        event.record()
        return k, host, event, tokens

    def collect(self, staged):
        """Wait for the step's copy and do the host bookkeeping (`fast_ops.py:560-576`)."""
        k, host, event, tokens = staged
        event.synchronize()
        if int(host[2 * k]) & _lib.STATUS_QUOTA_MISSED:
            raise AssertionError('low-entropy-last solid step did not meet its quota')
        positions = host[:k].long().clone()
        values_cpu = host[k:2 * k].to(torch.int16)
        self.solid_calls += 1
        self.actual += 1
        self.nfe += 1
        self.step_map.reshape(-1)[positions] = self.nfe
        self.values.reshape(-1)[positions] = values_cpu
        commit = dict(positions=positions.numpy().astype('int32'), values=values_cpu.numpy(), step=int(self.nfe))
        if self.solid_calls >= len(self.quotas):
            return self._finish(tokens), commit
        return None, commit

    def consume(self, logits, tokens):
        """One forward for this slot (`slot.py:117-164`); tokens [Y,Z,X] int16 updated in place."""
        if self.phase == 'idle':
            return None, None
        if self.phase == 'marking':
            self.mark(logits)
            if not self.quotas:
                return self._finish(tokens), None
            return None, None
        if not self.stageable():
            return self._finish(tokens), None
        return self.collect(self.stage(logits, tokens))

    def _finish(self, tokens):
        """`slot.py:166-176`: deferred voxels take air_token; the record goes to the caller."""
        last = self.last_static[0].bool()
        tokens.masked_fill_(last, self.air_token)
        last_cpu = last.cpu()
        self.step_map[last_cpu] = self.nfe
        self.values[last_cpu] = self.air_token
        record = dict(target=self.target, seed=self.seed, cap=self.cap, nfe=int(self.nfe), actual=int(self.actual),
                      last_count=int(self.last_count), last_frac=float(self.last_count) / self.total,
                      step_map=self.step_map.clone(), values=self.values.clone())
        self.phase = 'idle'
        self.target = None
        return record


class SelectGraphs:
    """One captured `FastLowEntropyLastSlot.select` per (bucket, slot) over the engine's static outputs and token rows
    (`fast_ops.py:584-623`). `lookup(logits)` returns the bucket whose output `logits` is."""

    def __init__(self, engine, slots):
        self.engine, self.slots = engine, slots
        self.graphs = {}
        if not getattr(engine, 'graphs', None):
            return
        device = engine.device
        current = torch.cuda.current_stream(device)
        warm = torch.cuda.Stream(device=device)
        warm.wait_stream(current)
        with torch.cuda.stream(warm), torch.inference_mode():
            for size, out in engine.outputs.items():
                for i in range(size):
                    slots[i].select(out[i], engine.tokens[i])
        current.wait_stream(warm)
        torch.cuda.synchronize(device)
        stream = torch.cuda.Stream(device=device)
        pool = torch.cuda.graph_pool_handle()   # one memory pool for every (bucket, slot) capture
        with torch.inference_mode():
            for size, out in sorted(engine.outputs.items()):
                for i in range(size):
                    graph = torch.cuda.CUDAGraph()
                    with torch.cuda.graph(graph, pool=pool, stream=stream, capture_error_mode='thread_local'):
                        slots[i].select(out[i], engine.tokens[i])
                    self.graphs[size, i] = graph
        for slot in slots:
            slot.chosen.zero_()
            slot.status.zero_()

    def lookup(self, logits):
        for size, out in self.engine.outputs.items():
            if logits.data_ptr() == out.data_ptr() and len(logits) == len(out):
                return size
        return None


def consume_batch(slots, logits, tokens, count, graphs=None):
    """`[slot.consume(logits[i], tokens[i]) for i < count]` with every staged solid step enqueued before the first
    host wait (`fast_ops.py:626-642`). Returns {index: (finished, commit)} for the non-idle slots."""
    size = graphs.lookup(logits) if graphs is not None else None
    staged, results = {}, {}
    for index in range(count):
        slot = slots[index]
        if slot.idle:
            continue
        if isinstance(slot, FastLowEntropyLastSlot) and slot.stageable():
            graph = graphs.graphs.get((size, index)) if graphs is not None and size is not None else None
            staged[index] = slot.stage(logits[index], tokens[index], graph)
        else:
            results[index] = slot.consume(logits[index], tokens[index])
    for index, item in staged.items():
        results[index] = slots[index].collect(item)
    return dict(sorted(results.items()))
