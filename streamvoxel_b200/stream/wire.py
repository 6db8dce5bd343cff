"""The commit wire format: what a finished or progressing window sends to a viewer or a coordinator.

Restated from the reference's live protocol so a consumer of its stream can read ours unchanged:
* frame rows (`streamvoxel/common/live_rows.py:42-66`): the visible (non-air) voxels a window committed in one cell,
  positions sorted and stored as uint16 deltas, then their uint16 global block ids, lzma-compressed (preset 2),
  base64-encoded, with a sha256 of the sparse content;
* per-slot commit merging (`streamvoxel/stream/worker.py:90-100`): several forwards of one window become one row, a
  later step winning on a repeated position;
* packets (`streamvoxel/common/live_wire.py:20-25,58-75`): a dict with `seq`, `kind` and a sha256 over its
  sorted-key compact JSON; consecutive packets travel as one zlib (level 6) base64 line.
"""
from __future__ import annotations

import base64
import hashlib
import json
import lzma
import zlib

import numpy as np

KINDS = ('session', 'window_start', 'frame', 'window_commit', 'reset', 'complete', 'failed')


def encoded(data):
    return base64.b64encode(data).decode('ascii')


def decoded(text):
    return base64.b64decode(text, validate=True)


def packet_sha(packet):
    """sha256 of the packet without its `sha256` field, as sorted-key compact JSON."""
    body = {k: v for k, v in packet.items() if k != 'sha256'}
    return hashlib.sha256(json.dumps(body, sort_keys=True, separators=(',', ':')).encode()).hexdigest()


def make_packet(seq, kind, **data):
    if kind not in KINDS:
        raise ValueError(f'Unknown packet kind {kind}')
    packet = dict(seq=int(seq), kind=kind, **data)
    packet['sha256'] = packet_sha(packet)
    return packet


def verify_packet(packet, expected_seq):
    if packet.get('kind') not in KINDS:
        raise ValueError(f'Unknown packet kind {packet.get("kind")}')
    if packet['seq'] != expected_seq or packet_sha(packet) != packet['sha256']:
        raise ValueError('Preview sequence/hash mismatch')
    return packet


def batch_line(packets):
    """Consecutive packets as one transport line; `unbatch` gives them back unchanged."""
    raw = json.dumps(packets, separators=(',', ':')).encode()
    return dict(kind='batch', count=len(packets), z=encoded(zlib.compress(raw, 6)))


def unbatch(line):
    packets = json.loads(zlib.decompress(decoded(line['z'])))
    if len(packets) != line['count']:
        raise ValueError('Batch length mismatch')
    return packets


def _sparse_sha(positions, ids):
    return hashlib.sha256(positions.astype('<u2').tobytes() + ids.astype('<u2').tobytes()).hexdigest()


def pack_row(target, positions, raw):
    """A frame row of cell `target`: `positions` are flat YZX indices of one [256,16,16] column, `raw` their global
    block ids; air (id 0) is left out (the viewer clears a cell when its window starts)."""
    positions = np.asarray(positions, np.int64)
    raw = np.asarray(raw, np.uint16)
    visible = raw != 0
    order = np.argsort(positions[visible], kind='stable')
    pos = positions[visible][order].astype(np.uint16)
    ids = raw[visible][order]
    body = np.diff(pos, prepend=np.uint16(0)).astype('<u2').tobytes() + ids.astype('<u2').tobytes()
    return dict(target=[int(v) for v in target], committed=int(len(raw)), visible=int(len(pos)),
                sparse=encoded(lzma.compress(body, preset=2)), sparse_sha256=_sparse_sha(pos, ids))


def unpack_row(row):
    """(positions int32, global ids uint16) of a frame row, checked against its hash."""
    body = lzma.decompress(decoded(row['sparse']))
    n = int(row['visible'])
    if len(body) != 4 * n:
        raise ValueError('Sparse row length mismatch')
    pos = np.cumsum(np.frombuffer(body[:2 * n], '<u2'), dtype=np.int64).astype(np.uint16)
    ids = np.frombuffer(body[2 * n:], '<u2').astype(np.uint16)
    if _sparse_sha(pos, ids) != row['sparse_sha256']:
        raise ValueError('Sparse row hash mismatch')
    return pos.astype(np.int32), ids


def merge_commits(commits):
    """One commit from several forwards of one window (positions ascending; the later step wins a repeated one)."""
    if len(commits) == 1:
        return commits[0]
    positions = np.concatenate([c['positions'] for c in commits])
    values = np.concatenate([c['values'] for c in commits])
    order = np.argsort(positions, kind='stable')
    positions, values = positions[order], values[order]
    keep = np.append(positions[1:] != positions[:-1], True)
    return dict(positions=positions[keep], values=values[keep], step=commits[-1]['step'], target=commits[-1]['target'])


def frame_row(commit, raw_map, slot, gpu):
    """The frame row of one slot's (merged) commit, compact ids mapped to global ids by `raw_map`; None when the
    commit has no visible voxel. `row` numbers slots across GPUs (64 per GPU)."""
    row = pack_row(commit['target'], commit['positions'], raw_map[np.asarray(commit['values'])])
    if not row['visible']:
        return None
    row.update(row=gpu * 64 + slot, step=commit['step'])
    return row


def whole_cell_commit(target, column, step):
    """The commit of a finished window sent as one row: every voxel of its [Y, Z, X] column."""
    values = np.asarray(column).reshape(-1)
    return dict(positions=np.arange(values.size, dtype=np.int32), values=values, step=int(step), target=tuple(target))


def window_commit_fields(record, gpu, slot, world, seconds=0.0, started_ns=0, finished_ns=0):
    """The fields of a `window_commit` packet for a finished window's record (`SlotBatch` record: target, nfe,
    last_frac, cap, actual)."""
    row = dict(target=[int(v) for v in record['target']], nfe=int(record['nfe']), last_frac=float(record['last_frac']),
               cap=int(record['cap']), seconds=float(seconds), started_unix_ns=int(started_ns),
               finished_unix_ns=int(finished_ns), world=int(world))
    return dict(row, gpu=int(gpu), slot=int(slot), actual=int(record['actual']))


class Publisher:
    """Sequenced, hashed packets kept in memory (a coordinator forwards them, or `batch_line` ships them)."""

    def __init__(self):
        self.packets = []

    def publish(self, kind, **data):
        packet = make_packet(len(self.packets), kind, **data)
        self.packets.append(packet)
        return packet['seq']
