"""The commit wire format (streamvoxel_b200.stream.wire) against fixtures made by the reference's live protocol code
(`tests/golden/make_golden.py --only wire`): frame rows byte-identical, merges, packet hashes and batch lines."""
import json
import os

import numpy as np
import pytest

from streamvoxel_b200.stream import wire

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), 'golden')


def _g():
    return np.load(os.path.join(GOLDEN, 'wire.npz'))


def test_frame_rows_are_byte_identical():
    g = _g()
    for i in range(12):
        want = json.loads(str(g[f'r{i}_row']))
        got = wire.pack_row(want['target'], g[f'r{i}_positions'], g[f'r{i}_raw'])
        assert json.dumps(got, sort_keys=True) == json.dumps(want, sort_keys=True), i
        pos, ids = wire.unpack_row(want)
        np.testing.assert_array_equal(pos, g[f'r{i}_unpacked_pos'])
        np.testing.assert_array_equal(ids, g[f'r{i}_unpacked_val'])


def test_unpack_rejects_a_tampered_row():
    g = _g()
    row = json.loads(str(g['r3_row']))
    row['sparse_sha256'] = '0' * 64
    with pytest.raises(ValueError):
        wire.unpack_row(row)


def test_merge_commits_matches_reference():
    g = _g()
    for i in range(6):
        commits = [dict(positions=g[f'm{i}_c{j}_positions'], values=g[f'm{i}_c{j}_values'], step=j + 1, target=(3, -4))
                   for j in range(int(g[f'm{i}_count']))]
        merged = wire.merge_commits(commits)
        np.testing.assert_array_equal(merged['positions'], g[f'm{i}_positions'])
        np.testing.assert_array_equal(merged['values'], g[f'm{i}_values'])


def test_packets_and_batch_lines_match_reference():
    g = _g()
    packets = json.loads(str(g['packets']))
    for seq, packet in enumerate(packets):
        assert wire.packet_sha(packet) == packet['sha256']
        wire.verify_packet(packet, seq)
        body = {k: v for k, v in packet.items() if k not in ('seq', 'kind', 'sha256')}
        assert wire.make_packet(seq, packet['kind'], **body)['sha256'] == packet['sha256']
    line = wire.batch_line(packets)
    assert json.dumps(line, sort_keys=True) == str(g['batch'])
    assert wire.unbatch(line) == packets


def test_finished_window_packet_round_trip():
    column = np.random.default_rng(0).integers(0, 40, (64, 16, 16)).astype(np.int16)
    raw_map = np.arange(40, dtype=np.uint16) * 3
    commit = wire.whole_cell_commit((2, 5), column, 33)
    row = wire.frame_row(commit, raw_map, slot=3, gpu=1)
    pos, ids = wire.unpack_row(row)
    flat = raw_map[column.reshape(-1)]
    np.testing.assert_array_equal(pos, np.flatnonzero(flat != 0))
    np.testing.assert_array_equal(ids, flat[flat != 0])
    assert row['row'] == 67 and row['committed'] == column.size
    fields = wire.window_commit_fields(dict(target=(2, 5), nfe=33, last_frac=0.5, cap=32, actual=32), 1, 3, 2)
    packet = wire.make_packet(0, 'window_commit', **fields)
    assert wire.verify_packet(packet, 0) is packet
