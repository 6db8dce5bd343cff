"""The config-1 driver: one column decoded from all-MASK by the time-free model on our engine and the shipped sampler."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_decode_low_entropy_last_completes_and_is_deterministic():
    from streamvoxel_b200 import model as sm
    from streamvoxel_b200.decode import UnconditionalForward, decode_low_entropy_last
    from streamvoxel_b200.sampling import low_entropy_last_quotas
    cfg = sm.small_test_config(layer_indices=())
    forward = UnconditionalForward(cfg, sm.synthetic_state_dict(cfg, seed=1, std=0.05))
    spec = dict(air_ids=(0,), air_token=0, last_eps=1e-4, block_size=4, steps=16)
    runs = [decode_low_entropy_last(forward, spec, 7, 'cuda', cfg.voxel_shape, cfg.classes) for _ in range(2)]
    (result, info), (again, _) = runs
    assert info['complete'] and info['nfe'] == 1 + len(low_entropy_last_quotas(
        int(np.prod(cfg.voxel_shape)), 16, info['last_count'], 'quartercos'))
    tokens, steps = result['compact'], result['commit_step']
    assert tokens.min() >= 0 and tokens.max() < cfg.classes          # every voxel decoded, no mask id left
    assert steps.min() >= 1 and steps.max() == info['nfe']            # every voxel has a commit step
    assert np.array_equal(tokens, again['compact']) and np.array_equal(steps, again['commit_step'])
