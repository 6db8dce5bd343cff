"""CPU oracle for the StreamVoxel column-generation hot path.

TEST INFRASTRUCTURE ONLY. The oracle restates the reference algorithms (zzf1955/StreamVoxel) on the CPU,
each function citing the reference file:line it follows. Only `tests/`, `__graft_entry__.smoke()` and the
CPU-baseline legs of `bench.py` may import it, and only as the checker or the timed CPU baseline. The product
package `streamvoxel_b200` never imports anything from here.

Pinning: `tests/golden/make_golden.py` imports the reference (in the build container only) and writes seeded
input/output fixtures to `tests/golden/*.npz`; `tests/test_oracle_golden.py` checks this oracle against them.

* `sampler`  - EASE sampler: entropy, 4^3 block-quota selection, low-entropy-last marking, quartercos quotas,
               the categorical draw rule, Philox4x32-10, and a whole-window slot.
* `eval_samplers` - the evaluation decoders (random / entropy / mixed / block selections, every schedule).
* `model`    - time-free DiT + compact ControlNet forward (fp32 torch on the CPU, optional bf16 rounding points)
               and the condition encoder.

The seeded synthetic inputs (columns, conditions, logits with the BASELINE shapes) are the product's own
`streamvoxel_b200.synth`, shared by the tests, the bench and the oracle checks.
"""
