"""The batched PyTorch CPU restatement of the DiT velocity forward
(oracle/torch_cpu.py, timed by bench.py as the batched CPU throughput line)
against the C oracle: masked v4 layout with position ids, and the plain
layout without mask."""
import numpy as np

import oracle as O
import synth
import torch_cpu
from helpers import rel


def test_batched_cpu_velocity_matches_oracle(orc):
    w = synth.dit_weights(1, n_layers=2)
    L, fm, patch = 16, 12, 4
    m = torch_cpu.BatchedDiT(w, 2)
    x = synth.normal(3, "tc.x", (3, L, 1024), 1.0)
    cond = synth.normal(3, "tc.c", (3, 1024), 1.0)
    for mask, pos in ((orc.fm_mask(L, fm, patch), orc.fm_pos(L, fm, patch)), (None, None)):
        want = np.stack([orc.dit_velocity(w, 2, x[r], cond[r], mask, pos, n_out=patch) for r in range(3)])
        got = m.velocity(x, cond, mask, pos, n_out=patch)
        assert rel(got, want) <= 1e-5
