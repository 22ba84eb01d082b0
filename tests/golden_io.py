"""Loads the golden fixtures written by tests/golden/make_golden.py."""
import hashlib
import os

import numpy as np
import torch

from attn_bwd_b200.generate import generate_input

GOLDEN_DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
CASES = ["tiny_aligned", "tiny_ragged", "tiny_p0", "rows_over_block", "ragged_cols", "config0"]
NAMES = ["grad_attn_output", "attn_weights", "attn_weights_dropped", "value_states", "dropout_mask"]


def _bf16(a):
    return torch.from_numpy(a.view(np.int16).copy()).view(torch.bfloat16)


def _sha(t):
    if t.dtype == torch.bool:
        return hashlib.sha256(t.numpy().tobytes()).hexdigest()
    return hashlib.sha256(t.contiguous().view(torch.uint8).numpy().tobytes()).hexdigest()


def load_case(name):
    """Returns (data_tuple_on_cpu, expected_dS, expected_dV, regenerated: bool)."""
    z = np.load(os.path.join(GOLDEN_DIR, name + ".npz"))
    bs, sq, skv, seed = (int(x) for x in z["meta"])
    p = float(z["p"][0])
    if "in_grad_attn_output" in z:
        ins = []
        for n in NAMES:
            a = z["in_" + n]
            ins.append(torch.from_numpy(a.copy()) if a.dtype == np.bool_ else _bf16(a))
        data = tuple(ins) + (p,)
        regenerated = False
    else:
        data = generate_input(bs, sq, skv, seed, dropout_p=p)
        regenerated = True
    for n, t in zip(NAMES, data[:5]):
        want = bytes(z["sha_" + n]).decode()
        assert _sha(t) == want, f"{name}: input {n} differs from the fixture (generator drift)"
    return data, _bf16(z["dS"]), _bf16(z["dV"]), regenerated
