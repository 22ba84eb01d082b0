"""Regenerates the golden fixtures from the REFERENCE implementation itself.

Run in a container where the reference checkout exists (path in REF_DIR or
the first argument).  Inputs come from attn_bwd_b200.generate.generate_input on
the CPU (a restatement of eval_modal_attn_bwd.py:139-169), outputs from the
reference's own ``attn_bwd/starting_point.py::custom_kernel`` run on the CPU.
Small cases store inputs and outputs; the config-0 case stores outputs and a
SHA-256 of each input (the inputs are regenerated from the seed at test time).

    python tests/golden/make_golden.py /path/to/reference
"""
import hashlib
import importlib.util
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "..", "..", "sol-1-advisor-token-fix_b200"))
from attn_bwd_b200.generate import generate_input  # noqa: E402

# (name, bs, sq, skv, seed, p, store_inputs)
CASES = [
    ("tiny_aligned", 1, 8, 16, 11, 0.1, True),
    ("tiny_ragged", 1, 5, 13, 12, 0.1, True),
    ("tiny_p0", 1, 4, 32, 13, 0.0, True),
    ("rows_over_block", 1, 130, 16, 14, 0.1, False),
    ("ragged_cols", 1, 3, 70, 15, 0.1, True),
    ("config0", 2, 64, 96, 1000, 0.1, False),
]


def u16(t):
    return t.contiguous().view(torch.int16).numpy().view(np.uint16) if t.dtype == torch.bfloat16 else t.numpy()


def sha(t):
    return hashlib.sha256(t.contiguous().view(torch.uint8).numpy().tobytes()).hexdigest() \
        if t.dtype != torch.bool else hashlib.sha256(t.numpy().tobytes()).hexdigest()


def main():
    ref = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("REF_DIR")
    spec = importlib.util.spec_from_file_location("starting_point", os.path.join(ref, "attn_bwd", "starting_point.py"))
    sp = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(sp)
    torch.manual_seed(0)
    for name, bs, sq, skv, seed, p, store in CASES:
        data = generate_input(bs, sq, skv, seed, dropout_p=p)
        with torch.no_grad():
            dS, dV = sp.custom_kernel(data)
        arrs = {"meta": np.array([bs, sq, skv, seed]), "p": np.array([p], dtype=np.float64),
                "dS": u16(dS), "dV": u16(dV)}
        names = ["grad_attn_output", "attn_weights", "attn_weights_dropped", "value_states", "dropout_mask"]
        for n, t in zip(names, data[:5]):
            if store:
                arrs["in_" + n] = u16(t)
            arrs["sha_" + n] = np.frombuffer(sha(t).encode(), dtype=np.uint8)
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **arrs)
        print(name, {k: v.shape for k, v in arrs.items()})


if __name__ == "__main__":
    main()
