"""Every output element of the large BASELINE configs (c2, c3, c4) against an fp32 checker.

The checker is the oracle's per-KV-group restatement of starting_point.py:27-70
(``_attn_bwd_group``: fp32 matmuls, mask and 1/(1-p), row sums, bf16 casts) run on the GPU
one (batch, kv-head) unit at a time, so that the full configs fit; it is test
infrastructure only (library GEMMs are fine here).  TF32 is off, so its matmuls are fp32.

Each case asserts the reference's tolerance (allclose rtol = atol = 1e-2,
eval_modal_attn_bwd.py:173-197) on every unit and prints, per config and output, the
maximum and mean absolute error and the worst margin max(|err| - (atol + rtol*|ref|))
(negative = inside the tolerance).
"""
import json

import pytest
import torch

import attn_bwd_b200 as ab
from attn_bwd_b200.generate import generate_input_lowmem
from oracle.attn_bwd_oracle import _attn_bwd_group

pytestmark = pytest.mark.gpu
RTOL = ATOL = 1e-2
CONFIGS = {"c2": (12, 301, 467), "c3": (2, 2048, 3072), "c4": (48, 640, 640)}


class _Stats:
    def __init__(self):
        self.max_abs = 0.0
        self.sum_abs = 0.0
        self.n = 0
        self.margin = -float("inf")
        self.bad_units = []

    def add(self, u, ref, out):
        ref = ref.float()
        d = (out.float() - ref).abs()
        self.max_abs = max(self.max_abs, d.max().item())
        self.sum_abs += d.sum(dtype=torch.float64).item()
        self.n += d.numel()
        self.margin = max(self.margin, (d - (ATOL + RTOL * ref.abs())).max().item())
        if not torch.allclose(ref, out.float(), rtol=RTOL, atol=ATOL):
            self.bad_units.append(u)

    def summary(self):
        return {"max_abs": self.max_abs, "mean_abs": self.sum_abs / max(self.n, 1),
                "worst_margin": self.margin, "bad_units": self.bad_units[:10]}


@pytest.mark.parametrize("cfg", ["c2", "c3", "c4"])
def test_config_every_unit(cfg, cuda):
    torch.backends.cuda.matmul.allow_tf32 = False
    bs, sq, skv = CONFIGS[cfg]
    data = generate_input_lowmem(bs, sq, skv, 1000 + int(cfg[1]), device=cuda)
    dS, dV = ab.custom_kernel(data)
    torch.cuda.synchronize()
    assert ab.poll_error() == 0
    dO, P, Pd, V, M, p = data
    st_s, st_v = _Stats(), _Stats()
    for u in range(bs * 8):
        b, kvh = divmod(u, 8)
        hs = slice(kvh * 10, kvh * 10 + 10)
        rS, rV = _attn_bwd_group((dO[b:b + 1, :, hs], P[b:b + 1, hs], Pd[b:b + 1, hs],
                                  V[b:b + 1, kvh:kvh + 1], M[b:b + 1, hs], p))
        st_s.add(u, rS[0], dS[b, hs])
        st_v.add(u, rV[0, 0], dV[b, kvh])
    report = {"config": cfg, "shape": [bs, sq, skv], "units": bs * 8,
              "dS": st_s.summary(), "dV": st_v.summary()}
    print("PARITY " + json.dumps(report))
    assert not st_s.bad_units, f"{cfg} dS outside tolerance in units {st_s.bad_units[:10]}"
    assert not st_v.bad_units, f"{cfg} dV outside tolerance in units {st_v.bad_units[:10]}"
