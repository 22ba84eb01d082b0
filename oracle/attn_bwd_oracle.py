"""CPU fp32 oracle for GQA attention backward — TEST INFRASTRUCTURE ONLY.

A restatement, in plain fp32 PyTorch on the CPU, of the reference's
``custom_kernel`` in attn_bwd/starting_point.py:27-70 (identical to the
evaluator's ``ref_kernel``, eval_modal_attn_bwd.py:96-135).  It is the checker
the parity tests compare the CUDA path against and the CPU implementation the
bench's reference arm times; the product never calls it.

Parity is pinned: tests/golden/ holds outputs of the reference's own
starting_point.custom_kernel on seeded inputs (tests/golden/make_golden.py), and
tests/test_oracle.py checks this restatement against them.
"""
import torch

H, KVH, G, D = 80, 8, 10, 128


def attn_bwd_reference(data):
    """(dS, dV) for the reference 6-tuple; all math in fp32, outputs bf16.

    Step by step (starting_point.py line numbers):
      40-42  V is shared by the 10 query heads of each KV head
      45     dO -> [bs, h, sq, d] fp32
      48     dP~ = dO @ V^T
      51-54  dP = dP~ * mask / (1 - p) if p > 0 else dP~
      57-59  dS = P * (dP - sum_j(dP * P)) -> bf16
      62-64  dV_h = P_drop^T @ dO
      67-68  dV = sum over the 10 heads of each group -> bf16
    """
    dO, P, Pd, V, mask, p = data
    bs, sq = dO.shape[0], dO.shape[1]
    skv = V.shape[2]
    dOf = dO.transpose(1, 2).float()                               # [bs, 80, sq, d]
    Vf = V.float().repeat_interleave(G, dim=1)                      # [bs, 80, skv, d]
    dPt = torch.matmul(dOf, Vf.transpose(-2, -1))                   # [bs, 80, sq, skv]
    if p > 0.0:
        dP = dPt * mask / (1.0 - p)
    else:
        dP = dPt
    Pf = P.float()
    r = (dP * Pf).sum(dim=-1, keepdim=True)
    dS = (Pf * (dP - r)).to(torch.bfloat16)
    dVh = torch.matmul(Pd.float().transpose(-2, -1), dOf)           # [bs, 80, skv, d]
    dV = dVh.view(bs, KVH, G, skv, D).sum(dim=2).to(torch.bfloat16)
    return dS, dV


def attn_bwd_units(data, units):
    """Oracle restricted to a list of units u = b*8 + kv_head.

    Returns {u: (dS [10, sq, skv], dV [skv, 128])}.  Each unit only reads its own
    batch row, heads 10*kvh..10*kvh+9 and V[b, kvh], so this is the full oracle's
    result for those units at a fraction of the memory (used for the large
    configs, whose full fp32 oracle needs tens of GB).
    """
    dO, P, Pd, V, mask, p = data
    out = {}
    for u in units:
        b, kvh = divmod(int(u), KVH)
        hs = slice(kvh * G, kvh * G + G)
        sub = (dO[b:b + 1, :, hs].cpu(),
               P[b:b + 1, hs].cpu(), Pd[b:b + 1, hs].cpu(),
               V[b:b + 1, kvh:kvh + 1].cpu(), mask[b:b + 1, hs].cpu(), p)
        dS, dV = _attn_bwd_group(sub)
        out[u] = (dS[0], dV[0, 0])
    return out


def _attn_bwd_group(sub):
    """Same math as attn_bwd_reference for one KV group (10 heads, 1 KV head)."""
    dO, P, Pd, V, mask, p = sub
    bs = dO.shape[0]
    skv = V.shape[2]
    dOf = dO.transpose(1, 2).float()
    Vf = V.float().expand(bs, G, skv, D)
    dPt = torch.matmul(dOf, Vf.transpose(-2, -1))
    dP = dPt * mask / (1.0 - p) if p > 0.0 else dPt
    Pf = P.float()
    dS = (Pf * (dP - (dP * Pf).sum(dim=-1, keepdim=True))).to(torch.bfloat16)
    dV = torch.matmul(Pd.float().transpose(-2, -1), dOf).sum(dim=1, keepdim=True).to(torch.bfloat16)
    return dS, dV
