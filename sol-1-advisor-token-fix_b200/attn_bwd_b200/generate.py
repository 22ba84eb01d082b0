"""Seeded inputs with the reference evaluator's distribution.

Restates ``generate_input`` of eval_modal_attn_bwd.py:139-169 (same draw order,
same ops): dO ~ N(0,1) bf16; logits ~ N(0,1) fp32 -> softmax over seq_kv -> bf16
P; mask = U[0,1) > p; P_drop = bf16(P * mask / (1-p)); V ~ N(0,1) bf16.  The
reference draws on a CUDA generator; here the generator's device is a
parameter.  With ``device="cpu"`` the same seed gives bit-identical inputs on
every machine running this torch build, which is what the golden fixtures and
CPU-vs-GPU parity tests rely on.

The module imports nothing from its package, so a CPU-only user (the benchmark's
reference arm) can load it by file path without loading the CUDA library.
"""
import torch

H, KVH, D = 80, 8, 128   # query heads, KV heads, head_dim (starting_point.py:22-24)


def generate_input(batch_size, seq_len_q, seq_len_kv, seed, dropout_p=0.1, device="cpu",
                   out_device=None):
    """Returns the reference's 6-tuple.  ``device`` is where the random numbers
    are drawn (and computed); ``out_device`` (default: same) is where the
    returned tensors live."""
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    bs, sq, skv = batch_size, seq_len_q, seq_len_kv
    dO = torch.randn(bs, sq, H, D, dtype=torch.bfloat16, device=device, generator=g)
    raw = torch.randn(bs, H, sq, skv, dtype=torch.float32, device=device, generator=g)
    P = torch.softmax(raw, dim=-1).to(torch.bfloat16)
    del raw
    mask = torch.rand(bs, H, sq, skv, device=device, generator=g) > dropout_p
    Pd = (P.float() * mask / (1.0 - dropout_p)).to(torch.bfloat16)
    V = torch.randn(bs, KVH, skv, D, dtype=torch.bfloat16, device=device, generator=g)
    out = (dO, P, Pd, V, mask, float(dropout_p))
    if out_device is not None and torch.device(out_device) != torch.device(device):
        out = tuple(t.to(out_device) if isinstance(t, torch.Tensor) else t for t in out)
    return out


def generate_input_lowmem(batch_size, seq_len_q, seq_len_kv, seed, dropout_p=0.1, device="cuda"):
    """Same distribution, drawn one batch row at a time on ``device`` (seed
    seed*1000+b for row b) so that large configs never hold the fp32
    temporaries of the whole tensor.  Not bit-identical to generate_input."""
    bs, sq, skv = batch_size, seq_len_q, seq_len_kv
    dO = torch.empty(bs, sq, H, D, dtype=torch.bfloat16, device=device)
    P = torch.empty(bs, H, sq, skv, dtype=torch.bfloat16, device=device)
    Pd = torch.empty_like(P)
    mask = torch.empty(bs, H, sq, skv, dtype=torch.bool, device=device)
    V = torch.empty(bs, KVH, skv, D, dtype=torch.bfloat16, device=device)
    for b in range(bs):
        d_b, p_b, pd_b, v_b, m_b, _ = generate_input(1, sq, skv, seed * 1000 + b, dropout_p, device)
        dO[b].copy_(d_b[0]); P[b].copy_(p_b[0]); Pd[b].copy_(pd_b[0]); V[b].copy_(v_b[0]); mask[b].copy_(m_b[0])
        del d_b, p_b, pd_b, v_b, m_b
    return dO, P, Pd, V, mask, float(dropout_p)
