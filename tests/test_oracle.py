"""The CPU oracle against the reference's own outputs (golden fixtures)."""
import pytest
import torch

from golden_io import CASES, load_case
from oracle.attn_bwd_oracle import attn_bwd_reference, attn_bwd_units


@pytest.mark.parametrize("name", CASES)
def test_oracle_matches_reference_outputs(name):
    data, dS_ref, dV_ref, _ = load_case(name)
    dS, dV = attn_bwd_reference(data)
    assert dS.shape == dS_ref.shape and dV.shape == dV_ref.shape
    assert dS.dtype == torch.bfloat16 and dV.dtype == torch.bfloat16
    # same fp32 math on the same CPU: at most one bf16 rounding step apart
    torch.testing.assert_close(dS.float(), dS_ref.float(), rtol=8e-3, atol=1e-6)
    torch.testing.assert_close(dV.float(), dV_ref.float(), rtol=8e-3, atol=1e-6)
    frac_exact = (dS == dS_ref).float().mean().item()
    assert frac_exact > 0.999


def test_inputs_regenerate_bit_identically():
    # config0 and rows_over_block store only hashes: load_case asserts the hashes
    for name in ("config0", "rows_over_block"):
        _, _, _, regenerated = load_case(name)
        assert regenerated


def test_unit_oracle_equals_full_oracle():
    data, _, _, _ = load_case("config0")
    dS, dV = attn_bwd_reference(data)
    units = [0, 5, 8, 15]
    got = attn_bwd_units(data, units)
    for u in units:
        b, kvh = divmod(u, 8)
        torch.testing.assert_close(got[u][0].float(), dS[b, kvh * 10:kvh * 10 + 10].float(), rtol=8e-3, atol=1e-6)
        torch.testing.assert_close(got[u][1].float(), dV[b, kvh].float(), rtol=8e-3, atol=1e-6)


def test_generator_distribution():
    from attn_bwd_b200.generate import generate_input
    dO, P, Pd, V, M, p = generate_input(1, 16, 64, 7)
    assert P.dtype == torch.bfloat16 and M.dtype == torch.bool and p == 0.1
    torch.testing.assert_close(P.float().sum(-1), torch.ones(1, 80, 16), atol=2e-2, rtol=0)
    keep = M.float().mean().item()
    assert 0.85 < keep < 0.95
    torch.testing.assert_close(Pd.float(), (P.float() * M / 0.9).to(torch.bfloat16).float())
