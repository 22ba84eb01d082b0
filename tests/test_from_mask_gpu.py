"""The call without attn_weights_dropped (attn_bwd_b200_shard_from_mask): its dV kernel forms
P_drop = bf16(P * mask / (1-p)) from P and the mask, the identity the reference's inputs are
made with (eval_modal_attn_bwd.py:159-161).  Checked against the oracle run on the generator's
own P_drop, at the reference's tolerance (rtol = atol = 1e-2), and dS against the regular call."""
import pytest
import torch

import attn_bwd_b200 as ab
from attn_bwd_b200.generate import generate_input
from oracle.attn_bwd_oracle import attn_bwd_reference

pytestmark = pytest.mark.gpu


def _to(data, dev):
    return tuple(t.to(dev) if isinstance(t, torch.Tensor) else t for t in data)


@pytest.mark.parametrize("shape,p", [((1, 64, 128), 0.1), ((2, 130, 640), 0.1), ((1, 33, 272), 0.3),
                                     ((1, 64, 96), 0.0), ((3, 17, 16), 0.5)],
                         ids=lambda x: "x".join(map(str, x)) if isinstance(x, tuple) else str(x))
def test_from_mask_matches_oracle(shape, p, cuda):
    data_cpu = generate_input(*shape, seed=91, dropout_p=p)
    data = _to(data_cpu, cuda)
    dS, dV = ab.attn_bwd_from_mask((data[0], data[1], None, data[3], data[4], p))
    rS_dev, rV_dev = ab.custom_kernel(data)
    torch.cuda.synchronize()
    assert ab.poll_error() == 0
    rS, rV = attn_bwd_reference(data_cpu)
    assert torch.equal(dS, rS_dev)      # the dS kernel is the same one
    assert torch.allclose(rS.float(), dS.float().cpu(), rtol=1e-2, atol=1e-2)
    assert torch.allclose(rV.float(), dV.float().cpu(), rtol=1e-2, atol=1e-2)
    assert torch.allclose(rV_dev.float(), dV.float(), rtol=1e-2, atol=1e-2)


def test_from_mask_shard_matches_full(cuda):
    bs, sq, skv = 2, 96, 256
    data = _to(generate_input(bs, sq, skv, seed=92), cuda)
    dS, dV = ab.attn_bwd_from_mask((data[0], data[1], None, data[3], data[4], 0.1))
    sl = lambda t: t.reshape(bs * 80, sq, skv)[30:110]
    sS, sV = ab.attn_bwd_from_mask((data[0], sl(data[1]), None, data[3], sl(data[4]), 0.1), 3, 11)
    assert torch.equal(sS, dS.reshape(bs * 80, sq, skv)[30:110])
    assert torch.equal(sV, dV.reshape(bs * 8, skv, 128)[3:11])


def test_from_mask_ragged_rows_unsupported(cuda):
    data = _to(generate_input(1, 16, 100, seed=93), cuda)
    with pytest.raises(ab.AttnBwdError) as e:
        ab.attn_bwd_from_mask((data[0], data[1], None, data[3], data[4], 0.1))
    assert e.value.code == 3
