"""The single-file submission (make_submission.py) loaded the way the reference evaluator
loads a submission: its TEXT written to a fresh temporary ``submission.py`` and imported
with importlib (eval_modal_attn_bwd.py:238-247), then called like its correctness loop
does (eval_modal_attn_bwd.py:266-302: generate on the GPU, keep a clone, call under
no_grad, synchronise, compare with the fp32 reference at rtol = atol = 1e-2)."""
import importlib.util
import os
import tempfile

import pytest
import torch

import make_submission

SOL_CASES = [(4, 256, 256, 1001), (8, 373, 449, 1002), (4, 211, 293, 1009)]   # eval_modal_attn_bwd.py:18-35


def _load_from_text(tmp):
    path = os.path.join(tmp, "submission.py")
    with open(path, "w") as f:
        f.write(make_submission.build_text())
    os.environ["ATTN_BWD_B200_CACHE"] = os.path.join(tmp, "cache")
    try:
        spec = importlib.util.spec_from_file_location("submission", path)
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
    finally:
        del os.environ["ATTN_BWD_B200_CACHE"]
    return mod


def test_text_builds_and_loads_without_gpu():
    """Nothing but the text is needed: it compiles its embedded sources and binds the C-ABI;
    CPU tensors are refused (no CPU path)."""
    with tempfile.TemporaryDirectory() as tmp:
        mod = _load_from_text(tmp)
        assert mod._lib.attn_bwd_b200_version() >= 100
        assert os.path.exists(os.path.join(tmp, "cache", mod._DIGEST, "libattn_bwd_b200.so"))
        with pytest.raises(ValueError, match="CUDA"):
            mod.custom_kernel((torch.zeros(1, 4, 80, 128, dtype=torch.bfloat16),) * 5 + (0.1,))


@pytest.mark.gpu
def test_evaluator_style_load_and_check(cuda):
    from attn_bwd_b200.generate import generate_input
    from oracle.attn_bwd_oracle import _attn_bwd_group
    torch.backends.cuda.matmul.allow_tf32 = False
    with tempfile.TemporaryDirectory() as tmp:
        mod = _load_from_text(tmp)
        for bs, sq, skv, seed in SOL_CASES:
            data = generate_input(bs, sq, skv, seed, device="cuda")
            data_copy = tuple(t.clone() if isinstance(t, torch.Tensor) else t for t in data)
            torch.cuda.synchronize()
            with torch.no_grad():
                dS, dV = mod.custom_kernel(data)
            torch.cuda.synchronize()
            dO, P, Pd, V, M, p = data_copy
            for u in range(bs * 8):
                b, kvh = divmod(u, 8)
                hs = slice(kvh * 10, kvh * 10 + 10)
                rS, rV = _attn_bwd_group((dO[b:b + 1, :, hs], P[b:b + 1, hs], Pd[b:b + 1, hs],
                                          V[b:b + 1, kvh:kvh + 1], M[b:b + 1, hs], p))
                assert torch.allclose(rS[0].float(), dS[b, hs].float(), rtol=1e-2, atol=1e-2), (bs, sq, skv, u)
                assert torch.allclose(rV[0, 0].float(), dV[b, kvh].float(), rtol=1e-2, atol=1e-2), (bs, sq, skv, u)
