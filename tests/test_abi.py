"""The C-ABI library: builds, loads without a GPU, exports every declared symbol,
and rejects bad arguments before touching the device."""
import ctypes
import os
import re

import pytest

from attn_bwd_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADERS = [os.path.join(ROOT, "include", f) for f in os.listdir(os.path.join(ROOT, "include")) if f.endswith(".h")]


def declared_functions():
    names = set()
    for h in HEADERS:
        src = open(h).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        for m in re.finditer(r"^\s*(?:const\s+)?[A-Za-z_][\w\s\*]*?\b(attn_bwd_b200\w*)\s*\(", src, flags=re.M):
            names.add(m.group(1))
    return names


def test_library_built_in_tree():
    assert os.path.exists(_lib.LIB_PATH), "run __graft_entry__.build() first"


def test_exports_every_declared_symbol():
    lib = _lib.load()
    names = declared_functions()
    assert {"attn_bwd_b200", "attn_bwd_b200_shard", "attn_bwd_b200_poll_error"} <= names
    for n in names:
        assert hasattr(lib, n), f"{n} declared in include/ but not exported"
        assert n in _lib.SIGNATURES, f"{n} has no ctypes signature"


def test_strerror_and_version():
    lib = _lib.load()
    assert lib.attn_bwd_b200_version() >= 100
    for code in range(8):
        assert len(_lib.strerror(code)) > 0
    assert _lib.strerror(99) == "unknown error"


@pytest.mark.parametrize("bs,sq,skv", [(-1, 4, 4), (1, -4, 4), (1, 4, -4)])
def test_negative_sizes_rejected_without_device(bs, sq, skv):
    lib = _lib.load()
    nul = ctypes.c_void_p(0)
    rc = lib.attn_bwd_b200(nul, nul, nul, nul, nul, 0.1, bs, sq, skv, nul, nul, nul)
    assert rc == _lib.EINVAL


def test_bad_unit_range_rejected_without_device():
    lib = _lib.load()
    nul = ctypes.c_void_p(0)
    rc = lib.attn_bwd_b200_shard(nul, nul, nul, nul, nul, 0.1, 2, 4, 16, 3, 17, nul, nul, nul)
    assert rc == _lib.EINVAL
    rc = lib.attn_bwd_b200_dv_shard(nul, nul, 2, 4, 16, 5, 4, nul, nul)
    assert rc == _lib.EINVAL


def test_torch_binding_loads_and_declines_cpu_tensors():
    """The C++ host binding is built in-tree, links the same library, and hands inputs
    it cannot take (here: CPU tensors) back to the general path instead of computing."""
    import torch
    import attn_bwd_b200 as ab
    assert ab._torch_fast_fn is not None
    dO = torch.zeros(1, 4, 80, 128, dtype=torch.bfloat16)
    P = torch.zeros(1, 80, 4, 8, dtype=torch.bfloat16)
    V = torch.zeros(1, 8, 8, 128, dtype=torch.bfloat16)
    M = torch.zeros(1, 80, 4, 8, dtype=torch.bool)
    assert ab._torch_fast_fn(dO, P, P, V, M, 0.1) is None


def test_host_call_argument_errors_without_gpu():
    import torch
    import attn_bwd_b200 as ab
    from attn_bwd_b200.generate import generate_input
    data = generate_input(1, 4, 16, seed=1, device="cpu")
    bad = (data[0].float(),) + tuple(data[1:])
    with pytest.raises(ValueError):
        ab.attn_bwd_host(bad)
    with pytest.raises(ValueError):
        ab.attn_bwd_host(data, 0, 9)
    with pytest.raises(TypeError):
        ab.attn_bwd_host((None,) + tuple(data[1:]))


def test_options_set_get_restore_without_gpu():
    """The measurement / test options are plain host state: settable without a device,
    restored by the context manager, unknown names and indices rejected."""
    import attn_bwd_b200 as ab
    lib = _lib.load()
    assert _lib.get_option("ds_mode") == -1
    with ab.options(ds_mode=0, graph=0):
        assert _lib.get_option("ds_mode") == 0 and _lib.get_option("graph") == 0
    assert _lib.get_option("ds_mode") == -1 and _lib.get_option("graph") == -1
    with pytest.raises(ValueError):
        ab.options(no_such_option=1)
    assert lib.attn_bwd_b200_set_option(99, 1) == _lib.EINVAL
    assert lib.attn_bwd_b200_get_option(99) == -2


def test_from_mask_rejects_bad_dropout_without_device():
    lib = _lib.load()
    nul = ctypes.c_void_p(0)
    for p in (-0.1, 1.0, float("nan")):
        rc = lib.attn_bwd_b200_shard_from_mask(nul, nul, nul, nul, p, 1, 4, 16, 0, 8, nul, nul, nul)
        assert rc == _lib.EINVAL
