"""ctypes binding of the C-ABI in include/attn_bwd_b200.h.

The shared library is built in-tree (``__graft_entry__.build()``) next to this
file.  There is no fallback: if the library is missing, every entry point
raises.
"""
import ctypes
import os

LIB_NAME = "libattn_bwd_b200.so"
# ATTN_BWD_B200_LIB may point at another build of the same library (e.g. a tuning variant).
LIB_PATH = os.environ.get("ATTN_BWD_B200_LIB") or os.path.join(os.path.dirname(os.path.abspath(__file__)), LIB_NAME)

# C-ABI error codes (enum in include/attn_bwd_b200.h)
OK, EINVAL, EALIGN, EUNSUPPORTED, ETMAP, ECUDA, EDEVICE, EKERNEL = range(8)

# Every symbol the header declares, with its ctypes signature.
_VP, _I, _F = ctypes.c_void_p, ctypes.c_int, ctypes.c_float
SIGNATURES = {
    "attn_bwd_b200": (_I, [_VP, _VP, _VP, _VP, _VP, _F, _I, _I, _I, _VP, _VP, _VP]),
    "attn_bwd_b200_shard": (_I, [_VP, _VP, _VP, _VP, _VP, _F, _I, _I, _I, _I, _I, _VP, _VP, _VP]),
    "attn_bwd_b200_ds_shard": (_I, [_VP, _VP, _VP, _VP, _F, _I, _I, _I, _I, _I, _VP, _VP]),
    "attn_bwd_b200_dv_shard": (_I, [_VP, _VP, _I, _I, _I, _I, _I, _VP, _VP]),
    "attn_bwd_b200_shard_from_mask": (_I, [_VP, _VP, _VP, _VP, _F, _I, _I, _I, _I, _I, _VP, _VP, _VP]),
    "attn_bwd_b200_host_shard": (_I, [_VP] * 5 + [_F, _I, _I, _I, _I, _I] + [_VP] * 9 + [_I, _VP]),
    "attn_bwd_b200_host": (_I, [_VP] * 5 + [_F, _I, _I, _I] + [_VP] * 9 + [_I, _VP]),
    "attn_bwd_b200_poll_error": (_I, []),
    "attn_bwd_b200_selftest_wait_timeout": (_I, [_I, _VP]),
    "attn_bwd_b200_strerror": (ctypes.c_char_p, [_I]),
    "attn_bwd_b200_version": (_I, []),
    "attn_bwd_b200_release": (_I, []),
    "attn_bwd_b200_set_option": (_I, [_I, _I]),
    "attn_bwd_b200_get_option": (_I, [_I]),
}

# Measurement / test options (ATTN_BWD_OPT_* in include/attn_bwd_b200.h); -1 = automatic.
OPTIONS = {"ds_mode": 0, "row_kind": 1, "ds_cluster": 2, "l2_prefetch": 3, "l2_hint": 4, "split": 5,
           "dv_sms": 6, "side_stream": 7, "graph": 8, "map_cache": 9}

_lib = None


class AttnBwdError(RuntimeError):
    """A C-ABI call returned a non-zero ATTN_BWD_E* code."""

    def __init__(self, fn, code):
        self.code = code
        super().__init__(f"{fn} failed: {code} ({strerror(code)})")


def load():
    """Load the in-tree library (once).  Raises if it has not been built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"attn_bwd_b200 CUDA library not built: {LIB_PATH} is missing "
                "(run __graft_entry__.build()); there is no CPU fallback")
        lib = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            f = getattr(lib, name)
            f.restype = res
            f.argtypes = args
        _lib = lib
    return _lib


def fast_fn():
    """The bound attn_bwd_b200 entry point (loads the library on first use)."""
    return load().attn_bwd_b200


def strerror(code):
    return load().attn_bwd_b200_strerror(int(code)).decode()


def set_option(name, value):
    """Sets one measurement / test option (process-wide; -1 restores the automatic choice)."""
    call("attn_bwd_b200_set_option", OPTIONS[name], int(value))


def get_option(name):
    return load().attn_bwd_b200_get_option(OPTIONS[name])


def call(name, *args):
    rc = getattr(load(), name)(*args)
    if rc != OK:
        raise AttnBwdError(name, rc)
