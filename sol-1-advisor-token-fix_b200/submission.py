"""Drop-in ``submission.py`` for the reference harness.

The reference evaluator writes a submission's source to a temporary
``submission.py``, imports it and calls its module-level ``custom_kernel``
(eval_modal_attn_bwd.py:238-247, 273).  This file is such a submission: it
locates the in-tree ``attn_bwd_b200`` package (directory given by the
ATTN_BWD_B200_HOME environment variable, else this file's directory) and
re-exports its ``custom_kernel``, which runs the sm_100a kernels through the
C-ABI.  Nothing else from the reference is needed.
"""
import os
import sys

_home = os.environ.get("ATTN_BWD_B200_HOME", os.path.dirname(os.path.abspath(__file__)))
if _home not in sys.path:
    sys.path.insert(0, _home)

from attn_bwd_b200 import custom_kernel, run  # noqa: E402,F401
