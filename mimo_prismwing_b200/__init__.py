"""B200 (sm_100a) block-FP8 routed-MoE path of Prismwing, behind include/pw_cuda.h.

    from mimo_prismwing_b200.runtime import WideMoeRuntime
"""
from ._lib import LIB_PATH, load  # noqa: F401

__all__ = ["LIB_PATH", "load"]
