"""B200-native (sm_100a) optimizer step for the adv_optm optimizers.

Drop-in classes with the constructor arguments, param-group keys and state
layout of adv_optm 2.5.4; the step runs in hand-written CUDA kernels through
the C ABI in include/advopt.h (libadvopt.so, built in-tree).
"""
from .optim import *  # noqa: F401,F403
from .optim import __all__ as _optim_all
from .distributed import ShardedOptimizer

__version__ = "0.1.0"
reference_version = "2.5.4"
__all__ = list(_optim_all) + ["ShardedOptimizer"]
