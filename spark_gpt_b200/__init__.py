"""B200-native (sm_100a) Qwen3-MoE expert layer for the spark-gpt trainer.

Drop-in replacements for train.py's MoE path:

* ``SparseMoE``, ``TopKRouter``, ``Experts``  (train.py:2134-2334)
* ``global_load_balancing_loss``               (train.py:3098-3197)

All compute runs in ``libb200moe.so`` (C ABI in ``include/b200moe.h``),
built with ``python -m spark_gpt_b200.build``.
"""

from .aux_loss import global_load_balancing_loss
from .faults import DeviceFault, check_faults
from .fp8 import fp8_update_scales
from .moe import Experts, SparseMoE, TopKRouter

__all__ = ["SparseMoE", "TopKRouter", "Experts", "global_load_balancing_loss", "DeviceFault",
           "check_faults", "fp8_update_scales"]
