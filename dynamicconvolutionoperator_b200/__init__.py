"""B200-native (sm_100a) DDPM: a drop-in for lartpang/DynamicConvolutionOperator's
``triton_impl.DDPM`` and ``_triton_kernels`` GPU path.

Public surface:
  * ``DDPM`` — the module (reference ``triton_impl.py:247-392``).
  * ``fused_dynamic_cat`` / ``fused_generator_dynamic_cat`` — the differentiable
    kernel-level ops (reference ``_triton_kernels.py:869``, ``:1056``).
  * ``data_parallel`` — batch-sharded training helpers over NCCL.
"""

from ._kernels import fused_dynamic_cat, fused_generator_dynamic_cat
from .ddpm import DDPM

__all__ = ["DDPM", "fused_dynamic_cat", "fused_generator_dynamic_cat"]
