"""B200-native heterogeneous multi-LoRA linear (drop-in for the reference's
``tlora`` package).

    from tlora_b200 import MultiLoRALinear
    m = MultiLoRALinear(4096, 4096, {0: 8, 1: 64}).cuda().bfloat16()
    y = m(x, adapter_ids)          # fused tcgen05 forward
    y.backward(dy)                 # analytic backward: dX, dA, dB (no dW)
    m.sgd_step(1e-3, [0])          # isolated per-adapter SGD
"""

from .multi_lora_linear import IndependentLoRALinear, LoRAAdapter, MultiLoRALinear
from . import ops
from ._lib import lib as native_library, launch_count

__all__ = [
    "LoRAAdapter",
    "IndependentLoRALinear",
    "MultiLoRALinear",
    "ops",
    "native_library",
    "launch_count",
]
