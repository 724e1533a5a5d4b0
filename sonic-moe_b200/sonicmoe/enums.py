"""Enums of the reference API (reference sonicmoe/enums.py:8-32), unchanged names and values."""
from enum import Enum

LIBRARY_NAME = "sonicmoe"


class KernelBackendMoE(Enum):
    scattermoe = "scattermoe"
    torch = "torch"
    sonicmoe = "sonicmoe"


class ActivationType(Enum):
    SWIGLU = "swiglu"
    GEGLU = "geglu"
    REGLU = "reglu"

    RELU_SQ = "relu_sq"
    RELU = "relu"
    GELU = "gelu_tanh_approx"
    SILU = "silu"


def is_glu(activation_type: ActivationType):
    return activation_type in [ActivationType.SWIGLU, ActivationType.REGLU, ActivationType.GEGLU]
