"""sonicmoe on B200: the reference's MoE module and functional entry points, FP8 (e4m3) forward on
hand-written sm_100a kernels (libsonic_b200.so).  Drop-in import path: put ``sonic-moe_b200/`` on
``PYTHONPATH`` and ``from sonicmoe import MoE`` resolves here."""

__version__ = "0.1.0+b200"

from .enums import ActivationType, KernelBackendMoE
from .functional import moe_general_routing_inputs, moe_TC_softmax_topk_layer
from .moe import MoE
