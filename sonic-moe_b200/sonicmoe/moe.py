"""``MoE`` module with the reference's constructor, parameters and forward signature
(reference ``sonicmoe/moe.py:57-276``), running the FP8 B200 engine.

Parameters keep the reference names and shapes (``router.weight`` [E, H], ``c_fc.weight``
[E, 2I, H] interleaved gate/up rows, ``c_proj.weight`` [E, H, I]), so reference state dicts load
unchanged.  ``forward(..., kernel_backend_moe=KernelBackendMoE.sonicmoe)`` is the only backend:
this package has no eager-torch or scattermoe execution path, and asking for one raises.
"""
import torch
import torch.nn as nn
import torch.nn.functional as F

from .enums import ActivationType, KernelBackendMoE, is_glu
from .functional import moe_TC_softmax_topk_layer


class Experts(nn.Module):
    def __init__(
        self, num_experts: int, in_features: int, out_features: int, add_bias: bool = True, std: float | None = None
    ) -> None:
        super().__init__()
        self.weight = nn.Parameter(torch.empty(num_experts, out_features, in_features))
        self.bias = nn.Parameter(torch.empty(num_experts, out_features)) if add_bias else None
        self.std = std
        self.num_experts = num_experts
        self.in_features = in_features
        self.out_features = out_features
        self.reset_parameters()

    def extra_repr(self):
        return "num_experts={}, in_features={}, out_features={}".format(
            self.num_experts, self.in_features, self.out_features
        )

    @torch.no_grad()
    def reset_parameters(self) -> None:
        nn.init.normal_(self.weight, mean=0, std=self.std)
        if self.bias is not None:
            self.bias.zero_()


class MoE(nn.Module):
    def __init__(
        self,
        num_experts: int,
        num_experts_per_tok: int,
        hidden_size: int,
        intermediate_size: int,
        activation_function: ActivationType,
        add_bias: bool,
        std: float,
    ) -> None:
        super().__init__()
        self.num_experts = num_experts
        self.top_k = num_experts_per_tok
        self.hidden_size = hidden_size
        self.intermediate_size = intermediate_size
        self.router = nn.Linear(in_features=self.hidden_size, out_features=num_experts, bias=False)
        self.activation_function = activation_function
        self.c_fc = Experts(
            num_experts=num_experts,
            in_features=self.hidden_size,
            out_features=2 * self.intermediate_size if is_glu(activation_function) else self.intermediate_size,
            add_bias=add_bias,
            std=std,
        )
        self.c_proj = Experts(
            num_experts=num_experts,
            in_features=self.intermediate_size,
            out_features=self.hidden_size,
            add_bias=add_bias,
            std=std,
        )
        # the reference records the current stream id here (moe.py:205); the engine uses the
        # current torch stream at call time, so nothing is queried at construction
        self.stream_id = None

    def forward(
        self,
        hidden_states: torch.Tensor,
        kernel_backend_moe: KernelBackendMoE = KernelBackendMoE.sonicmoe,
        is_inference_mode: bool = False,
    ) -> tuple[torch.Tensor, torch.Tensor]:
        if kernel_backend_moe != KernelBackendMoE.sonicmoe:
            raise NotImplementedError(
                f"backend {kernel_backend_moe} is not provided by the B200 engine; use KernelBackendMoE.sonicmoe"
            )
        original_shape = hidden_states.shape
        hidden_states = hidden_states.view(-1, self.hidden_size)
        hidden_states, router_logits, expert_frequency = moe_TC_softmax_topk_layer(
            hidden_states,
            self.router.weight,
            self.c_fc.weight.permute(1, 2, 0),
            self.c_fc.bias,
            self.c_proj.weight.permute(1, 2, 0),
            self.c_proj.bias,
            self.top_k,
            self.stream_id,
            self.activation_function,
            is_inference_mode or not self.training,
        )
        hidden_states = hidden_states.view(original_shape)
        if is_inference_mode:
            aux_loss = None
        else:
            aux_loss = self._compute_switch_loss(
                logits=router_logits,
                probs=F.softmax(router_logits, dim=-1, dtype=torch.float32),
                expert_frequency=expert_frequency,
            )
        return hidden_states, aux_loss

    def _compute_switch_loss(self, logits, probs, expert_frequency):
        """Switch load-balancing loss (reference moe.py:263-276), plain torch on the device."""
        logits = logits.view(-1, logits.size(-1))
        probs = probs.view(-1, probs.size(-1))
        num_experts = logits.size(1)
        acc_probs = probs.sum(0)
        expert_frequency = expert_frequency.float()
        return num_experts * (F.normalize(acc_probs, p=1, dim=0) * F.normalize(expert_frequency, p=1, dim=0)).sum()
