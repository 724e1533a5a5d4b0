"""CPU tests of the op boundary: the registered custom ops exist under the reference's names, a
whole MoE forward traces as one graph through them (torch.export in strict mode runs dynamo with
fake tensors, so no kernel runs and no GPU is needed), and training mode is refused explicitly."""
import pytest
import torch


def test_ops_registered_under_reference_names():
    import sonicmoe  # noqa: F401  (registers the ops)

    for ns, name in [("sonicmoe", "_topk_fwd"), ("sonicmoe", "_softmax_topk_fwd"),
                     ("triton_kernels", "TC_topk_router_metadata"),
                     ("triton_kernels", "general_routing_router_metadata"),
                     ("sonicmoe", "fp8_moe_tc_forward"), ("sonicmoe", "fp8_moe_general_forward")]:
        assert hasattr(getattr(torch.ops, ns), name), f"{ns}::{name} not registered"


def test_moe_forward_exports_as_one_graph():
    import sonicmoe

    T, H, I, E, K = 64, 256, 128, 8, 2
    m = sonicmoe.MoE(E, K, H, I, sonicmoe.ActivationType.SWIGLU, False, 0.02).to(torch.bfloat16).eval()
    x = torch.randn(T, H, dtype=torch.bfloat16)
    with torch.no_grad():
        ep = torch.export.export(m, (x,), strict=True)
    targets = [str(n.target) for n in ep.graph.nodes if n.op == "call_function"]
    assert any("fp8_moe_tc_forward" in t for t in targets), targets
    out = [n for n in ep.graph.nodes if n.op == "output"][0]
    o_meta = out.args[0][0].meta["val"]
    assert tuple(o_meta.shape) == (T, H) and o_meta.dtype == torch.bfloat16


def test_training_without_a_backward_is_refused():
    """Gradient requests the FP8 backward does not cover raise before any device work: the fused
    router."""
    import sonicmoe
    from sonicmoe.functional import moe_TC_softmax_topk_layer

    T, H, I, E, K = 16, 256, 128, 4, 2
    m = sonicmoe.MoE(E, K, H, I, sonicmoe.ActivationType.SWIGLU, False, 0.02)
    x = torch.randn(T, H)
    w1, w2 = m.c_fc.weight.permute(1, 2, 0), m.c_proj.weight.permute(1, 2, 0)
    with pytest.raises(NotImplementedError, match="fused_router"):
        moe_TC_softmax_topk_layer(x, m.router.weight, w1, None, w2, None, K, None, is_inference_mode_enabled=False,
                                  fused_router=True)

