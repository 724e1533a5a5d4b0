"""Generate the golden vectors in this folder by running the reference's own code on CPU.

Run in a checkout that has the reference importable (the reference is pure Python; its eager
torch path runs on CPU once ``torch.cuda.current_stream`` is shimmed, because
``sonicmoe/moe.py:205`` queries it unconditionally)::

    python tests/golden/make_golden.py --reference /path/to/sonic-moe

What is produced (all small, compressed .npz):

* ``routing_ref.npz``  -- the reference torch router (``sonicmoe/functional/forward.py:128-141``,
  called through ``_topk_softmax_fwd``'s fallback branch) on tie-free bf16 logits, for
  softmax-over-top-k, top-k-over-softmax and top-k-over-softmax with renormalisation.
* ``metadata_ref.npz`` -- ``_ref_TC_topk_router_metadata`` / ``_ref_general_routing_metadata``
  (``tests/metadata_test.py:17-70``) on the reference test's own input generators
  (``_make_topk_indices`` / ``_make_general_routing_inputs``, seed 0) for the small shapes of its
  test matrix and its edge cases (all tokens on the same experts, a single token, empty experts).
* ``layer_ref.npz``    -- ``MoE.forward(kernel_backend_moe=KernelBackendMoE.torch,
  is_inference_mode=True)`` (``sonicmoe/moe.py:207-360``) on a small SwiGLU layer, and the
  per-expert loop of ``benchmarks/moe-cute.py:204-244`` (its ``swiglu(h, concat_layout)``) for the
  concatenated w1 layout with top-k-over-softmax + renormalisation.
* ``c1_ref.npz``       -- the config-1 layer (T=256, H=512, I=256, E=8, K=2, seed 1111) through
  ``MoE.forward(torch)``: a few output rows and whole-output checksums; the test regenerates the
  inputs from the same seeded ``torch.Generator``.
"""
import argparse
import os
import sys
import types

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def _import_reference(path):
    sys.path.insert(0, path)
    torch.cuda.current_stream = lambda *a, **k: types.SimpleNamespace(cuda_stream=0)
    # tests/metadata_test.py imports `parameterized` at module level; it is only a decorator source.
    if "parameterized" not in sys.modules:
        fake = types.ModuleType("parameterized")

        class _P:
            @staticmethod
            def expand(*a, **k):
                return lambda f: f

        fake.parameterized = _P
        sys.modules["parameterized"] = fake
    import sonicmoe  # noqa: F401
    from sonicmoe import KernelBackendMoE, MoE
    from sonicmoe.enums import ActivationType
    from sonicmoe.functional import forward as ref_forward
    import tests.metadata_test as ref_meta  # noqa: E402

    return MoE, KernelBackendMoE, ActivationType, ref_forward, ref_meta


def _bf16_bits(t: torch.Tensor) -> np.ndarray:
    return t.to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)


def make_routing(ref_forward):
    out = {}
    g = torch.Generator().manual_seed(1234)
    cases = [(256, 128, 8), (64, 96, 7), (32, 64, 4)]
    for T, E, K in cases:
        # tie-free logits on a 1/32 grid (exact in bf16); gaps >> the 7 truncated mantissa bits
        base = torch.stack([torch.randperm(E, generator=g) for _ in range(T)]).float()
        logits = ((base - E // 2) / 32.0).to(torch.bfloat16)
        out[f"logits_{T}_{E}_{K}"] = _bf16_bits(logits)
        for name, sot, norm in (("sot", True, False), ("tos", False, False), ("tosn", False, True)):
            scores = torch.empty(T, K, dtype=torch.float32)
            idx = torch.empty(T, K, dtype=torch.int32)
            # The reference op itself.  Its E argument only selects the branch
            # (forward.py:119); E=4097 takes the torch branch (forward.py:128-141), which runs on
            # CPU and reads the real width from the logits tensor.
            ref_forward._topk_softmax_fwd(
                logits, scores, idx, 4097, K, is_softmax_over_topk=sot, norm_topk_probs=norm
            )
            out[f"scores_{name}_{T}_{E}_{K}"] = scores.numpy()
            out[f"idx_{name}_{T}_{E}_{K}"] = idx.numpy()
    np.savez_compressed(os.path.join(HERE, "routing_ref.npz"), **out)


def make_metadata(ref_meta):
    out = {}
    dev = torch.device("cpu")
    shapes = [(10, 8, 2), (236, 16, 4), (1024, 128, 8), (1000, 96, 7), (50, 384, 3), (2048, 512, 10)]
    for T, E, K in shapes:
        ref_meta.TestCommons.set_seed(0)
        idx = ref_meta._make_topk_indices(T, E, K, dev)
        res = ref_meta._ref_TC_topk_router_metadata(idx, E)
        key = f"tc_{T}_{E}_{K}"
        out[key + "_idx"] = idx.numpy()
        for n, v in zip(("freq", "off", "gather", "scatter", "rev"), res):
            out[key + "_" + n] = v.numpy()
    # edge cases of tests/metadata_test.py:201-263
    same = torch.zeros(64, 2, dtype=torch.int32)
    same[:, 1] = 1
    single = torch.tensor([[3, 5]], dtype=torch.int32)
    for name, idx, E in (("same", same, 8), ("single", single, 8)):
        res = ref_meta._ref_TC_topk_router_metadata(idx, E)
        out[f"edge_{name}_idx"] = idx.numpy()
        for n, v in zip(("freq", "off", "gather", "scatter", "rev"), res):
            out[f"edge_{name}_{n}"] = v.numpy()
    for T, E, avg_k in [(10, 8, 2), (236, 16, 4), (1000, 96, 7), (50, 384, 3)]:
        ref_meta.TestCommons.set_seed(0)
        tok, exp_ = ref_meta._make_general_routing_inputs(T, E, avg_k, dev)
        res = ref_meta._ref_general_routing_metadata(tok, exp_, T, E)
        key = f"gen_{T}_{E}_{avg_k}"
        out[key + "_tok"] = tok.numpy()
        out[key + "_exp"] = exp_.numpy()
        for n, v in zip(("freq", "off", "gather", "scatter", "rev", "tokoff"), res):
            out[key + "_" + n] = v.numpy()
    # empty experts (tests/metadata_test.py:474-516)
    ref_meta.TestCommons.set_seed(0)
    idx = ref_meta._make_topk_indices(32, 64, 2, dev)
    res = ref_meta._ref_TC_topk_router_metadata(idx, 64)
    out["edge_empty_idx"] = idx.numpy()
    for n, v in zip(("freq", "off", "gather", "scatter", "rev"), res):
        out["edge_empty_" + n] = v.numpy()
    np.savez_compressed(os.path.join(HERE, "metadata_ref.npz"), **out)


def make_layer(MoE, KernelBackendMoE, ActivationType, ref_path):
    out = {}
    T, H, I, E, K = 32, 128, 128, 4, 2
    torch.manual_seed(42)
    moe = MoE(E, K, H, I, ActivationType.SWIGLU, False, 0.02)
    # bf16-representable fp32 values, so the fixture stores them as bf16 bits
    with torch.no_grad():
        for p in moe.parameters():
            p.copy_(p.to(torch.bfloat16).float())
    x = torch.randn(T, H).to(torch.bfloat16).float()
    with torch.no_grad():
        o, aux = moe(x, kernel_backend_moe=KernelBackendMoE.torch, is_inference_mode=True)
    out["x"] = _bf16_bits(x)
    out["router_w"] = _bf16_bits(moe.router.weight.detach())
    out["w1"] = _bf16_bits(moe.c_fc.weight.detach())
    out["w2"] = _bf16_bits(moe.c_proj.weight.detach())
    out["o"] = o.numpy()
    out["shape"] = np.array([T, H, I, E, K])

    # per-expert loop of benchmarks/moe-cute.py:204-244 with its own swiglu, concat layout,
    # top-k over softmax with renormalisation
    sys.path.insert(0, os.path.join(ref_path, "benchmarks"))
    import importlib

    try:
        bench = importlib.import_module("moe-cute")
        swiglu = bench.swiglu
    except Exception:  # the benchmark imports cutlass/triton at module level
        swiglu = None
    if swiglu is not None:
        w1 = moe.c_fc.weight.detach()
        w2 = moe.c_proj.weight.detach()
        logits = torch.nn.functional.linear(x, moe.router.weight.detach())
        probs = logits.softmax(dim=-1, dtype=torch.float32)
        scores, experts = probs.topk(K, dim=-1)
        scores = scores / scores.sum(dim=-1, keepdim=True)
        ref_o = torch.zeros_like(x)
        for i in range(E):
            T_idx, E_idx = torch.argwhere(experts == i).split(1, dim=1)
            T_idx, E_idx = T_idx.squeeze(-1), E_idx.squeeze(-1)
            if T_idx.numel() > 0:
                w1_out = torch.nn.functional.linear(x[T_idx, :], w1[i])
                w1_out = swiglu(w1_out, concat_layout=True)
                w2_out = torch.nn.functional.linear(w1_out, w2[i])
                ref_o[T_idx, :] += w2_out * scores[T_idx, E_idx, None]
        out["concat_tosn_o"] = ref_o.numpy()
        out["concat_tosn_scores"] = scores.numpy()
        out["concat_tosn_idx"] = experts.to(torch.int32).numpy()
    np.savez_compressed(os.path.join(HERE, "layer_ref.npz"), **out)


def make_c1(MoE, KernelBackendMoE, ActivationType):
    T, H, I, E, K = 256, 512, 256, 8, 2
    g = torch.Generator().manual_seed(1111)
    router_w = torch.randn(E, H, generator=g) * 0.02
    w1 = torch.randn(E, 2 * I, H, generator=g) * 0.02
    w2 = torch.randn(E, H, I, generator=g) * 0.02
    x = torch.randn(T, H, generator=g)
    moe = MoE(E, K, H, I, ActivationType.SWIGLU, False, 0.02)
    with torch.no_grad():
        moe.router.weight.copy_(router_w)
        moe.c_fc.weight.copy_(w1)
        moe.c_proj.weight.copy_(w2)
        o, _ = moe(x, kernel_backend_moe=KernelBackendMoE.torch, is_inference_mode=True)
    o64 = o.double()
    np.savez_compressed(
        os.path.join(HERE, "c1_ref.npz"),
        rows=o[:8].numpy(),
        sum=np.array(o64.sum().item()),
        abssum=np.array(o64.abs().sum().item()),
        sumsq=np.array((o64 * o64).sum().item()),
        input_sum=np.array(x.double().sum().item() + w1.double().sum().item()),
    )


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("SONICMOE_REFERENCE"),
                    help="checkout of the reference sonic-moe (or set SONICMOE_REFERENCE)")
    args = ap.parse_args()
    if not args.reference:
        ap.error("give the reference checkout with --reference or SONICMOE_REFERENCE")
    os.chdir(args.reference)  # so that `tests.metadata_test` resolves to the reference's tests
    MoE, KernelBackendMoE, ActivationType, ref_forward, ref_meta = _import_reference(args.reference)
    torch.set_num_threads(min(8, os.cpu_count() or 1))
    make_routing(ref_forward)
    make_metadata(ref_meta)
    make_layer(MoE, KernelBackendMoE, ActivationType, args.reference)
    make_c1(MoE, KernelBackendMoE, ActivationType)
    print("golden vectors written to", HERE)


if __name__ == "__main__":
    main()
