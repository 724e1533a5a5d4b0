"""GPU test of sm_route_metadata_noalloc, the routing-metadata entry point that allocates nothing.

It serves callers that cannot allocate device memory when they route tokens (a host recording the
step into a CUDA graph, where cudaMalloc is not allowed during capture, or a runtime that reserved
all device memory up front).  Its scratch is a 1 MiB static device array shared by every call.

The test calls it through the C ABI twice in a row and checks that both calls give exactly the
outputs of the existing workspace-based entry point, sm_route_metadata, and of the CPU oracle's
restatement of the reference metadata (oracle.metadata.tc_metadata; integer arrays: exact equality
is the tolerance).  The two calls use different routings, so a stale leftover in the
shared array from the first call would show up in the second.  This file sorts last so that a run
stopping at the first failure has already run every other test; it also passes alone.
"""
import ctypes

import numpy as np
import pytest
import torch

from oracle.metadata import tc_metadata

pytestmark = pytest.mark.gpu


def _indices(T, E, K, seed):
    rs = np.random.RandomState(seed)
    return torch.from_numpy(np.stack([np.sort(rs.permutation(E)[:K]) for _ in range(T)]).astype(np.int32))


def _outputs(T, K, E, dev):
    TK = T * K
    return [torch.full((E,), -7, dtype=torch.int32, device=dev), torch.full((E + 1,), -7, dtype=torch.int32, device=dev)] + [
        torch.full((TK,), -7, dtype=torch.int32, device=dev) for _ in range(3)
    ]


def _run_noalloc(lib, idx, T, K, E, dev):
    freq, off, xg, ss, sr = _outputs(T, K, E, dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    rc = lib.sm_route_metadata_noalloc(
        idx.data_ptr(), T, K, E, freq.data_ptr(), off.data_ptr(), xg.data_ptr(), ss.data_ptr(), sr.data_ptr(),
        err.data_ptr(), torch.cuda.current_stream().cuda_stream,
    )
    assert rc == 0, lib.sm_last_error().decode()
    return (freq, off, xg, ss, sr), err


def _run_workspace(lib, idx, T, K, E, dev):
    freq, off, xg, ss, sr = _outputs(T, K, E, dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    ws_bytes = lib.sm_route_metadata_workspace(T, T * K, E)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    rc = lib.sm_route_metadata(
        idx.data_ptr(), T, K, E, freq.data_ptr(), off.data_ptr(), xg.data_ptr(), ss.data_ptr(), sr.data_ptr(),
        ws.data_ptr(), ctypes.c_size_t(ws_bytes), err.data_ptr(), torch.cuda.current_stream().cuda_stream,
    )
    assert rc == 0, lib.sm_last_error().decode()
    return (freq, off, xg, ss, sr), err


def test_noalloc_metadata_matches_workspace_entry_point_twice():
    assert torch.cuda.is_available(), "GPU test needs a CUDA device"
    from sonicmoe import _native

    lib = _native.load()
    dev = torch.device("cuda", 0)
    # call 1: config-2 routing shape; call 2: a different shape and routing reusing the array
    for T, E, K, seed in ((32768, 128, 8, 1), (1000, 96, 7, 2)):
        idx = _indices(T, E, K, seed).to(dev)
        got, err_a = _run_noalloc(lib, idx, T, K, E, dev)
        want, err_b = _run_workspace(lib, idx, T, K, E, dev)
        torch.cuda.synchronize()
        assert err_a.item() == 0 and err_b.item() == 0
        for name, a, b in zip(("freq", "offset", "x_gather", "s_scatter", "s_reverse"), got, want):
            assert torch.equal(a, b), f"T={T} E={E} K={K}: {name} differs from sm_route_metadata"
        ref = tc_metadata(idx.cpu().numpy(), E)
        for name, a, r in zip(("freq", "offset", "x_gather", "s_scatter", "s_reverse"), got, ref):
            np.testing.assert_array_equal(a.cpu().numpy(), r, err_msg=f"T={T} E={E} K={K}: {name} vs oracle")


def test_noalloc_rejects_sizes_beyond_its_static_scratch():
    from sonicmoe import _native

    lib = _native.load()
    dev = torch.device("cuda", 0)
    small = torch.zeros(4097, dtype=torch.int32, device=dev)
    # E * ceil(T/128) tile counts alone exceed the 1 MiB array; rejected before any launch
    rc = lib.sm_route_metadata_noalloc(
        small.data_ptr(), 1 << 20, 8, 4096, small.data_ptr(), small.data_ptr(), None, None, None, small.data_ptr(),
        torch.cuda.current_stream().cuda_stream,
    )
    assert rc == _native.SM_EINVAL
    assert "scratch" in lib.sm_last_error().decode()
