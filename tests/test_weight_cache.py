"""CPU: the functional layer's prepared-weight cache follows the weight tensor, not its address.

`weight_prep` is replaced by a counting stub, so no GPU is needed.  A new weight tensor of the
same shape (possibly allocated where a freed one lived) must be quantised again; an unchanged
tensor must not; an in-place update must.
"""
import gc

import torch


def _with_counting_prep(monkeypatch):
    from sonicmoe import functional as fn

    calls = []

    def fake_prep(w, concat_glu=False, with_t=False):
        calls.append((w.data_ptr(), concat_glu))
        return ("prepared", len(calls))

    monkeypatch.setattr(fn.ops, "weight_prep", fake_prep)
    return fn, calls


def test_same_tensor_hits_and_inplace_update_misses(monkeypatch):
    fn, calls = _with_counting_prep(monkeypatch)
    w = torch.randn(4, 256, 128)
    a = fn.prepare_fp8_weights(w.permute(1, 2, 0))
    b = fn.prepare_fp8_weights(w.permute(1, 2, 0))  # a new view object of the same weight
    assert a is b and len(calls) == 1
    fn.prepare_fp8_weights(w.permute(1, 2, 0), concat_glu=True)  # other layout: own entry
    assert len(calls) == 2
    w.add_(1.0)  # in-place update bumps the version counter
    fn.prepare_fp8_weights(w.permute(1, 2, 0))
    assert len(calls) == 3


def test_new_tensor_is_never_served_a_freed_tensors_entry(monkeypatch):
    fn, calls = _with_counting_prep(monkeypatch)
    for i in range(6):
        w = torch.randn(4, 256, 128)  # same shape every time; the allocator may reuse the address
        fn.prepare_fp8_weights(w.permute(1, 2, 0))
        del w
        gc.collect()
    assert len(calls) == 6
    assert len(fn._WEIGHT_CACHE) == 0  # entries died with their tensors
