"""evie_gqa_decode_paged_noalloc, the allocation-free form of the paged GQA decode attention.

It exists for callers that cannot let a library allocate device memory (engines that reserve nearly all GPU memory
for their own allocator at start-up, latency-critical paths that cannot afford cudaMalloc's synchronisation): its
split scratch is a fixed array inside the library. These tests call it through the C ABI and hold it to the results
of the allocating entry point, on two calls in a row (the second sees the first call's leftover scratch). This file
sorts last so that a run stopping at the first failure has already run every other test."""
import ctypes as C

import numpy as np
import pytest
import torch

from tests._inputs import gqa_inputs

TOL = 2e-5  # the tolerance of the paged GQA parity tests


def _call(L, fn, x, out, scale, max_pages=None):
    B, Hq, hd = x["q"].shape
    _, Hkv, page, _ = x["kp"].shape
    mp = x["pt"].shape[1] if max_pages is None else max_pages
    return getattr(L, fn)(x["q"].data_ptr(), x["gate"].data_ptr(), x["kp"].data_ptr(), x["vp"].data_ptr(),
                          x["pt"].data_ptr(), x["ctx"].data_ptr(), out.data_ptr(), B, Hq, Hkv, hd, page, mp,
                          C.c_float(scale), torch.cuda.current_stream().cuda_stream)


@pytest.mark.gpu
@pytest.mark.parametrize("Hq,Hkv", [(16, 4), (8, 4)])
def test_noalloc_matches_allocating_entry_point(Hq, Hkv, cuda):
    """GQA group 4 (the bulk-copy kernel) and group 2 (the CUDA-core kernel, whose per-split partials scale with the
    group), each with contexts of several 512-token splits."""
    import evie_b200

    L = evie_b200.lib()
    scale = 1.0 / 16.0
    for call, (ctx, seed) in enumerate([([300, 5000, 1, 12000], 31), ([9000, 0, 700, 2047], 32)]):
        x = {k: v.to(cuda) for k, v in gqa_inputs(len(ctx), Hq, Hkv, ctx, seed).items()}
        ref = torch.empty(x["q"].shape, device=cuda, dtype=torch.float32)
        got = torch.full(x["q"].shape, float("nan"), device=cuda, dtype=torch.float32)
        assert _call(L, "evie_gqa_decode_paged", x, ref, scale) == 0, L.evie_last_global_error()
        assert _call(L, "evie_gqa_decode_paged_noalloc", x, got, scale) == 0, L.evie_last_global_error()
        torch.cuda.synchronize()
        err = float((got - ref).abs().max())
        assert err < TOL, f"call {call}: max abs difference {err}"


@pytest.mark.gpu
def test_noalloc_rejects_sizes_beyond_its_scratch(cuda):
    import evie_b200

    L = evie_b200.lib()
    B = 64
    # every page-table entry names the one real page and every context is 1 token, so the inputs are valid
    x = {
        "q": torch.zeros(B, 16, 256, dtype=torch.bfloat16, device=cuda),
        "gate": torch.zeros(B, 16, 256, dtype=torch.bfloat16, device=cuda),
        "kp": torch.zeros(1, 4, 256, 256, dtype=torch.bfloat16, device=cuda),
        "vp": torch.zeros(1, 4, 256, 256, dtype=torch.bfloat16, device=cuda),
        "pt": torch.zeros(B, 64, dtype=torch.int32, device=cuda),
        "ctx": torch.ones(B, dtype=torch.int32, device=cuda),
    }
    out = torch.zeros(B, 16, 256, dtype=torch.float32, device=cuda)
    rc = _call(L, "evie_gqa_decode_paged_noalloc", x, out, 1.0 / 16.0)  # 64 x 4 x 32 splits: beyond 32 MiB
    assert rc == 1
    assert b"split scratch" in L.evie_last_global_error()
    assert float(out.abs().max()) == 0.0
