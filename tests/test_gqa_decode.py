"""Gated GQA decode attention over a paged bf16 KV cache (evie_gqa_decode_paged) against the oracle's
restatement of Model::attention's core (softmax over the whole context, P.V, sigmoid gate)."""
import numpy as np
import pytest
import torch

import oracle
from tests._inputs import bf16_bits, gqa_inputs


def _check(B, Hq, Hkv, ctx, seed, cuda, page=256, nan_tail=False):
    from evie_b200 import ops

    x = gqa_inputs(B, Hq, Hkv, ctx, seed, page=page)
    if nan_tail:  # every cache position past a sequence's context holds NaN; none may reach an output
        nan = torch.tensor(float("nan"), dtype=torch.bfloat16)
        for b, c in enumerate(ctx):
            for j in range(c, (c + page - 1) // page * page):
                x["kp"][x["pt"][b, j // page], :, j % page] = nan
                x["vp"][x["pt"][b, j // page], :, j % page] = nan
    scale = 1.0 / 16.0
    ref = oracle.gqa_decode(bf16_bits(x["q"]), bf16_bits(x["kp"]), bf16_bits(x["vp"]), x["pt"].numpy(),
                            x["ctx"].numpy(), bf16_bits(x["gate"]), scale)
    out = ops.gqa_decode_paged(x["q"].to(cuda), x["gate"].to(cuda), x["kp"].to(cuda), x["vp"].to(cuda),
                               x["pt"].to(cuda), x["ctx"].to(cuda), scale)
    torch.cuda.synchronize()
    out = out.cpu().numpy()
    assert np.isfinite(out).all()
    # fp32 arithmetic on identical bf16 inputs; differences come from summation order only
    assert np.abs(out - ref).max() < 2e-5, float(np.abs(out - ref).max())
    return out


@pytest.mark.gpu
@pytest.mark.parametrize("ctx", [[1], [0, 5], [63, 64, 65], [255, 256, 257], [511, 512, 513], [1000, 2048, 4097]])
def test_gqa_decode_edges(ctx, cuda):
    _check(len(ctx), 16, 4, ctx, 11, cuda)


@pytest.mark.gpu
@pytest.mark.parametrize("ctx", [[1, 17, 250], [513, 1000, 4097]])
def test_gqa_decode_garbage_past_context(ctx, cuda):
    """Tiles are read whole: the rows past each context (here NaN) are masked in the scores and zeroed in V."""
    _check(len(ctx), 16, 4, ctx, 13, cuda, nan_tail=True)


@pytest.mark.gpu
@pytest.mark.parametrize("page", [64, 128])
def test_gqa_decode_group4_small_pages(page, cuda):
    """Pages no larger than a warp's 128 tokens (the op accepts multiples of 64): a warp's tiles cross pages, and
    each 16-token tile finds its own page (the tensor-core kernels)."""
    _check(3, 16, 4, [100, 700, 1300], 14, cuda, page=page, nan_tail=True)


@pytest.mark.gpu
def test_gqa_decode_group2_and_small_pages(cuda):
    _check(3, 8, 4, [100, 700, 1300], 12, cuda, page=64)


@pytest.mark.gpu
def test_gqa_decode_ctx1k_32k_sample(cuda):
    """The B=64 attention shapes (16 q / 4 kv heads, hd 256, 256-token pages) with contexts drawn from U[1024, 32768]."""
    g = torch.Generator().manual_seed(4)
    ctx = torch.randint(1024, 32769, (8,), generator=g).tolist()
    _check(8, 16, 4, ctx, 4, cuda)


@pytest.mark.gpu
def test_gqa_decode_repeat_is_deterministic(cuda):
    """The in-kernel split merge resets its tickets: back-to-back calls give bit-identical results."""
    from evie_b200 import ops

    x = gqa_inputs(4, 16, 4, [3000, 9000, 1, 600], 21)
    args = [x[k].to(cuda) for k in ("q", "gate", "kp", "vp", "pt", "ctx")]
    a = ops.gqa_decode_paged(*args, 1 / 16)
    b = ops.gqa_decode_paged(*args, 1 / 16)
    torch.cuda.synchronize()
    assert torch.equal(a, b)
