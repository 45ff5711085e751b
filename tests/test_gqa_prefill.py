"""Prefill attention (evie_gqa_prefill_paged, the tcgen05 kernel behind the model's prefill rows) against the oracle's
restatement of the attention core of Model::attention (model.rs:445-464) on the same bf16 pages.

Cases: ragged sequences in one call, rows whose context starts before the call (pos0 > 0), contexts that cross
256-token pages, blocks of 32 rows that end inside a sequence, both attention geometries (16/4 and 8/2 heads), and
a peaked softmax (queries scaled up). Cache entries past each sequence's last position hold NaN: the kernel must
never let them reach an output (their scores are masked and their V rows are zeroed before P V)."""
import numpy as np
import pytest
import torch

import oracle
from tests._inputs import bf16_bits

# f32 summation-order tolerance; q enters the tensor core as bf16 hi + lo (~2^-17 relative), so the score error, and
# with it the bound, grows with the size of the scores (qscale)
TOL = 2e-5


def _case(seq_rows, seq_pos0, Hq, Hkv, seed, qscale=1.0, page=256, hd=256):
    g = torch.Generator().manual_seed(seed)
    n = len(seq_rows)
    ends = [p + r for p, r in zip(seq_pos0, seq_rows)]
    pages_per = [(e + page - 1) // page for e in ends]
    max_pages = max(pages_per)
    n_pages = sum(pages_per)
    perm = torch.randperm(n_pages, generator=g)
    pt = torch.zeros(n, max_pages, dtype=torch.int32)
    o = 0
    for s, k in enumerate(pages_per):
        pt[s, :k] = perm[o:o + k].to(torch.int32)
        o += k
    kp = torch.randn(n_pages, Hkv, page, hd, generator=g).to(torch.bfloat16)
    vp = torch.randn(n_pages, Hkv, page, hd, generator=g).to(torch.bfloat16)
    nan = torch.tensor(float("nan"), dtype=torch.bfloat16)
    for s, e in enumerate(ends):  # positions past the sequence's last row: anything, here NaN
        for j in range(e, pages_per[s] * page):
            kp[pt[s, j // page], :, j % page] = nan
            vp[pt[s, j // page], :, j % page] = nan
    R = sum(seq_rows)
    q = torch.randn(R, Hq, hd, generator=g) * qscale
    gate = torch.randn(R, Hq, hd, generator=g)
    row_seq = np.concatenate([np.full(r, s, np.int32) for s, r in enumerate(seq_rows)])
    row_pos = np.concatenate([np.arange(p, p + r, dtype=np.int32) for p, r in zip(seq_pos0, seq_rows)])
    return dict(q=q, gate=gate, kp=kp, vp=vp, pt=pt, row_seq=row_seq, row_pos=row_pos)


@pytest.mark.gpu
@pytest.mark.parametrize("seq_rows,seq_pos0,Hq,Hkv,qscale", [
    ([300], [0], 16, 4, 1.0),                 # one prompt crossing a page, the last block partial (300 = 9 x 32 + 12)
    ([37, 100, 5], [0, 250, 600], 16, 4, 1.0),  # ragged; two sequences continue earlier context, across pages
    ([64, 33], [0, 190], 8, 2, 1.0),           # the 0.8B geometry
    ([96], [31], 16, 4, 4.0),                  # peaked softmax (scores ~N(0, 16))
])
def test_prefill_attention_matches_oracle(seq_rows, seq_pos0, Hq, Hkv, qscale, cuda):
    from evie_b200 import ops

    x = _case(seq_rows, seq_pos0, Hq, Hkv, 7 + sum(seq_rows), qscale)
    scale = 1.0 / 16.0
    ref = oracle.gqa_rows(x["q"].numpy(), bf16_bits(x["kp"]), bf16_bits(x["vp"]), x["pt"].numpy(), x["row_seq"],
                          x["row_pos"], x["gate"].numpy(), scale)
    out = ops.gqa_prefill_paged(x["q"].to(cuda), x["gate"].to(cuda), x["kp"].to(cuda), x["vp"].to(cuda),
                                x["pt"].to(cuda), seq_rows, seq_pos0, scale)
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    assert np.isfinite(got).all()
    err = float(np.abs(got - ref).max())
    assert err < TOL * max(1.0, qscale), err


def test_prefill_attention_rejects_bad_arguments():
    """Argument checks run before any device work."""
    import ctypes as C

    from evie_b200 import lib

    L = lib()
    rows = (C.c_int32 * 1)(4)
    pos0 = (C.c_int32 * 1)(0)
    rc = L.evie_gqa_prefill_paged(None, None, None, None, 1, None, 1, rows, pos0, 1, None, 16, 4, 128, 256, 1.0, None)
    assert rc == 1 and b"head_dim 256" in L.evie_last_global_error()
    rc = L.evie_gqa_prefill_paged(None, None, None, None, 1, None, 1, rows, pos0, 1, None, 12, 4, 256, 256, 1.0, None)
    assert rc == 1 and b"4 x Hkv" in L.evie_last_global_error()
