"""Reduced captures: the k most active neurons per captured frame (evie_top_active, evie_read_top_active) against
the oracle's restatement of evie's top_active tool (crates/evie/src/mcp.rs:242-256), bit for bit. The reference
leaves the order of equal |q| undefined; both sides fix it as the lower flat index first."""
import numpy as np
import pytest

import oracle


def _np_top_active(frame, k):
    mag = np.abs(frame.astype(np.int32))
    order = np.lexsort((np.arange(frame.size), -mag))  # |q| descending, then index
    return order[:k].astype(np.int32)


def test_oracle_matches_numpy_ranking():
    rng = np.random.default_rng(0)
    for width, lo, hi in ((1000, -127, 128), (5000, -3, 4), (64, -1, 2)):
        f = rng.integers(lo, hi, width).astype(np.int8)
        for k in (1, 20, 100):
            assert np.array_equal(oracle.top_active(f, k), _np_top_active(f, k)[:min(k, width)])


def test_distinct_magnitudes_need_no_tie_rule():
    """Where every |q| differs the reference's order is fully determined; the oracle returns it."""
    f = np.array([5, -9, 2, 7, -1, 0, 3], np.int8)
    assert list(oracle.top_active(f, 4)) == [1, 3, 0, 6]


@pytest.mark.gpu
@pytest.mark.parametrize("width,lo,hi", [(294912, -127, 128), (294912, -4, 5), (3584 * 24, -127, 128), (60, -2, 3)])
def test_top_active_op_matches_oracle(width, lo, hi, cuda):
    import torch

    from evie_b200 import ops

    rng = np.random.default_rng(width + hi)
    rows = 24
    f = rng.integers(lo, hi, (rows, width)).astype(np.int8)
    f[3, :] = 0  # a row of ties only
    for k in (1, 20, 100):
        got = ops.top_active(torch.from_numpy(f).to(cuda), k).cpu().numpy()
        kk = min(k, width)
        for r in range(rows):
            assert np.array_equal(got[r, :kk], oracle.top_active(f[r], k)), (k, r)


@pytest.mark.gpu
def test_read_top_active_after_forward(cuda, tmp_path):
    """evie_read_top_active on the frames a capturing evie_forward left on the device equals top_active of the
    frames copied back, for every row; after a decode-loop call it covers that call's last step."""
    from evie_b200 import checkpoint as ck
    from evie_b200.gpu import GpuModel, GpuSeq

    path = str(tmp_path / "tiny")
    ck.write_checkpoint(path, ck.tiny_config(vocab_size=2048, num_hidden_layers=4), seed=6)
    m = GpuModel(path, max_ctx=128, slots=2, max_rows=64)
    m.set_scale(np.full(m.layers * m.neurons, 0.02, np.float32))
    rng = np.random.default_rng(2)
    prompts = [rng.integers(0, 2048, 17).astype(np.uint32), rng.integers(0, 2048, 5).astype(np.uint32)]
    out = m.forward([GpuSeq(i, 0, p) for i, p in enumerate(prompts)], capture=True)
    got = m.top_active(30)
    assert got.shape == (22, 30)
    for r in range(22):
        assert np.array_equal(got[r], oracle.top_active(out.frames[r], 30)), r
    frames = np.zeros((3, 2, m.layers * m.neurons), np.int8)
    m.decode_greedy([GpuSeq(i, len(p), out.next_tokens[i:i + 1]) for i, p in enumerate(prompts)], 3, capture=True,
                    frames=frames)
    got = m.top_active(7)
    assert got.shape == (2, 7)
    for r in range(2):
        assert np.array_equal(got[r], oracle.top_active(frames[2, r], 7)), r
    m.close()
