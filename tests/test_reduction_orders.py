"""Summation orders of the q/k head norm in the DeltaNet conv, replayed in float32 on the CPU.

The one-thread-per-channel conv kernels (conv_silu_norm_kernel, conv_rows_kernel) sum a head block's 128 squares
with block_sum<128>: a butterfly over each warp's 32 lanes (xor 16, 8, 4, 2, 1), then the four warp sums in order.
The decode kernel (conv_decode4_kernel) holds four channels per lane: lane xors 4, 2, 1, then the lane's
elements as (e0 + e2) + (e1 + e3), then the four 32-channel groups in order. Both trees add the same pairs, so the
sums are bit-identical, which keeps decode and prefill rows on the same head norm."""
import numpy as np


def _block_sum_128(v):
    """block_sum<128> over one value per thread (thread t = channel t)."""
    v = v.astype(np.float32)
    partial = []
    for w in range(4):
        x = v[32 * w:32 * w + 32].copy()
        for off in (16, 8, 4, 2, 1):
            x = (x + x[np.arange(32) ^ off]).astype(np.float32)
        partial.append(x[0])
    t = np.float32(0.0)
    for p in partial:
        t = np.float32(t + p)
    return t


def _lane4_tree(v):
    """conv_decode4_kernel: lane l holds channels 4l .. 4l + 3 (element e = channel % 4)."""
    sq = v.astype(np.float32).reshape(32, 4).copy()  # [lane][element]
    for off in (4, 2, 1):
        sq = (sq + sq[np.arange(32) ^ off]).astype(np.float32)
    grp = ((sq[:, 0] + sq[:, 2]).astype(np.float32) + (sq[:, 1] + sq[:, 3]).astype(np.float32)).astype(np.float32)
    g0, g1, g2, g3 = grp[0], grp[8], grp[16], grp[24]
    return np.float32(np.float32(np.float32(g0 + g1) + g2) + g3)


def test_decode_conv_norm_sums_in_the_cta_wide_order():
    rng = np.random.default_rng(0)
    for scale in (1e-3, 1.0, 37.0):
        for _ in range(200):
            out = (rng.standard_normal(128) * scale).astype(np.float32)
            sq = (out * out).astype(np.float32)
            assert _lane4_tree(sq).tobytes() == _block_sum_128(sq).tobytes()


def test_the_two_trees_differ_from_a_plain_sequential_sum():
    """The check has teeth: a different association order does change some sums."""
    rng = np.random.default_rng(1)
    differs = 0
    for _ in range(200):
        sq = (rng.standard_normal(128) ** 2).astype(np.float32)
        seq = np.float32(0.0)
        for x in sq:
            seq = np.float32(seq + x)
        differs += seq.tobytes() != _block_sum_128(sq).tobytes()
    assert differs > 0
