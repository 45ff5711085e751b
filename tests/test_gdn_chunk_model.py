"""The chunked DeltaNet prefill inside the forward pass (gdn_chunk.cu, model form) against the oracle's token-by-token
recurrence (model.rs:362-387).

One call carries four ragged segments: a sequence that continues 70 tokens fed by an earlier call (its recurrent
state and conv window enter the chunked kernel non-zero), a single-row segment, a segment of exactly one 64-row chunk
and one of 200 rows (four chunks, the last partial). Segments sit back to back in the call's rows, so every partial
last chunk loads rows of the next segment into its tiles; those rows must not reach its results. Then greedy decode
steps on the states the chunked kernel left behind. The tiny checkpoint has 2 key heads and 4 value heads, so value
heads share key heads as in the Qwen3.5 models. Bars: the model tests' (logits within 2e-3 with the f32 KV cache,
greedy ids identical)."""
import numpy as np
import pytest

import oracle
from evie_b200 import checkpoint as ck

LOGIT_TOL = 2e-3
SEGS = [130, 1, 64, 200]  # rows per segment in the ragged call; segment 0 continues a 70-token prefix
PREFIX = 70
STEPS = 4


@pytest.fixture(scope="module")
def tiny_ckpt(tmp_path_factory):
    path = str(tmp_path_factory.mktemp("ckpt") / "tiny_chunk")
    ck.write_checkpoint(path, ck.tiny_config(vocab_size=2048, num_hidden_layers=8), seed=2)
    return path


@pytest.mark.gpu
def test_ragged_chunked_prefill_then_decode(tiny_ckpt, cuda, monkeypatch):
    from evie_b200.gpu import GpuModel, GpuSeq

    rng = np.random.default_rng(17)
    prefix = rng.integers(0, 2048, PREFIX).astype(np.uint32)
    prompts = [rng.integers(0, 2048, n).astype(np.uint32) for n in SEGS]

    ref = oracle.Model(tiny_ckpt)
    caches = [ref.new_cache() for _ in SEGS]
    ref.forward([dict(cache=caches[0], tokens=prefix)])
    lg, _, _ = ref.forward([dict(cache=caches[i], tokens=prompts[i]) for i in range(len(SEGS))])
    ref_logits = [np.stack(lg)]
    ref_ids = []
    for _ in range(STEPS):
        nxt = [oracle.greedy(lg[i]) for i in range(len(SEGS))]
        ref_ids.append(nxt)
        lg, _, _ = ref.forward([dict(cache=caches[i], tokens=np.array([nxt[i]], np.uint32)) for i in range(len(SEGS))])
        ref_logits.append(np.stack(lg))

    monkeypatch.setenv("EVIE_KV_F32", "1")
    m = GpuModel(tiny_ckpt, max_ctx=512, slots=len(SEGS), max_rows=sum(SEGS))
    m.forward([GpuSeq(0, 0, prefix)])
    pos = [PREFIX, 0, 0, 0]
    out = m.forward([GpuSeq(i, pos[i], prompts[i]) for i in range(len(SEGS))])
    errs = [float(np.abs(out.logits - ref_logits[0]).max(axis=1).max())]
    per_seg = np.abs(out.logits - ref_logits[0]).max(axis=1)
    pos = [p + n for p, n in zip(pos, SEGS)]
    for step in range(STEPS):
        got = [int(t) for t in out.next_tokens]
        assert got == ref_ids[step], f"greedy ids diverge at step {step}: {got} vs {ref_ids[step]}"
        out = m.forward([GpuSeq(i, pos[i], np.array([got[i]], np.uint32)) for i in range(len(SEGS))])
        pos = [p + 1 for p in pos]
        errs.append(float(np.abs(out.logits - ref_logits[step + 1]).max()))
    m.close()
    assert max(errs) < LOGIT_TOL, f"per call {np.round(errs, 6).tolist()}, per segment {per_seg.tolist()}"


@pytest.mark.gpu
def test_chunked_and_sequential_prefill_agree(tiny_ckpt, cuda, monkeypatch):
    """The same ragged call through the chunked kernel and through the token-sequential kernel (EVIE_GDN_SEQ=1)."""
    from evie_b200.gpu import GpuModel, GpuSeq

    rng = np.random.default_rng(23)
    prompts = [rng.integers(0, 2048, n).astype(np.uint32) for n in SEGS]
    monkeypatch.setenv("EVIE_KV_F32", "1")
    outs = []
    for seq in ("0", "1"):
        monkeypatch.setenv("EVIE_GDN_SEQ", seq)
        m = GpuModel(tiny_ckpt, max_ctx=512, slots=len(SEGS), max_rows=sum(SEGS))
        out = m.forward([GpuSeq(i, 0, prompts[i]) for i in range(len(SEGS))])
        nxt = m.forward([GpuSeq(i, SEGS[i], np.array([int(out.next_tokens[i])], np.uint32))
                         for i in range(len(SEGS))])
        outs.append((out.logits.copy(), nxt.logits.copy()))
        m.close()
    for a, b in zip(outs[0], outs[1]):
        assert np.abs(a - b).max() < LOGIT_TOL
