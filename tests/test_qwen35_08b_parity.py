"""Qwen3.5-0.8B parity run: the public 0.8B shapes (24 layers, MLP width 3584, 18 DeltaNet + 6 gated-attention
layers), every weight bf16 N(0, 0.02) from seed 0 with norm gains stored as 1.0, batch 1, a 64-token prompt of uniform random ids
from seed 1, then 64 greedy decode steps. The GPU path must produce the oracle's greedy ids exactly and logits
within 2e-3 max-abs at every step. The checkpoint (about 2 GB) is written to a temporary directory."""
import os
import tempfile

import numpy as np
import pytest
import torch

import oracle
from evie_b200 import checkpoint as ck

STEPS = 64
# Both cache formats are held to identical greedy ids, each against the oracle run with the same key/value storage:
# the f32 cache (EVIE_KV_F32=1) against the reference arithmetic as it is, with logits within 2e-3 max-abs; the
# default bf16 paged cache against the oracle with kv_bf16 (each appended key and value rounded to bf16, its one
# documented deviation from model.rs:441-442), with logits within 1e-2.
# Why the bf16 bound is wider: on these random weights the attention scores are ~N(0, 4^2), a peaked softmax, and a
# key or value that lies near a bf16 rounding boundary rounds the other way when the f32 value before rounding moves
# by a few ulps. The oracle disagrees with itself that way: scaling its keys and values by 1 + 1e-5 r (r uniform in
# [-1, 1)) before rounding moves its own logits by ~6.5e-3 over these 65 steps (1e-7: 2.7e-3, 1e-6: 3.6e-3). Any
# implementation whose f32 arithmetic is ordered differently lands in that band, so the test measures the band
# (BAND_JITTER) and checks that it lies above 2e-3.
LOGIT_TOL = {True: 2e-3, False: 1e-2}
BAND_JITTER = 1e-5


def parity_prompt(vocab: int) -> np.ndarray:
    g = torch.Generator().manual_seed(1)
    return torch.randint(0, vocab, (64,), generator=g).numpy().astype(np.uint32)


@pytest.fixture(scope="module")
def c0_ckpt():
    path = os.path.join(os.environ.get("EVIE_CKPT_DIR", tempfile.gettempdir()), "evie_qwen35_0p8b_seed0")
    return ck.ensure_checkpoint(path, ck.text_config(ck.QWEN35_0_8B), seed=0)


@pytest.fixture(scope="module")
def c0_reference(c0_ckpt):
    """The oracle's greedy run: ids and per-step logits (prefill logits first), per key/value storage format."""
    runs = {}

    def run(kv_bf16: bool, kv_perturb: float = 0.0):
        key = (kv_bf16, kv_perturb)
        if key not in runs:
            oracle.set_threads(os.cpu_count() or 1)
            m = oracle.Model(c0_ckpt, kv_bf16=kv_bf16, kv_perturb=kv_perturb)
            prompt = parity_prompt(m.cfg.vocab)
            cache = m.new_cache()
            lg, _, _ = m.forward([dict(cache=cache, tokens=prompt)])
            ids, logits = [], [lg[0].copy()]
            for _ in range(STEPS):
                t = oracle.greedy(logits[-1])
                ids.append(t)
                lg, _, _ = m.forward([dict(cache=cache, tokens=np.array([t], np.uint32))])
                logits.append(lg[0].copy())
            runs[key] = (prompt, ids, logits)
        return runs[key]

    return run


def _margin(l):
    top = np.sort(l)[-2:]
    return float(top[1] - top[0])


@pytest.mark.gpu
@pytest.mark.parametrize("kv_f32", [True, False])
def test_08b_greedy_ids_and_logits(c0_ckpt, c0_reference, kv_f32, cuda):
    from evie_b200.gpu import GpuModel, GpuSeq

    prompt, ids_ref, logits_ref = c0_reference(not kv_f32)
    os.environ["EVIE_KV_F32"] = "1" if kv_f32 else "0"
    try:
        m = GpuModel(c0_ckpt, max_ctx=256, slots=1, max_rows=64)
    finally:
        os.environ.pop("EVIE_KV_F32", None)
    out = m.forward([GpuSeq(0, 0, prompt)])
    errs = [float(np.abs(out.logits[0] - logits_ref[0]).max())]
    ids = []
    pos = len(prompt)
    for step in range(STEPS):
        t = int(out.next_tokens[0])
        ids.append(t)
        if t != ids_ref[step]:
            break
        out = m.forward([GpuSeq(0, pos, np.array([t], np.uint32))])
        pos += 1
        errs.append(float(np.abs(out.logits[0] - logits_ref[step + 1]).max()))
    m.close()
    first_diff = next((i for i, (a, b) in enumerate(zip(ids, ids_ref)) if a != b), None)
    assert first_diff is None, (
        f"greedy ids diverge at step {first_diff} (oracle top1-top2 margin {_margin(logits_ref[first_diff]):.2e})")
    if not kv_f32:
        # the oracle's own spread under a 1e-5 relative jitter before the bf16 rounding
        _, ids_j, logits_j = c0_reference(True, BAND_JITTER)
        band = max(float(np.abs(a - b).max()) for a, b in zip(logits_j, logits_ref))
        assert ids_j == ids_ref and band > 2e-3, band
    assert max(errs) < LOGIT_TOL[kv_f32], f"max logit error {max(errs):.3e} (per step: {np.round(errs, 6).tolist()})"
