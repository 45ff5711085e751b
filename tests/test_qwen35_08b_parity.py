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
# 2e-3 is the contract with the oracle's f32 KV cache (EVIE_KV_F32=1). With the bf16 paged KV cache (the default
# storage) the keys and values are rounded to 8 significant bits; on these random weights the attention scores
# are ~N(0, 4^2), a peaked softmax that turns that rounding into ~1-2e-2 logit differences (measured 2.1e-2 max).
# The bf16 cache is held to identical greedy ids and a 3e-2 logit bound.
LOGIT_TOL = {True: 2e-3, False: 3e-2}


def parity_prompt(vocab: int) -> np.ndarray:
    g = torch.Generator().manual_seed(1)
    return torch.randint(0, vocab, (64,), generator=g).numpy().astype(np.uint32)


@pytest.fixture(scope="module")
def c0_ckpt():
    path = os.path.join(os.environ.get("EVIE_CKPT_DIR", tempfile.gettempdir()), "evie_qwen35_0p8b_seed0")
    return ck.ensure_checkpoint(path, ck.text_config(ck.QWEN35_0_8B), seed=0)


@pytest.fixture(scope="module")
def c0_reference(c0_ckpt):
    """The oracle's greedy run: ids and per-step logits (prefill logits first)."""
    oracle.set_threads(os.cpu_count() or 1)
    m = oracle.Model(c0_ckpt)
    prompt = parity_prompt(m.cfg.vocab)
    cache = m.new_cache()
    lg, _, _ = m.forward([dict(cache=cache, tokens=prompt)])
    ids, logits = [], [lg[0].copy()]
    for _ in range(STEPS):
        t = oracle.greedy(logits[-1])
        ids.append(t)
        lg, _, _ = m.forward([dict(cache=cache, tokens=np.array([t], np.uint32))])
        logits.append(lg[0].copy())
    return prompt, ids, logits


def _margin(l):
    top = np.sort(l)[-2:]
    return float(top[1] - top[0])


@pytest.mark.gpu
@pytest.mark.parametrize("kv_f32", [True, False])
def test_08b_greedy_ids_and_logits(c0_ckpt, c0_reference, kv_f32, cuda):
    from evie_b200.gpu import GpuModel, GpuSeq

    prompt, ids_ref, logits_ref = c0_reference
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
    assert max(errs) < LOGIT_TOL[kv_f32], f"max logit error {max(errs):.3e} (per step: {np.round(errs, 6).tolist()})"
