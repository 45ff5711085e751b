"""bench.py's accounting, on the CPU: the count of our kernel launches per decode step, the algorithmic bytes of the
projection groups against the checkpoint's own tensor list, and the DRAM-traffic lookup from the committed ncu
summaries."""
import types

import numpy as np
import pytest

import bench
from evie_b200 import checkpoint as ck


def _model_4b(B=64):
    return types.SimpleNamespace(cfg=ck.text_config(ck.QWEN35_4B), B=B)


def test_launch_count_matches_the_decode_launch_list():
    """164 of our kernels per 4B decode step, as in the ncu launch list of the decode step: embedding + norm; per
    layer the mixer-side kernels, two add+norms and SwiGLU; logits/argmax, its finish and the row advance."""
    assert bench.ModelDecode.launches_per_step(_model_4b()) == 164


def test_projection_groups_cover_every_projection_weight_once():
    m = _model_4b()
    groups = bench.ModelDecode.group_bytes(m, ctx=4100)
    proj = sum(v for k, v in groups.items() if k.startswith("gemm_")) + groups["lm_head_gemm"]
    names = ("embed_tokens", "in_proj_qkv", "in_proj_z", "in_proj_b", "in_proj_a", "out_proj", "q_proj", "k_proj",
             "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj")
    want = sum(2 * int(np.prod(shape)) for name, shape, _ in ck.tensor_specs(m.cfg)
               if any(f".{t}.weight" in name for t in names))
    assert proj == want  # bf16: the tied embedding once, as the LM head


def test_traffic_lookup():
    assert bench.profiled_traffic("gdn_chunk_prefill_kernel") == 1019800576  # a captured launch
    # the model's decode attention: the captured traffic-to-algorithmic ratio of the same kernel
    assert bench.profiled_traffic("gqa_attention", 1.0e9) == pytest.approx(1.014e9)
    assert bench.profiled_traffic("gqa_attention") is None
    assert bench.profiled_traffic("no_such_kernel") is None
