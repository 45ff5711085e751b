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
    """293 of our kernels per 4B decode step, as in the ncu launch list of the decode step: embedding + norm; per
    layer four projection GEMMs, the mixer-side kernels, two add+norms and SwiGLU; the LM head, logits/argmax, its
    finish and the row advance."""
    assert bench.ModelDecode.launches_per_step(_model_4b()) == 293


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
    assert bench.profiled_traffic("gqa_attention", 1.0e9) == pytest.approx(1.0083e9)
    assert bench.profiled_traffic("gqa_decode_tma_kernel") == 4710427332  # the B=16 capture scaled to B=64
    assert bench.profiled_traffic("gqa_attention") is None
    assert bench.profiled_traffic("no_such_kernel") is None


def test_cpu_baseline_threads_follow_evies_default(monkeypatch):
    """evie's --threads default: half the logical CPUs, clamped to [1, 8] (crates/evie/src/main.rs:111)."""
    import bench

    monkeypatch.delenv("EVIE_CPU_THREADS", raising=False)
    for cpus, want in [(1, 1), (2, 1), (7, 3), (16, 8), (64, 8)]:
        monkeypatch.setattr(bench, "host_cpus", lambda c=cpus: c)
        assert bench.evie_threads() == want
    monkeypatch.setenv("EVIE_CPU_THREADS", "3")
    assert bench.evie_threads() == 3


def test_seeded_oracle_cache_stands_at_the_context(tmp_path):
    """The CPU baseline decodes at the GPU's context from caches put at that position without a prefill: the cache
    reports the position, holds that many key/value rows per attention layer, and a decode step appends one."""
    import numpy as np

    import oracle
    from evie_b200 import checkpoint as ck

    path = str(tmp_path / "tiny")
    ck.write_checkpoint(path, ck.tiny_config(vocab_size=256, num_hidden_layers=4), seed=0)
    m = oracle.Model(path)
    c = m.seeded_cache(300, 1)
    assert c.pos == 300
    full = [i for i, k in enumerate(m.cfg.layer_kinds) if k != "linear"]
    lin = [i for i, k in enumerate(m.cfg.layer_kinds) if k == "linear"]
    row = m.cfg.n_kv_heads * m.cfg.head_dim
    assert full and lin and c.read(full[0], "k").size == 300 * row
    assert np.abs(c.read(lin[0], "state")).max() > 0
    lg, _, _ = m.forward([dict(cache=c, tokens=np.array([5], np.uint32))])
    assert c.pos == 301 and c.read(full[0], "v").size == 301 * row and np.isfinite(lg).all()
