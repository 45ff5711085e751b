"""Isolated hot-path ops on torch CUDA tensors, through the C ABI of libevie_cuda.so.

torch provides device memory and the stream; the computation is the library's sm_100a kernels.
"""
from __future__ import annotations

import torch

from . import check, lib


def _ptr(t: torch.Tensor) -> int:
    assert t.is_cuda and t.is_contiguous(), "expected a contiguous CUDA tensor"
    return t.data_ptr()


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def gdn_decode_step(q, k, v, g, beta, state, o=None):
    """One Gated DeltaNet recurrent step (evie_gdn_decode_step). state [B,H,128,128] f32 is updated in place.

    q, k: [B,H,128] bf16; v: [B,H,128] bf16; g (log decay), beta: [B,H] f32. Returns o [B,H,128] f32."""
    B, H, dk, dv = state.shape
    assert q.dtype == k.dtype == v.dtype == torch.bfloat16 and state.dtype == torch.float32
    if o is None:
        o = torch.empty(B, H, dv, device=state.device, dtype=torch.float32)
    check(lib().evie_gdn_decode_step(_ptr(q), _ptr(k), _ptr(v), _ptr(g), _ptr(beta), _ptr(state), _ptr(o), B, H,
                                     dk, dv, _stream()))
    return o


def gdn_chunk_prefill(q, k, v, g, beta, state, o=None, chunk: int = 64):
    """Chunked Gated DeltaNet prefill (evie_gdn_chunk_prefill). q,k,v: [B,T,H,128] bf16; g,beta: [B,T,H] f32;
    state [B,H,128,128] f32: initial in, final out. Returns o [B,T,H,128] bf16."""
    B, T, H, dk = q.shape
    dv = v.shape[-1]
    if o is None:
        o = torch.empty(B, T, H, dv, device=q.device, dtype=torch.bfloat16)
    check(lib().evie_gdn_chunk_prefill(_ptr(q), _ptr(k), _ptr(v), _ptr(g), _ptr(beta), _ptr(state), _ptr(o), B, T,
                                       H, dk, dv, chunk, _stream()))
    return o


def gdn_prefill_tokenwise(q, k, v, g, beta, state, o=None):
    """Token-by-token Gated DeltaNet prefill (evie_gdn_prefill_tokenwise); same layouts as gdn_chunk_prefill."""
    B, T, H, dk = q.shape
    dv = v.shape[-1]
    if o is None:
        o = torch.empty(B, T, H, dv, device=q.device, dtype=torch.bfloat16)
    check(lib().evie_gdn_prefill_tokenwise(_ptr(q), _ptr(k), _ptr(v), _ptr(g), _ptr(beta), _ptr(state), _ptr(o), B,
                                           T, H, dk, dv, _stream()))
    return o


def gqa_prefill_paged(q, gate, k_pages, v_pages, page_table, seq_rows, seq_pos0, scale, out=None):
    """Gated GQA attention for prefill rows (evie_gqa_prefill_paged). q, gate: [R,Hq,256] f32; k_pages, v_pages:
    [P,Hkv,page,256] bf16; page_table [n_seqs,max_pages] int32 (device); seq_rows, seq_pos0: lists of n_seqs ints
    (sequence s owns the next seq_rows[s] rows, at positions seq_pos0[s] ...). Returns out [R,Hq,256] f32."""
    import ctypes as C

    R, Hq, hd = q.shape
    P, Hkv, page, _ = k_pages.shape
    n = len(seq_rows)
    if out is None:
        out = torch.empty(R, Hq, hd, device=q.device, dtype=torch.float32)
    rows = (C.c_int32 * n)(*seq_rows)
    pos0 = (C.c_int32 * n)(*seq_pos0)
    check(lib().evie_gqa_prefill_paged(_ptr(q), _ptr(gate), _ptr(k_pages), _ptr(v_pages), P, _ptr(page_table),
                                       page_table.shape[1], rows, pos0, n, _ptr(out), Hq, Hkv, hd, page,
                                       float(scale), _stream()))
    return out


def split_planes(x: torch.Tensor) -> torch.Tensor:
    """The split operand of an f32 matrix x [R,K]: [2,R,K] bf16 with hi = bf16(x) and lo = bf16(x - hi)."""
    hi = x.to(torch.bfloat16)
    lo = (x - hi.float()).to(torch.bfloat16)
    return torch.stack([hi, lo]).contiguous()


def proj_gemm(w, x2, max_planes: int = 16):
    """Projection GEMM (evie_proj_gemm): w [M,K] bf16, x2 [2,R,K] bf16 split operand. Returns the K-slice planes
    [planes,R,M] f32 whose sum (in slice order) is x w^T."""
    M, K = w.shape
    R = x2.shape[1]
    assert w.dtype == x2.dtype == torch.bfloat16 and x2.shape == (2, R, K)
    y = torch.empty(max_planes, R, M, device=w.device, dtype=torch.float32)
    import ctypes as C

    planes = C.c_int(0)
    check(lib().evie_proj_gemm(_ptr(w), _ptr(x2), _ptr(y), y.numel(), M, K, R, max_planes, C.byref(planes),
                               _stream()))
    return y[: planes.value]


def sampler_seed_state(seed: int) -> int:
    """Sampler::new's generator state for a seed (sampling.rs:27-29)."""
    return int(lib().evie_sampler_seed_state(seed))


def sample(logits, params, rng, histories):
    """Sampler::sample (sampling.rs:41-93) for each row of logits [B,V] f32 (CUDA) with params[b] = dict(temperature,
    top_p, min_p, repetition_penalty) and histories[b] a list of token ids. rng: list of B generator states, advanced
    in place. Returns the B tokens (synchronous)."""
    import ctypes as C

    import numpy as np

    from . import capi

    B, V = logits.shape
    ps = (capi.SampleParams * B)(*[capi.SampleParams(p.get("temperature", 0.0), p.get("top_p", 1.0),
                                                     p.get("min_p", 0.0), p.get("repetition_penalty", 1.0), 0)
                                   for p in params])
    st = (C.c_uint64 * B)(*rng)
    off = np.zeros(B + 1, np.int64)
    off[1:] = np.cumsum([len(h) for h in histories])
    flat = np.concatenate([np.asarray(h, np.uint32) for h in histories] + [np.zeros(1, np.uint32)])
    hist = torch.from_numpy(flat.astype(np.int32)).to(logits.device)
    out = np.zeros(B, np.uint32)
    check(lib().evie_sample(_ptr(logits), B, V, ps, st, _ptr(hist), off.ctypes.data, out.ctypes.data, _stream()))
    rng[:] = list(st)
    return out


def top_active(frames, k: int, out=None):
    """evie's top_active (mcp.rs:242-256) for every row of frames [rows, width] int8 (CUDA): [rows, k] int32 flat
    indices, by |q| descending, equal |q| by increasing index."""
    rows, width = frames.shape
    if out is None:
        out = torch.empty(rows, k, device=frames.device, dtype=torch.int32)
    check(lib().evie_top_active(_ptr(frames), rows, width, k, _ptr(out), _stream()))
    return out


def poll_device_errors() -> None:
    """Raises EvieError if a kernel gave up a bounded device-side wait since the last poll (synchronises)."""
    check(lib().evie_poll_device_errors())


def bounded_wait_probe(limit_ns: int) -> int:
    """Runs the failure path of the kernels' bounded waits (evie_bounded_wait_probe): one thread waits at most
    limit_ns on an mbarrier that nothing completes and counts the give-up for poll_device_errors. Returns 1 if it
    gave up."""
    import ctypes as C

    out = C.c_int(-1)
    check(lib().evie_bounded_wait_probe(C.c_uint64(int(limit_ns)), C.byref(out)))
    return out.value


def gqa_decode_paged(q, gate, k_pages, v_pages, page_table, ctx_lens, scale, out=None):
    """Gated GQA decode attention over a paged bf16 KV cache (evie_gqa_decode_paged).

    q, gate: [B,Hq,256] bf16; k_pages, v_pages: [P,Hkv,page,256] bf16; page_table [B,max_pages] int32;
    ctx_lens [B] int32. Returns out [B,Hq,256] f32."""
    B, Hq, hd = q.shape
    _, Hkv, page, _ = k_pages.shape
    if out is None:
        out = torch.empty(B, Hq, hd, device=q.device, dtype=torch.float32)
    check(lib().evie_gqa_decode_paged(_ptr(q), _ptr(gate), _ptr(k_pages), _ptr(v_pages), _ptr(page_table),
                                      _ptr(ctx_lens), _ptr(out), B, Hq, Hkv, hd, page, page_table.shape[1],
                                      float(scale), _stream()))
    return out
