"""Seeded synthetic inputs shared by the parity tests and bench.py (torch CPU generator, so that the oracle and the
GPU read identical bytes)."""
import numpy as np
import torch


def bf16_bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def gdn_decode_inputs(B, H, seed, d=128, device="cpu"):
    """Decode-step distributions: S ~ N(0, 0.1) f32; q, k ~ N(0,1) bf16 L2-normalised per head; v ~ N(0,1) bf16;
    beta = sigmoid(N(0,1)); log decay g ~ U(-5, 0). With device != "cpu" the tensors are drawn there (another
    generator: the same distributions, other values), for timing without a host-side draw."""
    g = torch.Generator(device=device).manual_seed(seed)
    kw = dict(generator=g, device=device)
    S = torch.randn(B, H, d, d, **kw) * 0.1
    q = torch.randn(B, H, d, **kw)
    k = torch.randn(B, H, d, **kw)
    q = (q / q.norm(dim=-1, keepdim=True)).to(torch.bfloat16)
    k = (k / k.norm(dim=-1, keepdim=True)).to(torch.bfloat16)
    v = torch.randn(B, H, d, **kw).to(torch.bfloat16)
    beta = torch.sigmoid(torch.randn(B, H, **kw))
    logd = -5.0 * torch.rand(B, H, **kw)
    return dict(S=S, q=q, k=k, v=v, g=logd, beta=beta)


def gdn_prefill_inputs(B, T, H, seed, d=128, s0=False, device="cpu"):
    """Chunked-prefill distributions (token-major [B, T, H, d]); the initial state is zero unless s0."""
    g = torch.Generator(device=device).manual_seed(seed)
    kw = dict(generator=g, device=device)
    q = torch.randn(B, T, H, d, **kw)
    k = torch.randn(B, T, H, d, **kw)
    q = (q / q.norm(dim=-1, keepdim=True)).to(torch.bfloat16)
    k = (k / k.norm(dim=-1, keepdim=True)).to(torch.bfloat16)
    v = torch.randn(B, T, H, d, **kw).to(torch.bfloat16)
    beta = torch.sigmoid(torch.randn(B, T, H, **kw))
    logd = -5.0 * torch.rand(B, T, H, **kw)
    S = torch.randn(B, H, d, d, **kw) * 0.1 if s0 else torch.zeros(B, H, d, d, device=device)
    return dict(S=S, q=q, k=k, v=v, g=logd, beta=beta)


def gqa_inputs(B, Hq, Hkv, ctx, seed, hd=256, page=256, shuffle_pages=True, device="cpu"):
    """Paged-attention distributions: bf16 KV ~ N(0,1) in `page`-token pages (page table a random permutation);
    q ~ N(0,1) bf16; gate logits ~ N(0,1) bf16."""
    g = torch.Generator().manual_seed(seed)
    gd = torch.Generator(device=device).manual_seed(seed) if device != "cpu" else g
    ctx = [int(c) for c in ctx]
    pages_per = [(c + page - 1) // page for c in ctx]
    max_pages = max(1, max(pages_per))
    n_pages = max(1, sum(pages_per))
    perm = torch.randperm(n_pages, generator=g) if shuffle_pages else torch.arange(n_pages)
    pt = torch.zeros(B, max_pages, dtype=torch.int32)
    o = 0
    for b, n in enumerate(pages_per):
        pt[b, :n] = perm[o:o + n].to(torch.int32)
        o += n
    kw = dict(generator=gd, device=device)
    kp = torch.randn(n_pages, Hkv, page, hd, **kw).to(torch.bfloat16)
    vp = torch.randn(n_pages, Hkv, page, hd, **kw).to(torch.bfloat16)
    q = torch.randn(B, Hq, hd, **kw).to(torch.bfloat16)
    gate = torch.randn(B, Hq, hd, **kw).to(torch.bfloat16)
    return dict(q=q, gate=gate, kp=kp, vp=vp, pt=pt.to(device), ctx=torch.tensor(ctx, dtype=torch.int32, device=device))
