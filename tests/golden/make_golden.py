"""Generates the golden fixtures that pin the CPU oracle (run in this repository's image: `python
tests/golden/make_golden.py`).

evie-core itself (Rust) cannot be built here, and its repository holds no golden vectors for this path. Its README
states that its CPU engine matches HF transformers' Qwen3.5 (identical token ids, logits within 2e-5), and its own
dump tool (tools/reference.py) runs transformers for that comparison. This script does the same on seeded synthetic
inputs, in float32 on the CPU:

  qwen35_tiny.npz  a small Qwen3.5-shaped checkpoint (evie_b200.checkpoint.tiny_config(vocab_size=1024), seed 0):
                   transformers' logits for a 24-token prompt and 6 greedy continuation steps;
  gdn.npz          transformers' torch_recurrent_gated_delta_rule and torch_chunk_gated_delta_rule on one set of
                   gated-delta-rule inputs (dk = dv = 64, so that the functions' internal q * dk^-0.5 is exact).
"""
import hashlib
import os
import sys
import tempfile

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from evie_b200 import checkpoint as ck  # noqa: E402


def sha256(path):
    h = hashlib.sha256()
    with open(path, "rb") as f:
        for chunk in iter(lambda: f.read(1 << 20), b""):
            h.update(chunk)
    return h.hexdigest()


def tiny_model():
    from transformers.models.qwen3_5 import configuration_qwen3_5 as CC
    from transformers.models.qwen3_5 import modeling_qwen3_5 as M

    cfg = ck.tiny_config(vocab_size=1024)
    path = os.path.join(tempfile.mkdtemp(), "tiny")
    ck.write_checkpoint(path, cfg, seed=0)
    hc = CC.Qwen3_5TextConfig(**{k: v for k, v in cfg.items() if k != "model_type"})
    hc._attn_implementation = "eager"
    model = M.Qwen3_5ForCausalLM(hc).float().eval()
    sd = {}
    import json
    import struct

    with open(os.path.join(path, "model.safetensors"), "rb") as f:
        n = struct.unpack("<Q", f.read(8))[0]
        header = json.loads(f.read(n))
        base = 8 + n
        for name, h in header.items():
            if name == "__metadata__":
                continue
            s, e = h["data_offsets"]
            f.seek(base + s)
            raw = np.frombuffer(f.read(e - s), np.uint16)
            t = torch.from_numpy((raw.astype(np.uint32) << 16).view(np.float32).reshape(h["shape"]).copy())
            sd[name.replace("model.language_model.", "model.")] = t
    sd["lm_head.weight"] = sd["model.embed_tokens.weight"]
    missing = model.load_state_dict(sd, strict=False)
    assert not missing.missing_keys and not missing.unexpected_keys
    g = torch.Generator().manual_seed(1)
    prompt = torch.randint(0, cfg["vocab_size"], (24,), generator=g)
    with torch.no_grad():
        out = model(prompt[None], use_cache=True)
        pkv = out.past_key_values
        logits = [out.logits[0, -1].numpy().copy()]
        ids = []
        for _ in range(6):
            t = int(np.argmax(logits[-1]))
            ids.append(t)
            out = model(torch.tensor([[t]]), past_key_values=pkv, use_cache=True)
            pkv = out.past_key_values
            logits.append(out.logits[0, -1].numpy().copy())
    np.savez_compressed(os.path.join(HERE, "qwen35_tiny.npz"), prompt=prompt.numpy().astype(np.uint32),
                        ids=np.array(ids, np.uint32), logits=np.stack(logits).astype(np.float32),
                        checkpoint_sha256=np.array(sha256(os.path.join(path, "model.safetensors"))),
                        config=np.array(json.dumps(cfg)))


def gdn():
    from transformers.models.qwen3_5 import modeling_qwen3_5 as M

    g = torch.Generator().manual_seed(7)
    B, T, H, d = 1, 70, 2, 64
    q = torch.randn(B, T, H, d, generator=g)
    k = torch.randn(B, T, H, d, generator=g)
    q = (q / q.norm(dim=-1, keepdim=True)).to(torch.bfloat16)
    k = (k / k.norm(dim=-1, keepdim=True)).to(torch.bfloat16)
    v = torch.randn(B, T, H, d, generator=g).to(torch.bfloat16)
    beta = torch.sigmoid(torch.randn(B, T, H, generator=g))
    logd = -5.0 * torch.rand(B, T, H, generator=g)
    S0 = torch.randn(B, H, d, d, generator=g) * 0.1
    # the transformers functions scale q by d^-0.5 internally; pre-scaling by sqrt(64) = 8 makes that exact
    args = (q.float() * 8.0, k.float(), v.float(), logd, beta)
    o_rec, s_rec = M.torch_recurrent_gated_delta_rule(*args, initial_state=S0.clone(), output_final_state=True)
    o_chk, s_chk = M.torch_chunk_gated_delta_rule(*args, chunk_size=64, initial_state=S0.clone(),
                                                  output_final_state=True)
    bits = lambda t: t.contiguous().view(torch.int16).numpy().view(np.uint16)  # noqa: E731
    np.savez_compressed(os.path.join(HERE, "gdn.npz"), q=bits(q), k=bits(k), v=bits(v), g=logd.numpy(),
                        beta=beta.numpy(), S0=S0.numpy(), o_recurrent=o_rec.numpy(), S_recurrent=s_rec.numpy(),
                        o_chunk=o_chk.numpy(), S_chunk=s_chk.numpy())


if __name__ == "__main__":
    tiny_model()
    gdn()
    print("wrote", sorted(f for f in os.listdir(HERE) if f.endswith(".npz")))
