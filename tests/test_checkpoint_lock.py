"""ensure_checkpoint from several processes at once (one per GPU in a multi-GPU bench): exactly one writes, every
caller returns a complete, identical checkpoint."""
import hashlib
import multiprocessing as mp
import os

from evie_b200 import checkpoint as ck


def _worker(path, q):
    cfg = ck.tiny_config(vocab_size=256, num_hidden_layers=4)
    ck.ensure_checkpoint(path, cfg, seed=3)
    with open(os.path.join(path, "model.safetensors"), "rb") as f:
        q.put(hashlib.sha256(f.read()).hexdigest())  # hash() is salted per process


def test_concurrent_writers_share_one_checkpoint(tmp_path):
    path = str(tmp_path / "ckpt")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(path, q)) for _ in range(3)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    digests = {q.get() for _ in procs}
    assert len(digests) == 1
    assert os.path.exists(os.path.join(path, "SYNTHETIC"))
