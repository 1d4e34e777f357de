"""Worker for the tensor-parallel decoder check (one process per GPU, NCCL).

Run as ``python -m torch.distributed.run --nproc-per-node N tests/tp_worker.py
OUT.json [batch] [p2p|nccl]``: every rank builds the same seeded weights, shards them, prefills a
prompt and decodes a few steps (eagerly and from a captured CUDA graph); rank 0
also runs the unsharded decoder on its GPU and writes the normwise logit
differences and token agreement to OUT.json.  Test infrastructure only.
"""

import datetime
import json
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

from xanosmerks_b200.llama import LlamaConfig, LlamaDecoder, LlamaWeights, synth_llama_weights  # noqa: E402


def rel(a, b):
    a, b = a.double(), b.double()
    return float((a - b).abs().max() / b.abs().max().clamp_min(1e-30))


def main():
    out_path = sys.argv[1]
    batch = int(sys.argv[2]) if len(sys.argv) > 2 else 2
    collective = sys.argv[3] if len(sys.argv) > 3 else "p2p"
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
    rank, world = dist.get_rank(), dist.get_world_size()
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", rank)))
    cfg = LlamaConfig(num_layers=2, vocab_size=4096)
    full = synth_llama_weights(cfg, seed=5, device="cuda")
    dec = LlamaDecoder(LlamaWeights.from_full(cfg, full, rank, world), batch=batch, max_ctx=64,
                       collective=collective)
    ref = LlamaDecoder(LlamaWeights.from_full(cfg, full), batch=batch, max_ctx=64) if rank == 0 else None
    ids = torch.from_numpy(np.random.default_rng(6).integers(0, cfg.vocab_size, size=(batch, 9)))
    report = {"world": world, "batch": batch, "collective": collective, "steps": []}

    def compare(tag):
        if rank == 0:
            report["steps"].append({"step": tag, "rel_err": rel(dec.logits, ref.logits),
                                    "same_tokens": bool(torch.equal(dec.next_ids, ref.next_ids))})

    dec.prefill(ids)
    if ref is not None:
        ref.prefill(ids)
    compare("prefill")
    # eager steps; the reference is fed the tensor-parallel decoder's tokens (teacher forcing)
    for s in range(2):
        if ref is not None:
            ref.next_ids.copy_(dec.next_ids)
        dec.decode_step()
        dec.length += 1
        if ref is not None:
            ref.decode_step()
            ref.length += 1
        compare(f"eager{s}")
    dec.capture()
    for s in range(3):
        if ref is not None:
            ref.next_ids.copy_(dec.next_ids)
        dec.replay(1)
        if ref is not None:
            ref.decode_step()
            ref.length += 1
        compare(f"graph{s}")
    torch.cuda.synchronize()
    # every rank must agree on the tokens (replicated head after the all-reduced residual stream)
    toks = [torch.zeros_like(dec.next_ids) for _ in range(world)]
    dist.all_gather(toks, dec.next_ids)
    report["ranks_agree"] = all(torch.equal(t, toks[0]) for t in toks)
    dec.close()   # releases the graph (it may hold NCCL calls) and the peer-memory buffers
    torch.cuda.synchronize()
    dist.barrier()
    if rank == 0:
        with open(out_path, "w") as f:
            json.dump(report, f)
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
