"""One rank of a tensor-parallel run (launched by torch.distributed.run).

    python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 \
        --master-port P tests/tp_worker.py MODEL.gguf OUT.npz PROMPT_LEN STEPS [SEED [fp16]]

Every rank opens the model with its slice on GPU `rank`, exchanges its
exchange-area handle through a gloo process group, prefills a seeded random
prompt and generates STEPS - 1 greedy tokens (with a binary16 KV cache when
the last argument is fp16). Rank 0 writes the picks, the
prompt's last logits (all ranks' vocab slices put together) and the device
time per decode step to OUT.npz.
"""
import datetime
import os
import sys

import numpy as np
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "-1.7-atlas---apollo_b200", "python"))
import atlas_cuda  # noqa: E402


def main():
    path, out = sys.argv[1], sys.argv[2]
    n_prompt, steps = int(sys.argv[3]), int(sys.argv[4])
    seed = int(sys.argv[5]) if len(sys.argv) > 5 else 5
    kv_fp16 = len(sys.argv) > 6 and sys.argv[6] == "fp16"
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=120))
    rt = atlas_cuda.Runtime(path, device=int(os.environ.get("LOCAL_RANK", rank)), max_context=n_prompt + steps + 8,
                            tp_rank=rank, tp_size=world, kv_fp16=kv_fp16)
    vocab = rt.vocab
    prompt = np.random.default_rng(seed).integers(0, vocab, n_prompt).astype(np.uint32)
    atlas_cuda.connect_tp(rt)
    dist.barrier()
    logits, first = rt.prefill(prompt)
    picks = rt.generate(first, n_prompt, steps - 1)
    sl = rt.tp_slice()
    mine = logits[sl.vocab_row0:sl.vocab_row0 + sl.vocab_rows].copy()
    dec_ms = rt.stats()[1] / max(1, steps - 1)
    gathered = [None] * world
    dist.all_gather_object(gathered, (sl.vocab_row0, mine, np.concatenate([[first], picks]).astype(np.uint32), dec_ms))
    dist.barrier()
    rt.close()
    if rank == 0:
        full = np.zeros(vocab, np.float32)
        for r0, part, _, _ in gathered:
            full[r0:r0 + part.size] = part
        all_picks = np.stack([g[2] for g in gathered])
        np.savez(out, prompt=prompt, logits=full, picks=all_picks, ms=np.array([g[3] for g in gathered]))
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
