"""One rank of a tensor-parallel parity run (launched by torchrun from
test_gpu_tp.py): loads its share of the model, connects to the other ranks,
runs teacher-forced steps and a greedy decode, and rank 0 writes every
step's whole-vocabulary logits (assembled from the ranks' shares) and the
ids to a JSON file.

    torchrun --nproc-per-node N tests/tp_worker.py MODEL.gguf OUT.json
"""
import datetime
import json
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "ai-agent-framework_b200"))

import numpy as np  # noqa: E402
import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

import b2decode  # noqa: E402
from b2decode import tp  # noqa: E402
from b2decode import gguf_writer as gw  # noqa: E402


def tokens(vocab):
    return (np.concatenate([[1], gw.make_prompt(vocab, 70, seed=5), gw.make_prompt(vocab, 10, seed=6)]).astype(np.int32),
            71)


def main():
    path, out = sys.argv[1], sys.argv[2]
    rank, world, local = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"]), int(os.environ["LOCAL_RANK"])
    # a host channel for the handle exchange and the results (no NCCL needed)
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=120))
    try:
        torch.cuda.set_device(local)
        m = b2decode.Model(path, num_ctx=256, device=local, tp_size=world, tp_rank=rank)
        tp.connect(m)
        toks, npre = tokens(m.cfg["vocab_size"])
        steps = [m.forward(toks[:npre])] + [m.forward([t]) for t in toks[npre:]]
        m.reset()
        first = m.forward_argmax(toks[:npre])
        greedy = [first] + m.decode_greedy(first, 12).tolist()
        parts = [None] * world
        dist.all_gather_object(parts, (m.cfg["vocab_begin"], [s.tolist() for s in steps]))
        if rank == 0:
            full = []
            for k in range(len(steps)):
                full.append(np.concatenate([np.asarray(p[1][k], np.float32) for p in sorted(parts)]).tolist())
            with open(out, "w") as f:
                json.dump({"logits": full, "greedy": [int(x) for x in greedy], "status": m.device_status()}, f)
        m.close()
    finally:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
