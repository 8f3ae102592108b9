"""Worker for test_tp_gpu.py (launched by torchrun, one process per GPU): a
tensor-parallel Engine on seeded random weights decodes the golden prompt;
rank 0 writes the tokens to the path given on the command line."""
import json
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def main():
    out_path, config = sys.argv[1], sys.argv[2]
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    import datetime

    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device(f"cuda:{local}"))
    from hackthenorth_b200 import tp
    from hackthenorth_b200.config import get_config
    from hackthenorth_b200.weights import random_state_dict
    from hackthenorth_b200.engine import Engine

    cfg = get_config(config)
    if config == "qwen3-small":
        g = np.load(os.path.join(ROOT, "tests", "golden", "qwen3_small_greedy.npz"))
        prompt, n_new = g["prompt"].tolist(), len(g["tokens"])
    else:
        with open(os.path.join(ROOT, "tests", "golden", "qwen3_0p6b_greedy.json")) as f:
            gj = json.load(f)
        prompt, n_new = gj["prompt"], 32
    uid = tp.shared_unique_id()
    state = random_state_dict(cfg, 0)  # CPU draw, identical on every rank and in the golden vectors
    engine = Engine(None, f"cuda:{local}", cfg=cfg, state=state, tp_rank=dist.get_rank(),
                    tp_size=dist.get_world_size(), unique_id=uid)
    toks = [s[0] for s in engine.generate([prompt], n_new)]
    engine.state.check()
    toks2 = [s[0] for s in engine.generate([prompt], n_new)]  # graph replay with a fresh prompt state
    if dist.get_rank() == 0:
        with open(out_path, "w") as f:
            json.dump({"tokens": toks, "again": toks2}, f)
    del engine
    torch.cuda.synchronize()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
