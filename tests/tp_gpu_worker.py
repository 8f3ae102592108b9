"""Worker for test_tp_gpu.py (launched by torchrun, one process per GPU): a
tensor-parallel Engine on seeded random weights decodes the golden prompt;
rank 0 writes the tokens to the path given on the command line.

With a third argument ``verify``: the speculative stream (verify passes with a
seeded synthetic draft of the golden continuation) and one 5-row verify pass
(predictions, the full logits gathered from the vocabulary shards, the rows'
K/V gathered from the head shards), written by rank 0 as .npz.

With ``prefill``: a seeded 300-row prompt through the tensor-parallel block
prefill (first token, last-row logits gathered from the vocabulary shards,
every prompt row's K/V gathered from the head shards) and the first token of
the same prompt run row by row, written by rank 0 as .npz."""
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
    mode = sys.argv[3] if len(sys.argv) > 3 else "decode"
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
    if mode in ("verify", "prefill"):
        if mode == "verify":
            verify_case(engine, cfg, prompt, g["tokens"].tolist(), out_path)
        else:
            prefill_case(engine, cfg, out_path)
        del engine
        torch.cuda.synchronize()
        dist.destroy_process_group()
        return
    toks = [s[0] for s in engine.generate([prompt], n_new, draft_tokens=0)]  # plain decode
    engine.state.check()
    # the default generate (prompt-lookup speculation, tensor-parallel verify)
    # with a fresh prompt state
    toks2 = [s[0] for s in engine.generate([prompt], n_new)]
    if dist.get_rank() == 0:
        with open(out_path, "w") as f:
            json.dump({"tokens": toks, "again": toks2}, f)
    del engine
    torch.cuda.synchronize()
    dist.destroy_process_group()


def _gather(t, dim):
    parts = [torch.empty_like(t) for _ in range(dist.get_world_size())]
    dist.all_gather(parts, t.contiguous())
    return torch.cat(parts, dim=dim)


PREFILL_ROWS = 300


def prefill_case(engine, cfg, out_path):
    dev = engine.device
    T = PREFILL_ROWS
    prompt = torch.randint(0, cfg.vocab, (T,), generator=torch.Generator().manual_seed(T))
    st = engine.new_state(T, 4, keep_logits=True)
    st.prefill(prompt.to(dev), batched=True)
    st.check()
    token = st.read_token()[0]
    position = int(st.position.item())
    logits = _gather(st.logits.reshape(1, -1), 1)[0]
    keys = _gather(st.keys[:, :, :T], 1)
    values = _gather(st.values[:, :, :T], 1)
    rows = engine.new_state(T, 4)
    rows.prefill(prompt.to(dev), batched=False)
    rows.check()
    token_rows = rows.read_token()[0]
    if dist.get_rank() == 0:
        np.savez(out_path, prompt=prompt.numpy(), token=token, token_rows=token_rows, position=position,
                 logits=logits.float().cpu().numpy(), keys=keys.float().cpu().numpy(),
                 values=values.float().cpu().numpy())


def verify_case(engine, cfg, prompt, gold, out_path):
    from hackthenorth_b200 import _lib
    from hackthenorth_b200.speculate import SyntheticDraft

    drafter = SyntheticDraft(gold, cfg.vocab, p=0.7, seed=3, draft_length=4)
    spec = [s[0] for s in engine.generate([prompt], len(gold), draft_tokens=4, drafter=drafter)]
    engine.state.check()
    # one verify pass: current token + 2 golden drafts + 2 seeded random drafts
    st = engine.new_state(len(prompt), 4, draft_tokens=8)
    st.prefill(torch.tensor(prompt, dtype=torch.int64, device=engine.device))
    current = st.read_token()[0]
    rng = torch.Generator().manual_seed(21)
    drafts = gold[1:3] + torch.randint(0, cfg.vocab, (2,), generator=rng).tolist()
    n = len(drafts) + 1
    dev = engine.device
    ids = torch.tensor([current, *drafts], dtype=torch.int64, device=dev)
    preds = torch.zeros(n, dtype=torch.int64, device=dev)
    logits = torch.zeros(n, cfg.vocab // engine.tp_size, dtype=torch.bfloat16, device=dev)
    L = _lib.load()
    _lib.check(L.qb_verify(engine.ctx, ids.data_ptr(), n, st.position.data_ptr(), preds.data_ptr(),
                           logits.data_ptr(), _lib.stream_handle()), engine.ctx)
    st.check()
    p0 = len(prompt)
    full = _gather(logits, 1)
    keys = _gather(st.keys[:, :, p0:p0 + n], 1)
    values = _gather(st.values[:, :, p0:p0 + n], 1)
    if dist.get_rank() == 0:
        np.savez(out_path, spec=np.array(spec), preds=preds.cpu().numpy(), current=current,
                 drafts=np.array(drafts), position=int(st.position.item()),
                 logits=full.float().cpu().numpy(), keys=keys.float().cpu().numpy(),
                 values=values.float().cpu().numpy())


if __name__ == "__main__":
    main()
