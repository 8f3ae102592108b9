"""Tensor-parallel host logic on the CPU: two gloo ranks run the sharded
restatement (oracle/tp_oracle.py) with the same shard layout as
hackthenorth_b200.weights.PackedWeights and fp32 partial sums all-reduced
before the single bf16 rounding; the result must match the unsharded oracle."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from conftest import ROOT

LOGIT_ATOL = 0.0625


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _tiny():
    from hackthenorth_b200.config import ModelConfig

    return ModelConfig("tiny-tp", hidden=256, n_heads=8, n_kv_heads=4, head_dim=128, ffn=512, n_layers=2,
                       vocab=96, rope_theta=1e6)


def _worker(rank, world, port, out_path):
    import sys

    sys.path.insert(0, ROOT)
    import torch.distributed as dist

    from hackthenorth_b200.weights import random_state_dict
    from oracle.tp_oracle import OracleQwen3TP

    torch.set_num_threads(1)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        cfg = _tiny()
        state = random_state_dict(cfg, 3)
        o = OracleQwen3TP(cfg, state, 40, rank, world)
        prompt = [5, 17, 29, 41, 53, 65, 77]
        logits, tok = o.forward_rows(prompt, 0)
        rows = [logits[-1]]
        toks = [int(tok[-1])]
        pos = len(prompt)
        for _ in range(5):
            lg, t = o.forward_rows([toks[-1]], pos)
            pos += 1
            rows.append(lg[0])
            toks.append(int(t[0]))
        # verify-style multi-row pass at the end (k+1 = 3 rows)
        lg3, t3 = o.forward_rows([toks[-1], 7, 8], pos)
        if rank == 0:
            torch.save({"rows": torch.stack(rows), "toks": toks, "verify": lg3}, out_path)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2])
def test_tensor_parallel_shards_match_unsharded_oracle(tmp_path, world, cpu_threads):
    from hackthenorth_b200.weights import random_state_dict
    from oracle.qwen3_oracle import OracleQwen3

    out = str(tmp_path / "tp.pt")
    mp.start_processes(_worker, args=(world, _free_port(), out), nprocs=world, start_method="spawn")
    got = torch.load(out)
    cfg = _tiny()
    ref = OracleQwen3(cfg, random_state_dict(cfg, 3), 40)
    prompt = [5, 17, 29, 41, 53, 65, 77]
    logits, tok = ref.forward_rows(prompt, 0)
    rows, toks, pos = [logits[-1]], [int(tok[-1])], len(prompt)
    for _ in range(5):
        lg, t = ref.forward_rows([toks[-1]], pos)
        pos += 1
        rows.append(lg[0])
        toks.append(int(t[0]))
    lg3, _ = ref.forward_rows([toks[-1], 7, 8], pos)
    assert got["toks"] == toks
    assert (got["rows"].float() - torch.stack(rows).float()).abs().max() <= LOGIT_ATOL
    assert (got["verify"].float() - lg3.float()).abs().max() <= LOGIT_ATOL


def test_packed_weights_shards_tile_the_full_matrices():
    from hackthenorth_b200.weights import PackedWeights, interleave_gate_up, random_state_dict

    cfg = _tiny()
    state = random_state_dict(cfg, 3)
    full = PackedWeights(cfg, state, "cpu")
    parts = [PackedWeights(cfg, state, "cpu", r, 2) for r in range(2)]
    D = cfg.head_dim
    for i in range(cfg.n_layers):
        p = f"model.layers.{i}."
        q, k, v = (state[p + f"self_attn.{n}_proj.weight"] for n in "qkv")
        for r, pw in enumerate(parts):
            hq, hkv = cfg.n_heads // 2, cfg.n_kv_heads // 2
            exp = torch.cat((q[r * hq * D:(r + 1) * hq * D], k[r * hkv * D:(r + 1) * hkv * D],
                             v[r * hkv * D:(r + 1) * hkv * D]))
            assert torch.equal(pw.layers[i]["qkv"], exp)
        assert torch.equal(torch.cat([pw.layers[i]["o"] for pw in parts], 1), full.layers[i]["o"])
        assert torch.equal(torch.cat([pw.layers[i]["down"] for pw in parts], 1), full.layers[i]["down"])
        g, u = state[p + "mlp.gate_proj.weight"], state[p + "mlp.up_proj.weight"]
        f = cfg.ffn // 2
        for r, pw in enumerate(parts):
            assert torch.equal(pw.layers[i]["gu"], interleave_gate_up(g[r * f:(r + 1) * f], u[r * f:(r + 1) * f]))
    assert torch.equal(torch.cat([pw.lm_head for pw in parts]), full.lm_head)
    with pytest.raises(ValueError):
        PackedWeights(cfg, state, "cpu", 0, 3)
