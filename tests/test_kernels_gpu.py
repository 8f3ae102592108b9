"""GPU kernels through the C-ABI vs the CPU oracle (and fp32 SDPA for attention).

Tolerances: GEMV outputs are fp32-accumulated and rounded to bf16 once, like the
oracle, but the fp32 summation order differs, so an output may land one bf16
ulp away (|diff| <= 2^-7 |ref| + 1e-6 here) and only a small fraction may
differ at all. Attention: <= 1e-2 relative to fp32 SDPA.
Argmax ids must be exact (lowest index on ties). Cache writes of V are bit-exact.
"""
import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN

pytestmark = pytest.mark.gpu
BF16 = torch.bfloat16
DEV = "cuda:0"


def _close_bf16(out, ref, max_frac=0.05, rel=2 ** -7, scale=None):
    """``scale``: magnitude of an intermediate that was rounded before a final
    add (the projection before its residual); a one-ulp difference there is
    bounded by rel*|scale| even when the output itself is near zero."""
    out = out.detach().float().cpu().reshape(-1)
    ref = ref.detach().float().cpu().reshape(-1)
    assert torch.isfinite(out).all()
    diff = (out - ref).abs()
    mag = ref.abs() if scale is None else torch.maximum(ref.abs(), scale.detach().float().cpu().reshape(-1).abs())
    bound = rel * mag + 1e-6
    assert bool((diff <= bound).all()), f"max diff {diff.max().item()} (rel bound {rel})"
    frac = (out != ref).float().mean().item()
    assert frac <= max_frac, f"{frac:.3%} of outputs differ"


@pytest.fixture(scope="module", autouse=True)
def _lib_ready(built_lib):
    torch.manual_seed(1234)
    yield
    from hackthenorth_b200 import ops

    ops.check_device_errors(DEV)


@pytest.mark.parametrize("K,N", [(1024, 4096), (2560, 6144), (4096, 6144), (256, 96), (12288, 512), (384, 1024), (128, 300)])
def test_norm_projection_matches_oracle(K, N):
    from hackthenorth_b200 import ops
    from oracle.qwen3_oracle import norm_projection

    x = torch.randn(K).to(BF16)
    gain = torch.randn(K).to(BF16)
    w = (torch.randn(N, K) * 0.02).to(BF16)
    out = ops.norm_projection(x.to(DEV), gain.to(DEV), w.to(DEV))
    _close_bf16(out, norm_projection(x, gain, w, 1e-6))
    plain = ops.norm_projection(x.to(DEV), None, w.to(DEV))
    _close_bf16(plain, torch.nn.functional.linear(x[None], w)[0])


@pytest.mark.parametrize("K,F", [(1024, 3072), (2560, 9728), (4096, 12288 // 8)])
def test_gate_up_swiglu_matches_oracle(K, F):
    from hackthenorth_b200 import ops
    from hackthenorth_b200.weights import interleave_gate_up
    from oracle.qwen3_oracle import norm_projection

    x = torch.randn(K).to(BF16)
    gain = torch.randn(K).to(BF16)
    gate = (torch.randn(F, K) * 0.02).to(BF16)
    up = (torch.randn(F, K) * 0.02).to(BF16)
    out = ops.norm_projection(x.to(DEV), gain.to(DEV), interleave_gate_up(gate, up).to(DEV), swiglu=True)
    _close_bf16(out, norm_projection(x, gain, gate, 1e-6, swiglu_pair=up), max_frac=0.08, rel=2 ** -6)


def test_output_projection_halfway_rounding_known_answer():
    # dryft/tests/test_fused_kernels.py:179-187 (K padded to 256): exactly 0, not 1/256.
    from hackthenorth_b200 import ops

    x = torch.ones(256, dtype=BF16, device=DEV)
    w = torch.zeros(3, 256, dtype=BF16, device=DEV)
    w[:, 0] = 1
    w[:, 1] = 1 / 256
    res = -torch.ones(3, dtype=BF16, device=DEV)
    assert bool((ops.output_projection_residual(x, w, res) == 0).all())


@pytest.mark.parametrize("K,N", [(4096, 2560), (9728, 2560), (12288, 4096), (2048, 1024), (384, 1024)])
def test_projection_residual_matches_oracle(K, N):
    from hackthenorth_b200 import ops
    from oracle.qwen3_oracle import linear

    for scale in (0.0, 0.25, 4.0):
        x = (torch.randn(K) * scale).to(BF16)
        w = (torch.randn(N, K) * 0.02).to(BF16)
        res = torch.randn(N).to(BF16)
        out = ops.output_projection_residual(x.to(DEV), w.to(DEV), res.to(DEV))
        proj = linear(x[None], w)[0]
        _close_bf16(out, proj + res, max_frac=0.08, rel=2 ** -6, scale=proj)


def test_greedy_head_matches_oracle_and_breaks_ties_low():
    from hackthenorth_b200 import ops
    from oracle.qwen3_oracle import greedy_token, rms_norm

    V, K = 151936, 2560
    w = (torch.randn(V, K) * 0.02).to(BF16)
    wd = w.to(DEV)
    gain = torch.randn(K).to(BF16)
    for scale in (0.0, 1.0, 4.0):
        x = (torch.randn(K) * scale).to(BF16)
        tok, logits = ops.greedy_token(x.to(DEV), wd, gain.to(DEV), return_logits=True)
        tok = int(tok.item())
        ref_logits, _ = greedy_token(rms_norm(x[None], gain, 1e-6), w)
        ref_logits = ref_logits[0].float()
        lg = logits.float().cpu()
        assert tok == int(lg.argmax())  # first maximal index of its own logits
        _close_bf16(lg, ref_logits, max_frac=0.05)
        assert ref_logits[tok] >= ref_logits.max() - 2 ** -7 * ref_logits.abs().max()
    wz = torch.zeros(1000, 256, dtype=BF16, device=DEV)
    wz[3] = 1
    wz[-1] = 1
    assert int(ops.greedy_token(torch.ones(256, dtype=BF16, device=DEV), wz).item()) == 3


def _attn_case(hq, hkv, cap, queries, first, seed):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(queries, hq, 128, generator=g).to(BF16)
    k = torch.randn(hkv, cap, 128, generator=g).to(BF16)
    v = torch.randn(hkv, cap, 128, generator=g).to(BF16)
    pos = list(range(first, first + queries))
    return q, k, v, pos


@pytest.mark.parametrize("hq,hkv,cap,queries,first", [
    (32, 8, 129, 1, 128), (32, 8, 513, 4, 63), (32, 8, 257, 4, 126), (16, 8, 4096, 1, 4095),
    (32, 8, 4352, 5, 4000), (16, 8, 200, 5, 7), (32, 8, 32768, 1, 32767), (32, 8, 1000, 1, 0),
])
def test_grouped_attention_matches_oracle_and_sdpa(hq, hkv, cap, queries, first):
    from hackthenorth_b200 import ops
    from oracle.qwen3_oracle import grouped_attention, sdpa_reference

    q, k, v, pos = _attn_case(hq, hkv, cap, queries, first, seed=2)
    qd, kd, vd = q.to(DEV), k.to(DEV), v.to(DEV)
    pd = torch.tensor(pos, dtype=torch.int64, device=DEV)
    out = ops.grouped_attention(qd, kd, vd, pd).float().cpu()          # [Q, Hq, D]
    ref = sdpa_reference(q.transpose(0, 1), k, v, pos).transpose(0, 1)  # [Q, Hq, D]
    rel = ((out - ref).abs().max() / ref.abs().max()).item()
    assert rel <= 1e-2, rel
    if cap <= 4352:
        orc = grouped_attention(q.transpose(0, 1), k, v, pos).transpose(0, 1).float()
        assert ((out - orc).abs().max() / orc.abs().max()).item() <= 1e-2
    # Capacity past the last position must not be read, even when it is NaN.
    last = pos[-1]
    if last + 1 < cap:
        kd[:, last + 1:] = float("nan")
        vd[:, last + 1:] = float("nan")
        again = ops.grouped_attention(qd, kd, vd, pd).float().cpu()
        assert torch.equal(again, out)


def _sdpa_fp32_cuda(q, keys, values, positions):
    """fp32 attention in plain PyTorch on the GPU, per KV head: query row
    (i, head) sees keys 0..positions[i]; the same arithmetic as the reference's
    SDPA check (dryft/tests/test_fused_kernels.py:390-401) at sizes where the
    CPU restatement takes too long. q [Q, Hq, D]; keys/values [Hkv, cap, D]."""
    Qn, hq, d = q.shape
    hkv = keys.shape[0]
    G = hq // hkv
    n = int(positions[-1]) + 1
    out = torch.empty(Qn, hq, d, dtype=torch.float32, device=q.device)
    cols = torch.arange(n, device=q.device)
    mask = cols[None, :] <= positions[:, None]  # [Q, n]
    for h in range(hkv):
        qh = q[:, h * G:(h + 1) * G].float()                       # [Q, G, D]
        s = torch.einsum("qgd,kd->qgk", qh, keys[h, :n].float()) / d ** 0.5
        s = s.masked_fill(~mask[:, None, :], float("-inf"))
        out[:, h * G:(h + 1) * G] = torch.einsum("qgk,kd->qgd", torch.softmax(s, -1), values[h, :n].float())
    return out


@pytest.mark.parametrize("cap,queries", [(131072, 1), (131072, 5), (32768, 5)])
def test_grouped_attention_long_contexts_match_fp32(cap, queries):
    """The op sweep's long caches (GQA 32/8, D 128, N(0, 1) bf16 Q/K/V, query
    rows at the last positions): within 1e-2 relative of fp32 attention, and
    slots past the last position (NaN here) never read."""
    from hackthenorth_b200 import ops

    g = torch.Generator(device=DEV).manual_seed(2)
    q = torch.randn(queries, 32, 128, generator=g, device=DEV).to(BF16)
    k = torch.randn(8, cap + 64, 128, generator=g, device=DEV).to(BF16)
    v = torch.randn(8, cap + 64, 128, generator=g, device=DEV).to(BF16)
    pos = torch.arange(cap - queries, cap, dtype=torch.int64, device=DEV)
    k[:, cap:] = float("nan")
    v[:, cap:] = float("nan")
    out = ops.grouped_attention(q, k, v, pos).float()
    ref = _sdpa_fp32_cuda(q, k, v, pos)
    assert torch.isfinite(out).all()
    rel = ((out - ref).abs().max() / ref.abs().max()).item()
    assert rel <= 1e-2, rel


@pytest.mark.parametrize("hq,hkv,cap,queries,last", [(32, 8, 20000, 6, 19999), (16, 2, 30000, 3, 25000),
                                                     (8, 1, 17000, 3, 16990), (32, 8, 16384, 5, 9000),
                                                     (48, 12, 20000, 5, 19999)])
def test_grouped_attention_long_caches_many_rows_match_fp32(hq, hkv, cap, queries, last):
    """Long caches with 17..24 query rows per KV head run the rows kernel as
    several clusters per KV head, merged through the op scratch's partial rows
    and tickets (8, 2 and 1 KV heads; 24 rows; live keys well below the
    capacity; 12 KV heads, where no shape of several clusters may beat one
    cluster per head and the split kernel then runs with the op's split
    count): within 1e-2 relative of fp32 attention, slots past the last
    position (NaN here) never read, and a second call agrees (the merge
    tickets are left at zero)."""
    from hackthenorth_b200 import ops

    g = torch.Generator(device=DEV).manual_seed(hq + hkv + queries)
    q = torch.randn(queries, hq, 128, generator=g, device=DEV).to(BF16)
    k = torch.randn(hkv, cap, 128, generator=g, device=DEV).to(BF16)
    v = torch.randn(hkv, cap, 128, generator=g, device=DEV).to(BF16)
    pos = torch.arange(last - queries + 1, last + 1, dtype=torch.int64, device=DEV)
    k[:, last + 1:] = float("nan")
    v[:, last + 1:] = float("nan")
    ref = _sdpa_fp32_cuda(q, k, v, pos)
    first = None
    for _ in range(2):
        out = ops.grouped_attention(q, k, v, pos).float()
        assert torch.isfinite(out).all()
        rel = ((out - ref).abs().max() / ref.abs().max()).item()
        assert rel <= 1e-2, rel
        if first is None:
            first = out
        else:
            assert torch.equal(out, first)


def test_attention_matches_golden_sdpa():
    from hackthenorth_b200 import ops
    from tests.golden.make_golden import attention_inputs

    gold = np.load(os.path.join(GOLDEN, "attention_sdpa.npz"))
    for queries in (1, 5):
        q, k, v, pos = attention_inputs(512, queries)
        out = ops.grouped_attention(q.transpose(0, 1).contiguous().to(DEV), k.to(DEV), v.to(DEV),
                                    torch.tensor(pos, device=DEV)).float().cpu().transpose(0, 1)
        ref = torch.from_numpy(gold[f"q{queries}"])
        assert ((out - ref).abs().max() / ref.abs().max()).item() <= 1e-2


@pytest.mark.parametrize("hq,hkv,cap,position", [(32, 8, 41, 3), (32, 8, 41, 40), (16, 8, 4352, 4096),
                                                 (32, 8, 300, 0), (32, 8, 8192, 5000), (64, 8, 2048, 1500),
                                                 (4, 1, 20000, 17000), (32, 8, 33000, 32767), (8, 2, 600, 511)])
def test_rope_attention_matches_oracle_and_appends_cache(hq, hkv, cap, position):
    from hackthenorth_b200 import ops
    from hackthenorth_b200.config import ModelConfig
    from hackthenorth_b200.weights import rotary_table
    from oracle.qwen3_oracle import grouped_attention, norm_rope

    g = torch.Generator().manual_seed(111 + position)
    D = 128
    qkv = torch.randn((hq + 2 * hkv) * D, generator=g).to(BF16)
    qn = torch.randn(D, generator=g).to(BF16)
    kn = torch.randn(D, generator=g).to(BF16)
    keys = torch.randn(hkv, cap, D, generator=g).to(BF16)
    values = torch.randn(hkv, cap, D, generator=g).to(BF16)
    cfg = ModelConfig("t", hidden=1024, n_heads=hq, n_kv_heads=hkv, head_dim=D, ffn=1024, n_layers=1,
                      vocab=16, rope_theta=1e6)
    cos, sin = rotary_table(cfg, cap)
    kd, vd = keys.to(DEV), values.to(DEV)
    kd[:, position + 1:] = float("nan")
    vd[:, position + 1:] = float("nan")
    out = ops.rope_attention(qkv.to(DEV), qn.to(DEV), kn.to(DEV), cos.to(DEV), sin.to(DEV), kd, vd,
                             torch.tensor([position], device=DEV), n_heads=hq).float().cpu()
    q, k, v = qkv.split((hq * D, hkv * D, hkv * D))
    qr = norm_rope(q.view(hq, D), qn, 1e-6, cos[position], sin[position])
    kr = norm_rope(k.view(hkv, D), kn, 1e-6, cos[position], sin[position])
    ek, ev = keys.clone(), values.clone()
    ek[:, position] = kr
    ev[:, position] = v.view(hkv, D)
    ref = grouped_attention(qr[:, None], ek, ev, [position])[:, 0].float()
    assert ((out - ref).abs().max() / ref.abs().max()).item() <= 1e-2
    got_k = kd[:, position].float().cpu()
    assert torch.equal(vd[:, position].cpu(), ev[:, position])
    _close_bf16(got_k, kr.float(), max_frac=0.02)
    assert torch.equal(kd[:, :position].cpu(), keys[:, :position])
