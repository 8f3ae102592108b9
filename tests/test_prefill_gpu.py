"""Prefill on tcgen05 tensor cores: the projection GEMM (qb_gemm_bf16) against a
plain PyTorch fp32 reference of the same op, with the decode path's epilogue
roundings (dryft/engine/kernels/projection.py:13-83, down.py:8-35)."""
import pytest
import torch

pytestmark = pytest.mark.gpu
BF16 = torch.bfloat16
DEV = "cuda:0"


def _gemm(x, w, epilogue=0, residual=None):
    from hackthenorth_b200 import _lib

    L = _lib.load()
    T, K = x.shape
    N = w.shape[0]
    out = torch.empty(T, N // 2 if epilogue == 2 else N, dtype=BF16, device=DEV)
    scratch = torch.zeros(L.qb_op_scratch_bytes(), dtype=torch.uint8, device=DEV)
    _lib.check(L.qb_gemm_bf16(x.data_ptr(), w.data_ptr(), out.data_ptr(),
                              residual.data_ptr() if residual is not None else None, T, N, K, epilogue,
                              scratch.data_ptr(), _lib.stream_handle()))
    _lib.check(L.qb_op_check(scratch.data_ptr(), _lib.stream_handle()))
    return out


def _spacing(ref):
    """bf16 spacing (one ulp) at |ref|."""
    ref = ref.float()
    return torch.where(ref == 0, torch.full_like(ref, 2.0 ** -133), 2.0 ** (torch.floor(torch.log2(ref.abs())) - 7))


def _ulps(got, ref):
    """|got - ref| in units of ref's bf16 spacing."""
    return (got.float() - ref.float()).abs() / _spacing(ref)


@pytest.mark.parametrize("T,N,K", [(128, 256, 64), (128, 256, 4096), (200, 512, 1024), (1000, 6144, 4096),
                                   (4096, 1024, 12288), (37, 2048, 512), (64, 128, 1024)])
def test_gemm_matches_fp32_reference(built_lib, T, N, K):
    g = torch.Generator(device=DEV).manual_seed(T * 7 + N + K)
    x = torch.randn(T, K, generator=g, device=DEV).to(BF16)
    w = (torch.randn(N, K, generator=g, device=DEV) * 0.02).to(BF16)
    ref = (x.float() @ w.float().T)
    out = _gemm(x, w)
    # fp32 sums in another order: within half a bf16 ulp of the reference plus
    # an accumulation bound proportional to sum |x_k w_k| (tight where a long
    # sum cancels to a small value, where a relative ulp test would not be)
    mag = x.float().abs() @ w.float().abs().T
    half_ulp = 0.5 * _spacing(ref)
    err = (out.float() - ref).abs()
    assert bool((err <= half_ulp + mag * 2.0 ** -16).all()), float((err - half_ulp - mag * 2.0 ** -16).max())
    assert float((_ulps(out, ref.to(BF16)) <= 1.0).float().mean()) >= 0.999


def test_gemm_residual_and_swiglu_epilogues(built_lib):
    from oracle.qwen3_oracle import swiglu

    g = torch.Generator(device=DEV).manual_seed(5)
    T, K, N = 300, 2048, 768
    x = torch.randn(T, K, generator=g, device=DEV).to(BF16)
    w = (torch.randn(N, K, generator=g, device=DEV) * 0.02).to(BF16)
    res = torch.randn(T, N, generator=g, device=DEV).to(BF16)
    y = (x.float() @ w.float().T).to(BF16)
    out = _gemm(x, w, 1, res)
    exp = (y.float() + res.float()).to(BF16)
    assert float((_ulps(out, exp) <= 2.0).float().mean()) >= 0.999
    out2 = _gemm(x, w, 2)
    gate, up = y[:, 0::2], y[:, 1::2]
    exp2 = swiglu(gate.cpu(), up.cpu()).to(DEV)
    assert float((_ulps(out2, exp2) <= 2.0).float().mean()) >= 0.999


def test_gemm_throughput_report(built_lib):
    """Gate/up-shaped prefill GEMM (4096 rows x 24576 x 4096): time it with CUDA
    events and report TFLOP/s (the assertion only guards against a collapse)."""
    T, N, K = 4096, 24576, 4096
    x = torch.randn(T, K, device=DEV).to(BF16)
    w = (torch.randn(N, K, device=DEV) * 0.02).to(BF16)
    for _ in range(2):
        _gemm(x, w)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(5):
        _gemm(x, w)
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / 5
    tflops = 2 * T * N * K / ms / 1e9
    print(f"prefill GEMM {T}x{N}x{K}: {ms:.3f} ms, {tflops:.1f} TFLOP/s")
    assert tflops > 50


LOGIT_ATOL = 0.0625


@pytest.mark.parametrize("shape,T", [("small", 64), ("small", 300), ("8b-layer", 64), ("8b-layer", 700)])
def test_batched_prefill_matches_oracle(built_lib, cpu_threads, shape, T):
    """Prompt rows as dense blocks (tcgen05 GEMMs + causal flash attention):
    last-row logits within LOGIT_ATOL of the oracle, the first token equal
    unless the oracle holds a near tie, every appended K/V row within bf16
    rounding, position = T."""
    import dataclasses

    from hackthenorth_b200.config import QWEN3_8B, QWEN3_SMALL
    from hackthenorth_b200.engine import Engine
    from hackthenorth_b200.weights import random_state_dict
    from oracle.qwen3_oracle import OracleQwen3

    cfg = QWEN3_SMALL if shape == "small" else dataclasses.replace(QWEN3_8B, n_layers=1)
    state = random_state_dict(cfg, 9)
    engine = Engine(None, DEV, cfg=cfg, state=state)
    prompt = torch.randint(0, cfg.vocab, (T,), generator=torch.Generator().manual_seed(T)).tolist()
    st = engine.new_state(T, 4, keep_logits=True)
    st.prefill(torch.tensor(prompt, device=DEV), batched=True)
    st.check()
    assert int(st.position.item()) == T
    o = OracleQwen3(cfg, state, st.capacity)
    ref, ref_tok = o.forward_rows(prompt, 0)
    last = ref[-1].float()
    d = (st.logits.float().cpu() - last).abs()
    assert d.max() <= LOGIT_ATOL and d.mean() <= 0.01, (float(d.max()), float(d.mean()))
    if st.read_token()[0] != int(ref_tok[-1]):
        top2 = last.topk(2).values
        assert float(top2[0] - top2[1]) <= LOGIT_ATOL
    for l in range(cfg.n_layers):
        torch.testing.assert_close(st.keys[l, :, :T].float().cpu(), o.keys[l, :, :T].float(), atol=0.0625, rtol=0.02)
        torch.testing.assert_close(st.values[l, :, :T].float().cpu(), o.values[l, :, :T].float(), atol=0.0625,
                                   rtol=0.02)


def test_batched_prefill_then_decode_matches_row_prefill(built_lib):
    """The same 200-token prompt prefilled as dense blocks and row by row: the
    same first token and 16 decode tokens (up to a near tie of the row path's
    logits), logits within LOGIT_ATOL."""
    from hackthenorth_b200.config import QWEN3_SMALL
    from hackthenorth_b200.engine import Engine

    engine = Engine.from_random(QWEN3_SMALL, seed=0)
    prompt = torch.randint(0, QWEN3_SMALL.vocab, (200,), generator=torch.Generator().manual_seed(4)).tolist()
    runs = {}
    for batched in (True, False):
        st = engine.new_state(len(prompt), 17, keep_logits=True)
        st.prefill(torch.tensor(prompt, device=DEV), batched=batched)
        toks, logits = st.read_token(), [st.logits.float().cpu().clone()]
        for _ in range(16):
            st.step()
            toks += st.read_token()
            logits.append(st.logits.float().cpu().clone())
        st.check()
        runs[batched] = (toks, torch.stack(logits))
    (ta, la), (tb, lb) = runs[True], runs[False]
    for i in range(len(ta)):
        assert (la[i] - lb[i]).abs().max() <= LOGIT_ATOL, f"step {i}"
        if ta[i] != tb[i]:
            top2 = lb[i].topk(2).values
            assert float(top2[0] - top2[1]) <= LOGIT_ATOL
            break
