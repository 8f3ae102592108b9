"""The tensor-parallel reduction of the o-proj / down epilogue, on one GPU, and
a bounded device wait that runs out.

Rank 0 of a two-rank group runs through the C-ABI (qb_projection_residual_peer,
the op-level form of the fused o-proj / down sublayer under tensor
parallelism). Rank 1 is emulated on the host: its {token, fp32 partial} words
are written into rank 0's receive buffer before the call, and a plain device
buffer stands in for rank 1's receive words. No second kernel runs, so nothing
waits on anything that another launch would have to provide.

1. With rank 1's words in place, the output is exactly
   bf16(bf16(p0 + p1) + residual) (partials in rank order, as every rank of
   the engine computes it) and rank 0's own words reach both buffers.
2. Without them, rank 0's bounded wait (2 s) gives up: the kernel returns,
   qb_op_check reports QB_ERR_TIMEOUT, and the next call on the same device
   succeeds. This is the failure path of every peer, tagged-word and mbarrier
   wait in the library: record a site code in the error word, drain, return.
"""
import time

import pytest
import torch

pytestmark = pytest.mark.gpu
BF16 = torch.bfloat16
DEV = "cuda:0"


def _token(epoch, sublayer):
    return (epoch + 1) * 256 + sublayer + 1


def _words(token, partial):
    bits = partial.float().contiguous().view(torch.int32).to(torch.int64) & 0xFFFFFFFF
    return (token << 32) | bits


def _round_bf16(x):
    return x.to(BF16).float()


def _case(K=2048, N=1024, seed=3):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(2 * K, generator=g).to(BF16)
    w = (torch.randn(N, 2 * K, generator=g) * 0.02).to(BF16)
    res = torch.randn(N, generator=g).to(BF16)
    return x, w, res


@pytest.fixture(scope="module", autouse=True)
def _lib_ready(built_lib):
    yield


def test_peer_reduction_with_emulated_partner_is_exact():
    from hackthenorth_b200 import ops

    K, N = 2048, 1024
    x, w, res = _case(K, N)
    x0, x1 = x[:K].contiguous(), x[K:].contiguous()
    w0, w1 = w[:, :K].contiguous(), w[:, K:].contiguous()
    p1 = w1.float() @ x1.float()  # rank 1's fp32 partial, as the host computes it
    epoch, sub, parity = 5, 3, 1
    tok = _token(epoch, sub)
    recv0 = torch.zeros(2, 2, N, dtype=torch.int64, device=DEV)   # rank 0's receive words
    recv1 = torch.zeros(2, 2, N, dtype=torch.int64, device=DEV)   # stands in for rank 1's
    recv0[parity, 1] = _words(tok, p1).to(DEV)
    ep = torch.tensor([epoch], dtype=torch.int64, device=DEV)
    out = ops.projection_residual_peer(x0.to(DEV), w0.to(DEV), res.to(DEV), [recv0, recv1], rank=0, epoch=ep,
                                       sublayer=sub, parity=parity)
    ops.check_device_errors()
    sent = recv1[parity, 0].cpu()
    assert bool(((sent >> 32) == tok).all())
    assert torch.equal(recv0[parity, 0].cpu(), sent)  # the same words in its own buffer
    p0 = (sent & 0xFFFFFFFF).to(torch.int32).view(torch.float32)
    # rank 0's partial is its own fp32 sum (another order than the host's)
    torch.testing.assert_close(p0, w0.float() @ x0.float(), rtol=1e-4, atol=1e-4)
    # the epilogue: partials in rank order, one rounding, + residual, one rounding
    want = (_round_bf16((torch.zeros(N) + p0) + p1) + res.float()).to(BF16)
    assert torch.equal(out.cpu(), want)
    # and it is the unsharded projection + residual up to that summation order
    full = (_round_bf16(w.float() @ x.float()) + res.float()).to(BF16).float()
    d = (out.float().cpu() - full).abs()
    assert float(d.max()) <= 2 ** -7 * float(torch.maximum(full.abs(), (w.float() @ x.float()).abs()).max())


def test_bounded_peer_wait_gives_up_and_the_device_recovers():
    from hackthenorth_b200 import _lib, ops

    K, N = 2048, 1024
    x, w, res = _case(K, N, seed=4)
    x0, w0 = x[:K].contiguous().to(DEV), w[:, :K].contiguous().to(DEV)
    x1, w1 = x[K:].contiguous(), w[:, K:].contiguous()
    recv0 = torch.zeros(2, 2, N, dtype=torch.int64, device=DEV)
    recv1 = torch.zeros(2, 2, N, dtype=torch.int64, device=DEV)
    ep = torch.tensor([9], dtype=torch.int64, device=DEV)
    ops.check_device_errors()  # start from a clear error word
    t0 = time.perf_counter()
    ops.projection_residual_peer(x0, w0, res.to(DEV), [recv0, recv1], rank=0, epoch=ep, sublayer=0, parity=0)
    with pytest.raises(_lib.QbError) as err:
        ops.check_device_errors()  # nothing ever writes rank 1's words
    waited = time.perf_counter() - t0
    assert err.value.code == _lib.QB_ERR_TIMEOUT and "timed out" in str(err.value)
    assert 1.5 <= waited <= 60.0, waited
    # the context is usable: the next call (a new epoch, partner words present) completes
    ep.fill_(10)
    tok = _token(10, 0)
    p1 = w1.float() @ x1.float()
    recv0[0, 1] = _words(tok, p1).to(DEV)
    out = ops.projection_residual_peer(x0, w0, res.to(DEV), [recv0, recv1], rank=0, epoch=ep, sublayer=0, parity=0)
    ops.check_device_errors()
    p0 = (recv1[0, 0].cpu() & 0xFFFFFFFF).to(torch.int32).view(torch.float32)
    want = (_round_bf16((torch.zeros(N) + p0) + p1) + res.float()).to(BF16)
    assert torch.equal(out.cpu(), want)
    plain = ops.output_projection_residual(x0, w0, res.to(DEV))
    torch.cuda.synchronize()
    assert torch.isfinite(plain.float()).all()
