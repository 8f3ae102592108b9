"""The allocation-free attention entry point, checked against the ordinary one
and against fp32 SDPA.

``qb_grouped_attention_noalloc`` exists for callers that cannot let this
library allocate device memory: hosts that give out GPU memory only from pools
they sized at start-up, or that run under a fixed memory limit. It keeps its
split-KV partials in a static device array inside libqb.so instead of a
caller-provided scratch buffer. This file is named so pytest collects it last;
it must also pass when run on its own in a fresh process.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu
BF16 = torch.bfloat16
DEV = "cuda:0"
QB_ERR_UNSUPPORTED = 6


def _case(hq, hkv, cap, queries, first, seed):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(queries, hq, 128, generator=g).to(BF16)
    k = torch.randn(hkv, cap, 128, generator=g).to(BF16)
    v = torch.randn(hkv, cap, 128, generator=g).to(BF16)
    pos = list(range(first, first + queries))
    return q, k, v, pos


def _noalloc(lib, q, k, v, pos, status):
    out = torch.empty_like(q)
    stream = torch.cuda.current_stream().cuda_stream
    rc = lib.qb_grouped_attention_noalloc(q.data_ptr(), k.data_ptr(), v.data_ptr(), q.shape[1], k.shape[0],
                                          k.shape[1], q.shape[0], pos.data_ptr(), out.data_ptr(),
                                          status.data_ptr(), stream)
    assert rc == 0, lib.qb_last_error(None)
    return out


def _with_scratch(lib, q, k, v, pos):
    out = torch.empty_like(q)
    n = int(lib.qb_op_scratch_bytes())
    scratch = torch.zeros(n, dtype=torch.uint8, device=DEV)
    rc = lib.qb_grouped_attention(q.data_ptr(), k.data_ptr(), v.data_ptr(), q.shape[1], k.shape[0], k.shape[1],
                                  q.shape[0], pos.data_ptr(), out.data_ptr(), scratch.data_ptr(), n,
                                  torch.cuda.current_stream().cuda_stream)
    assert rc == 0, lib.qb_last_error(None)
    return out


def _rel(a, b):
    return ((a - b).abs().max() / b.abs().max()).item()


# (32, 8, ...): the configurations' GQA shape. (128, 32, ..., 8) and
# (256, 64, ..., 8) have 32 query rows per KV head, so one split of partials
# takes 32 or 64 heads x 32 rows x 129 floats (0.5 / 1.0 MiB) and the split
# count is cut to what fits the 2 MiB array (3 and 1 instead of 4 and 2).
@pytest.mark.parametrize("hq,hkv,cap,queries,first", [(32, 8, 4352, 1, 4095), (32, 8, 600, 5, 300),
                                                      (16, 8, 2048, 1, 2047), (128, 32, 1500, 8, 1400),
                                                      (256, 64, 700, 8, 650)])
def test_noalloc_attention_matches_sdpa_and_scratch_entry_point_twice(built_lib, hq, hkv, cap, queries, first):
    from oracle.qwen3_oracle import sdpa_reference

    lib = built_lib
    status = torch.full((1,), -7, dtype=torch.int32, device=DEV)  # the call must clear it
    outs = []
    for call in range(2):  # two calls in a row share (and must reset) the static array
        q, k, v, pos = _case(hq, hkv, cap, queries, first - call, seed=40 + call)
        qd, kd, vd = q.to(DEV), k.to(DEV), v.to(DEV)
        pd = torch.tensor(pos, dtype=torch.int64, device=DEV)
        got = _noalloc(lib, qd, kd, vd, pd, status)
        ref = _with_scratch(lib, qd, kd, vd, pd)
        torch.cuda.synchronize()
        assert int(status.item()) == 0
        g, r = got.float().cpu(), ref.float().cpu()
        assert torch.isfinite(g).all()
        # the fp32 SDPA of the reference's attention test, within 1e-2 relative
        sdpa = sdpa_reference(q.transpose(0, 1), k, v, pos).transpose(0, 1)
        assert _rel(g, sdpa) <= 1e-2
        # the scratch entry point: same kernel, maybe another split count
        assert _rel(g, r) <= 1e-2
        outs.append(g)
    assert not torch.equal(outs[0], outs[1])


def test_noalloc_rejects_shapes_beyond_its_limits(built_lib):
    lib = built_lib
    q, k, v, pos = _case(32, 8, 64, 1, 10, seed=1)
    q, k, v = q.to(DEV), k.to(DEV), v.to(DEV)
    pos = torch.tensor(pos, dtype=torch.int64, device=DEV)
    out = torch.empty_like(q)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    stream = torch.cuda.current_stream().cuda_stream
    # 9 query rows per call is above the entry point's maximum of 8
    rc = lib.qb_grouped_attention_noalloc(q.data_ptr(), k.data_ptr(), v.data_ptr(), 32, 8, 64, 9, pos.data_ptr(),
                                          out.data_ptr(), status.data_ptr(), stream)
    assert rc == QB_ERR_UNSUPPORTED and b"queries" in lib.qb_last_error(None)
    # 65 KV heads: above the 64 the array is sized for (at 64 heads x 32 rows
    # one split needs 1.0 MiB, so every accepted shape fits at least one split)
    kk = torch.zeros(65, 64, 128, dtype=BF16, device=DEV)
    qq = torch.zeros(1, 65, 128, dtype=BF16, device=DEV)
    oo = torch.empty_like(qq)
    rc = lib.qb_grouped_attention_noalloc(qq.data_ptr(), kk.data_ptr(), kk.data_ptr(), 65, 65, 64, 1,
                                          pos.data_ptr(), oo.data_ptr(), status.data_ptr(), stream)
    assert rc == QB_ERR_UNSUPPORTED and b"KV heads" in lib.qb_last_error(None)
    # missing positions pointer: an argument error, nothing launched
    rc = lib.qb_grouped_attention_noalloc(q.data_ptr(), k.data_ptr(), v.data_ptr(), 32, 8, 64, 1, None,
                                          out.data_ptr(), None, ctypes.c_void_p(stream))
    assert rc == 1
    torch.cuda.synchronize()
    assert int(status.item()) == 0
