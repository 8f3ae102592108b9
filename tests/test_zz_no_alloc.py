"""The allocation-free attention entry point, checked against the ordinary one.

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


def _case(hq, hkv, cap, queries, first, seed):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(queries, hq, 128, generator=g).to(BF16).to(DEV)
    k = torch.randn(hkv, cap, 128, generator=g).to(BF16).to(DEV)
    v = torch.randn(hkv, cap, 128, generator=g).to(BF16).to(DEV)
    pos = torch.arange(first, first + queries, dtype=torch.int64, device=DEV)
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


@pytest.mark.parametrize("hq,hkv,cap,queries,first", [(32, 8, 4352, 1, 4095), (32, 8, 600, 5, 300),
                                                      (16, 8, 2048, 1, 2047)])
def test_noalloc_attention_matches_scratch_entry_point_twice(built_lib, hq, hkv, cap, queries, first):
    lib = built_lib
    status = torch.full((1,), -7, dtype=torch.int32, device=DEV)  # the call must clear it
    outs = []
    for call in range(2):  # two calls in a row share (and must reset) the static array
        q, k, v, pos = _case(hq, hkv, cap, queries, first - call, seed=40 + call)
        got = _noalloc(lib, q, k, v, pos, status)
        ref = _with_scratch(lib, q, k, v, pos)
        torch.cuda.synchronize()
        assert int(status.item()) == 0
        g, r = got.float().cpu(), ref.float().cpu()
        assert torch.isfinite(g).all()
        # same kernel; the split count may be smaller to fit the static array
        assert ((g - r).abs().max() / r.abs().max()).item() <= 1e-2
        outs.append(g)
    assert not torch.equal(outs[0], outs[1])


def test_noalloc_rejects_shapes_beyond_its_limits(built_lib):
    lib = built_lib
    q, k, v, pos = _case(32, 8, 64, 1, 10, seed=1)
    out = torch.empty_like(q)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    stream = torch.cuda.current_stream().cuda_stream
    # 9 query rows per call is above the entry point's maximum of 8
    rc = lib.qb_grouped_attention_noalloc(q.data_ptr(), k.data_ptr(), v.data_ptr(), 32, 8, 64, 9, pos.data_ptr(),
                                          out.data_ptr(), status.data_ptr(), stream)
    assert rc == 6 and b"queries" in lib.qb_last_error(None)
    rc = lib.qb_grouped_attention_noalloc(q.data_ptr(), k.data_ptr(), v.data_ptr(), 32, 8, 64, 1, None,
                                          out.data_ptr(), None, ctypes.c_void_p(stream))
    assert rc == 1
