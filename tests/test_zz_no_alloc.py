"""The allocation-free attention entry point, called through the C ABI.

tqb200_dev_attention_decode_noalloc() serves callers that cannot allocate device
memory while they run (under a strict allocator, or with all device memory
reserved up front): its split-K scratch is a fixed device array.  This test checks
that two calls in a row, sharing that array, give the same output as the regular
attention entry point and as the oracle's attention_decode_ref restatement, within the
attention tolerance of the other tests (max relative error 1e-5).  The file is named so
that pytest collects it last."""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

import golden_cases as gc
from conftest import max_rel

pytestmark = pytest.mark.gpu


# (32, 8, 128) and (14, 2, 64) take the split kernel, whose partials live in the fixed
# array; head_dim 96 has no templated split kernel and takes the one-CTA-per-head kernel,
# which needs no scratch at all
@pytest.mark.parametrize("H,KVH,hd,seq,maxs", [(32, 8, 128, 300, 512), (14, 2, 64, 96, 128),
                                               (8, 2, 96, 40, 64)])
def test_no_alloc_attention_matches_regular_entry_point(tq, oracle, H, KVH, hd, seq, maxs):
    import torch
    torch.cuda.set_device(0)
    L = tq.load()
    scale = float(np.float32(1.0) / np.sqrt(np.float32(hd)))
    stream = torch.cuda.current_stream().cuda_stream
    for call in range(2):  # the second call runs on the scratch the first one left behind
        q, kc, vc = gc.attn_case(H, KVH, hd, seq + call, maxs)
        expected = tq.attention_decode(q, kc, vc, seq + call, maxs, H, KVH, hd, scale)
        assert max_rel(expected, oracle.attention(q, kc, vc, seq + call, maxs, H, KVH, hd,
                                                  scale)) < 1e-5
        dq, dk, dv = (torch.from_numpy(a).cuda() for a in (q, kc, vc))
        dout = torch.zeros(H * hd, device="cuda", dtype=torch.float32)
        st = L.tqb200_dev_attention_decode_noalloc(dq.data_ptr(), dk.data_ptr(), dv.data_ptr(),
                                                   seq + call, maxs, H, KVH, hd, C.c_float(scale),
                                                   dout.data_ptr(), stream)
        assert st == 0, L.tqb200_last_error()
        torch.cuda.synchronize()
        out = dout.cpu().numpy()
        assert max_rel(out, expected) < 1e-5
        assert max_rel(out, oracle.attention(q, kc, vc, seq + call, maxs, H, KVH, hd, scale)) < 1e-5


def test_no_alloc_attention_rejects_oversized_shapes(tq):
    L = tq.load()
    # 257 KV heads exceed the fixed ticket array: rejected before any device work (the
    # pointers are never dereferenced)
    p = 1 << 20
    st = L.tqb200_dev_attention_decode_noalloc(p, p, p, 1, 1, 257, 257, 64, C.c_float(1.0), p, None)
    assert st == 1 and b"fixed maximum" in L.tqb200_last_error()
