"""GPU test of icua_greedy_head_noalloc, the greedy head for callers that cannot allocate device
memory (hosts that own all device memory through their own pool, plugins that may not call
cudaMalloc after start-up, real-time loops that must stay out of the allocator).

The entry point keeps its per-CTA argmax partials in a fixed device array of the library instead
of caller scratch.  This test (kept last in collection order so that a stop-at-first-failure run
has already run every other test) compares it with icua_greedy_head, which takes caller scratch,
on the same inputs for two calls in a row: the token must be identical and the logits equal
within the GEMV tolerance of the kernel tests (here they are bit-identical: same kernels).
It passes alone in a fresh process and after the other tests.
"""
import ctypes as C

import numpy as np
import pytest

from instantcua_b200 import _lib as L
from instantcua_b200 import model

pytestmark = pytest.mark.gpu
GEMV_TOL = 1e-5


def test_noalloc_greedy_head_matches_allocating_entry_point(require_gpu):
    import torch

    vocab, k = 151936, 2048
    rng = np.random.default_rng(77)
    w = (rng.standard_normal((vocab, k), dtype=np.float32) * 0.02).astype(np.float32)
    codes, scales = model.quantize_q8(w)
    buf = np.empty(L.lib().icua_packed_bytes(L.FMT_Q8, vocab, k), np.uint8)
    L.check(L.lib().icua_pack_matrix(L.FMT_Q8, vocab, k, codes.ctypes.data, scales.ctypes.data, buf.ctypes.data))
    emb = torch.from_numpy(buf).cuda()
    norm = torch.from_numpy((1 + 0.1 * rng.standard_normal(k)).astype(np.float32)).cuda()
    scratch = torch.empty(L.lib().icua_greedy_head_scratch_bytes(vocab), dtype=torch.uint8, device="cuda")
    lib = L.lib()
    for call in range(2):
        x = torch.from_numpy(rng.standard_normal(k).astype(np.float32) * 2).cuda()
        la = torch.empty(vocab, device="cuda")
        lb = torch.empty(vocab, device="cuda")
        ta = torch.full((1,), -1, dtype=torch.int32, device="cuda")
        tb = torch.full((1,), -2, dtype=torch.int32, device="cuda")
        L.check(lib.icua_greedy_head(vocab, C.c_void_p(emb.data_ptr()), C.c_void_p(x.data_ptr()),
                                     C.c_void_p(norm.data_ptr()), C.c_void_p(la.data_ptr()),
                                     C.c_void_p(ta.data_ptr()), C.c_void_p(scratch.data_ptr()), None))
        L.check(lib.icua_greedy_head_noalloc(vocab, C.c_void_p(emb.data_ptr()), C.c_void_p(x.data_ptr()),
                                             C.c_void_p(norm.data_ptr()), C.c_void_p(lb.data_ptr()),
                                             C.c_void_p(tb.data_ptr()), None))
        torch.cuda.synchronize()
        a, b = la.cpu().numpy(), lb.cpu().numpy()
        assert int(ta.item()) == int(tb.item()) == int(np.argmax(a)), call
        assert np.abs(a - b).max() <= GEMV_TOL * np.abs(a).max(), call
    # no finite logit: both entry points report -1 rather than an id a caller could index with
    x = torch.full((k,), float("nan"), device="cuda")
    ta = torch.zeros((1,), dtype=torch.int32, device="cuda")
    tb = torch.zeros((1,), dtype=torch.int32, device="cuda")
    L.check(lib.icua_greedy_head(vocab, C.c_void_p(emb.data_ptr()), C.c_void_p(x.data_ptr()),
                                 C.c_void_p(norm.data_ptr()), None, C.c_void_p(ta.data_ptr()),
                                 C.c_void_p(scratch.data_ptr()), None))
    L.check(lib.icua_greedy_head_noalloc(vocab, C.c_void_p(emb.data_ptr()), C.c_void_p(x.data_ptr()),
                                         C.c_void_p(norm.data_ptr()), None, C.c_void_p(tb.data_ptr()), None))
    torch.cuda.synchronize()
    assert int(ta.item()) == int(tb.item()) == -1
