"""The allocation-free decode entry point against the workspace one.

skv_decode_attention_noalloc serves callers that cannot allocate device memory
(bindings without a CUDA allocator, services that forbid allocation while
decoding): its scratch is a fixed array inside the library.  It must give the
same output and window mass as skv_decode_attention given a caller
workspace, call after call (the shared scratch keeps the previous call's
contents), and refuse requests larger than its scratch.
"""

import ctypes as C

import numpy as np
import pytest
import torch

from tests._helpers import OUT_TOL, make_cache, rand, rope_tables, to_np

pytestmark = pytest.mark.gpu


def _call(lib, fn, desc, st, q, out, scores, ws=None):
    stream = torch.cuda.current_stream().cuda_stream
    args = [C.byref(desc), st.T, st.tier_pages, q.data_ptr(), q.stride(0), q.stride(1),
            out.data_ptr(), out.stride(0), out.stride(1), C.c_float(q.shape[-1] ** -0.5),
            scores.data_ptr(), scores.shape[-1]]
    if ws is not None:
        args += [ws.data_ptr(), ws.numel()]
    return fn(*args, stream)


@pytest.mark.parametrize("dt,tier", [("f16", False), ("bf16", True)])
def test_noalloc_matches_workspace_entry_point_twice(dt, tier):
    from stickykv_b200 import _lib
    lib = _lib.lib()
    g = torch.Generator().manual_seed(11)
    B, Hkv, G, D, P = 3, 2, 4, 64, 411
    Hq = Hkv * G
    cos, sin = rope_tables(5e5, D, P + 64)
    cache = make_cache(dt, B, Hkv, Hq, D, P, 16, cos, sin, tier=tier)
    cache.update(rand((B, Hkv, P, D), dt, g).cuda(), rand((B, Hkv, P, D), dt, g).cuda(), 0)
    st = cache._states[0]
    W = -(-(P - 4) // 8)
    st.sides[st.cur].scores[:, :, :W] = torch.rand(B, Hq, W, generator=g).cuda()
    st.has_scores, st.W, st.next_window_id = True, W, W
    for _ in range(9):  # one eviction: with the tier this fills int4 pages
        k1 = rand((B, Hkv, 1, D), dt, g).cuda()
        cache.update(k1, k1.clone(), 0)
    assert (st.tier_pages > 0) == tier
    desc = cache._desc(st, st.sides[st.cur])
    nbytes = lib.skv_decode_workspace_size(C.byref(desc), st.T)
    assert 0 < nbytes <= _lib.NOALLOC_SCRATCH_BYTES
    ws = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    cap = st.scores_cap
    for call in range(2):
        q = rand((B, Hq, D), dt, g, scale=2.0).cuda()
        out_ref = torch.empty(B, Hq, D, dtype=q.dtype, device="cuda")
        out_na = torch.full_like(out_ref, float("nan"))
        sc_ref = torch.zeros(B, Hq, cap, device="cuda")
        sc_na = torch.zeros(B, Hq, cap, device="cuda")
        assert _call(lib, lib.skv_decode_attention, desc, st, q, out_ref, sc_ref, ws) == 0
        assert _call(lib, lib.skv_decode_attention_noalloc, desc, st, q, out_na, sc_na) == 0, \
            lib.skv_last_cuda_error()
        torch.cuda.synchronize()
        np.testing.assert_allclose(to_np(out_na), to_np(out_ref), atol=OUT_TOL[dt], rtol=0,
                                   err_msg=f"call {call}")
        np.testing.assert_allclose(to_np(sc_na), to_np(sc_ref), rtol=1e-5, atol=1e-7,
                                   err_msg=f"call {call}")
        assert to_np(sc_na)[:, :, :W].sum() > 0


def test_noalloc_rejects_requests_beyond_its_scratch():
    from stickykv_b200 import _lib
    lib = _lib.lib()
    d = _lib.LayerDesc()
    d.batch, d.num_kv_heads, d.num_q_heads, d.head_dim = 64, 8, 32, 64
    d.kv_dtype, d.window_size, d.num_sink, d.sink_pad = 0, 8, 4, 8
    d.fp_capacity = 1 << 16
    d.k_fp = d.v_fp = 256  # never dereferenced: the size check fails first
    T = 60000
    assert lib.skv_decode_workspace_size(C.byref(d), T) > _lib.NOALLOC_SCRATCH_BYTES
    q = torch.zeros(64, 32, 64, device="cuda")
    rc = lib.skv_decode_attention_noalloc(C.byref(d), T, 0, q.data_ptr(), q.stride(0), q.stride(1),
                                          q.data_ptr(), q.stride(0), q.stride(1), C.c_float(0.125),
                                          None, 0, torch.cuda.current_stream().cuda_stream)
    assert rc == 4  # SKV_ERR_CAPACITY


def test_noalloc_after_a_larger_call_matches_a_nan_filled_workspace():
    """The shared scratch keeps whatever the previous call left there: a call
    with more rows, splits and windows, then a smaller one whose result must
    equal the workspace entry point's given a workspace full of NaN (so any
    read of a byte the call did not write would show)."""
    from stickykv_b200 import _lib
    lib = _lib.lib()
    g = torch.Generator().manual_seed(12)
    D, G, Hkv = 64, 4, 2
    Hq = Hkv * G
    results = []
    for B, P in ((6, 3001), (2, 517)):
        cos, sin = rope_tables(5e5, D, P + 64)
        cache = make_cache("f16", B, Hkv, Hq, D, P, 16, cos, sin, tier=True)
        cache.update(rand((B, Hkv, P, D), "f16", g).cuda(), rand((B, Hkv, P, D), "f16", g).cuda(), 0)
        st = cache._states[0]
        W = -(-(P - 4) // 8)
        st.sides[st.cur].scores[:, :, :W] = torch.rand(B, Hq, W, generator=g).cuda()
        st.has_scores, st.W, st.next_window_id = True, W, W
        for _ in range(9):
            k1 = rand((B, Hkv, 1, D), "f16", g).cuda()
            cache.update(k1, k1.clone(), 0)
        if st.pending is not None:
            cache._flush(st)
        desc = cache._desc(st, st.sides[st.cur])
        q = rand((B, Hq, D), "f16", g, scale=2.0).cuda()
        cap = st.scores_cap
        out_na = torch.full((B, Hq, D), float("nan"), dtype=q.dtype, device="cuda")
        sc_na = torch.zeros(B, Hq, cap, device="cuda")
        assert _call(lib, lib.skv_decode_attention_noalloc, desc, st, q, out_na, sc_na) == 0, \
            lib.skv_last_cuda_error()
        nbytes = lib.skv_decode_workspace_size(C.byref(desc), st.T)
        ws = torch.full((nbytes // 4,), float("nan"), device="cuda").view(torch.uint8)
        out_ref = torch.empty_like(out_na)
        sc_ref = torch.zeros_like(sc_na)
        assert _call(lib, lib.skv_decode_attention, desc, st, q, out_ref, sc_ref, ws) == 0
        torch.cuda.synchronize()
        results.append((to_np(out_na), to_np(out_ref), to_np(sc_na), to_np(sc_ref)))
    for i, (a, b, sa, sb) in enumerate(results):
        assert np.isfinite(a).all() and np.isfinite(sa).all(), f"call {i}"
        np.testing.assert_array_equal(a, b, err_msg=f"call {i}")
        np.testing.assert_array_equal(sa, sb, err_msg=f"call {i}")
