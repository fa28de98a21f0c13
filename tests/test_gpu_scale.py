"""GPU parity at the benchmarked geometries and on tie-heavy scores.

* Decode attention at the isolated decode-attention geometry that bench.py
  times (16 rows, 32 query / 8 kv heads, head_dim 64, fp16, budget 0.40 of
  4k/8k/16k/32k context, int4 tier) in its steady state after the first
  eviction, one step through the fused append: every row's output and window
  mass against the oracle on the cache's own contents (all splits and their
  merge are exercised).
* The isolated evict + re-rotate geometry (16 rows, 8 kv heads, bf16, 16384
  tokens, budget 0.40, int4 tier): after the first eviction every row's kept
  windows, re-rotated fp keys, values, int4 codes, scales and zeros, window
  scores and ids are bit-exact against the oracle.
* Ties: window scores drawn from a handful of values so that many windows tie
  at the top-k threshold; the kept windows must follow the lowest-index rule
  (reference policy.py:112-138 with ties fixed to the lowest index) bit for
  bit across several evictions.
"""

import math

import numpy as np
import pytest
import torch

from oracle import skv_oracle as O
from tests._helpers import (TORCH_DT, assert_out_close, fp_parts, make_cache, rand, rope_tables,
                            tier_codes_all, to_np)

pytestmark = pytest.mark.gpu
DEV = "cuda"


def setup_module(module):
    assert torch.cuda.is_available(), "GPU tests need CUDA"
    from stickykv_b200 import _lib
    _lib.lib()


def _steady_cache(ctx, B=16, Hkv=8, Hq=32, D=64, dt="f16", seed=1):
    """The bench's steady state: prefill ctx tokens, random accumulated
    scores, nine decode steps of which the ninth evicts."""
    g = torch.Generator(device=DEV).manual_seed(seed)
    cos, sin = rope_tables(5e5, D, ctx + 128)
    cache = make_cache(dt, B, Hkv, Hq, D, ctx, 0, cos, sin, tier=True)
    tdt = TORCH_DT[dt]
    k = torch.randn(B, Hkv, ctx, D, device=DEV, generator=g, dtype=tdt)
    v = torch.randn(B, Hkv, ctx, D, device=DEV, generator=g, dtype=tdt)
    cache.update(k, v, 0)
    del k, v
    st = cache._states[0]
    W = math.ceil((ctx - 4) / 8)
    st.sides[st.cur].scores[:, :, :W] = torch.rand(B, Hq, W, device=DEV, generator=g)
    st.has_scores, st.W, st.next_window_id = True, W, W
    q = torch.randn(B, Hq, 1, D, device=DEV, generator=g, dtype=tdt)
    for _ in range(9):
        kn = torch.randn(B, Hkv, 1, D, device=DEV, generator=g, dtype=tdt)
        cache.update(kn, kn.clone(), 0)
        cache.decode_attention(0, q, D ** -0.5)
    torch.cuda.synchronize()
    return cache, cos, sin, g


@pytest.mark.parametrize("ctx", [4096, 8192, 16384, 32768])
def test_bench_geometry_decode_matches_oracle(ctx):
    B, Hkv, Hq, D = 16, 8, 32, 64
    cache, cos, sin, g = _steady_cache(ctx)
    st = cache._states[0]
    r = cache.resolved
    # the steady state the bench times: every kept evictable window in the tier
    assert st.tier_pages * 8 == r.top_k_windows * r.window_size
    kn = torch.randn(B, Hkv, 1, D, device=DEV, generator=g, dtype=torch.float16)
    vn = torch.randn(B, Hkv, 1, D, device=DEV, generator=g, dtype=torch.float16)
    q = torch.randn(B, Hq, 1, D, device=DEV, generator=g, dtype=torch.float16)
    cache.update(kn, vn, 0)
    assert st.pending is not None  # this step's append is fused into the decode launch
    W = math.ceil((st.T - 4) / 8)
    before = to_np(st.sides[st.cur].scores[:, :, :W])
    out = cache.decode_attention(0, q, D ** -0.5)
    torch.cuda.synchronize()
    mass = to_np(st.sides[st.cur].scores[:, :, :W]) - before
    sk, sv, rk, rv = fp_parts(cache)
    np.testing.assert_array_equal(rk[:, :, -1], to_np(kn[:, :, 0]))
    np.testing.assert_array_equal(rv[:, :, -1], to_np(vn[:, :, 0]))
    kc, ks, kz, vc, vs, vz = tier_codes_all(cache)
    tk = O.dequant_group32(kc, ks, kz)
    tv = O.dequant_group32(vc, vs, vz)
    qn = to_np(q[:, :, 0])
    got = to_np(out[:, 0])
    for b0 in range(0, B, 4):  # every row, four at a time
        sl = slice(b0, b0 + 4)
        ref_out, ref_mass = O.tiered_decode_attention_grouped(
            qn[sl], sk[sl], sv[sl], tk[sl], tv[sl], rk[sl], rv[sl], 4, 8, D ** -0.5, cos, sin)
        assert_out_close(got[sl], ref_out, "f16", f"ctx {ctx} rows {b0}-{b0 + 3}")
        np.testing.assert_allclose(mass[sl], ref_mass, rtol=5e-3, atol=1e-6,
                                   err_msg=f"ctx {ctx} rows {b0}-{b0 + 3}")
    # the whole softmax: window mass plus the sinks' share is one per head
    assert np.all(mass.sum(-1) <= 1 + 1e-3)


def test_cfg3_first_eviction_bit_exact_on_every_row():
    dt, B, Hkv, Hq, D, P = "bf16", 16, 8, 32, 64, 16384
    g = torch.Generator().manual_seed(2)
    cos, sin = rope_tables(5e5, D, P + 64)
    cache = make_cache(dt, B, Hkv, Hq, D, P, 0, cos, sin, tier=True)
    r = cache.resolved
    assert (r.top_k_windows, r.local_tokens) == (613, 1640)
    oc = O.OracleCache(O.resolve(8, 4, 0.25, 0.4, P, Hkv, D, 2, 0), dt, cos, sin, tier=True)
    k, v = rand((B, Hkv, P, D), dt, g), rand((B, Hkv, P, D), dt, g)
    cache.update(k.to(DEV), v.to(DEV), 0)
    oc.update(to_np(k), to_np(v), None)
    del k, v
    st = cache._states[0]
    W = math.ceil((P - 4) / 8)
    scores = torch.rand(B, Hq, W, generator=g)
    st.sides[st.cur].scores[:, :, :W] = scores.to(DEV)
    st.has_scores, st.W, st.next_window_id = True, W, W
    oc.add_scores(to_np(scores))
    for t in range(9):
        k1, v1 = rand((B, Hkv, 1, D), dt, g), rand((B, Hkv, 1, D), dt, g)
        cache.update(k1.to(DEV), v1.to(DEV), 0)
        evicted = oc.update(to_np(k1), to_np(v1), None)
        assert evicted == (t == 8)
    torch.cuda.synchronize()
    assert cache.get_seq_length(0) == oc.seq_length == 6548
    assert st.tier_pages * 8 == oc.n_tier_tokens == 613 * 8
    np.testing.assert_array_equal(to_np(st.original_window_ids), oc.original_window_ids)
    np.testing.assert_array_equal(to_np(st.window_scores), oc.window_scores)
    sk, sv, rk, rv = fp_parts(cache)
    np.testing.assert_array_equal(sk, oc.k[:, :, :4])
    np.testing.assert_array_equal(sv, oc.v[:, :, :4])
    np.testing.assert_array_equal(rk, oc.k[:, :, 4:])
    np.testing.assert_array_equal(rv, oc.v[:, :, 4:])
    names = ("k codes", "k scales", "k zeros", "v codes", "v scales", "v zeros")
    for name, a, b in zip(names, tier_codes_all(cache), oc.tier_codes):
        np.testing.assert_array_equal(a, b, err_msg=name)


def _tie_scores(rng, B, Hq, W, levels, all_equal=False):
    """Scores identical across heads (the head mean is then exact) taking one
    of a few dyadic levels per window: sums stay exact, ties stay ties."""
    if all_equal:
        per_w = np.full((B, W), 0.5, np.float32)
    else:
        per_w = rng.choice(np.asarray(levels, np.float32), size=(B, W))
    return np.ascontiguousarray(np.broadcast_to(per_w[:, None, :], (B, Hq, W)))


@pytest.mark.parametrize("dt,tier,all_equal", [("f16", True, False), ("bf16", False, False),
                                                ("bf16", True, True), ("f32", False, False)])
def test_tied_scores_keep_lowest_window_index(dt, tier, all_equal):
    B, Hkv, Hq, D, P, steps = 4, 2, 8, 64, 1203, 25
    g = torch.Generator().manual_seed(21)
    rng = np.random.default_rng(21)
    cos, sin = rope_tables(5e5, D, P + steps + 64)
    cache = make_cache(dt, B, Hkv, Hq, D, P, steps, cos, sin, tier=tier)
    r = cache.resolved
    oc = O.OracleCache(O.resolve(8, 4, 0.25, 0.4, P, Hkv, D, O.DTYPE_SIZES[dt], steps), dt, cos, sin, tier=tier)
    k, v = rand((B, Hkv, P, D), dt, g), rand((B, Hkv, P, D), dt, g)
    cache.update(k.to(DEV), v.to(DEV), 0)
    oc.update(to_np(k), to_np(v), None)
    levels = (0.25, 0.5, 0.75)
    sc = _tie_scores(rng, B, Hq, math.ceil((P - 4) / 8), levels, all_equal)
    n_evict = 0
    for t in range(steps):
        k1, v1 = rand((B, Hkv, 1, D), dt, g), rand((B, Hkv, 1, D), dt, g)
        cache.update(k1.to(DEV), v1.to(DEV), 0, cache_kwargs={"window_scores": torch.from_numpy(sc).to(DEV)})
        evicted = oc.update(to_np(k1), to_np(v1), sc)
        st = cache._states[0]
        assert cache.get_seq_length(0) == oc.seq_length
        if evicted:
            n_evict += 1
            W = oc.last_retained.shape[1]
            np.testing.assert_array_equal(to_np(st.original_window_ids), oc.original_window_ids,
                                          err_msg=f"eviction {n_evict}")
            np.testing.assert_array_equal(to_np(st.window_scores), oc.window_scores)
            if tier:
                for a, b in zip(tier_codes_all(cache), oc.tier_codes):
                    np.testing.assert_array_equal(a, b)
                sk, sv, rk, rv = fp_parts(cache)
                np.testing.assert_array_equal(rk, oc.k[:, :, 4:])
                np.testing.assert_array_equal(rv, oc.v[:, :, 4:])
            else:
                np.testing.assert_array_equal(to_np(st.key_states), oc.k)
                np.testing.assert_array_equal(to_np(st.value_states), oc.v)
            assert W == r.top_k_windows + cache.local_windows
        n = math.ceil((cache.get_seq_length(0) - 4) / 8)
        sc = _tie_scores(rng, B, Hq, n, levels, all_equal)
    assert n_evict == (steps - 1) // 8

