"""GPU parity: the native kernels (called through the C ABI by the drop-in
cache) against the CPU oracle and the reference's golden vectors.

Bit-exact: kept windows, original ids, position map, re-rotated fp keys,
copied values, int4 codes/scales/page bytes.  Tolerance: attention outputs
against the oracle rounded to the KV dtype, max-abs per dtype in
_helpers.OUT_TOL (or one dtype ulp where that is larger; see
_helpers.assert_out_close); window mass to 1e-4 relative.
"""

import math
import os

import numpy as np
import pytest
import torch

from oracle import skv_oracle as O
from tests._helpers import (OUT_TOL, TORCH_DT, assert_out_close, fp_parts, make_cache, rand, rope_tables,
                            tier_codes, to_np)

pytestmark = pytest.mark.gpu
G = os.path.join(os.path.dirname(__file__), "golden")
DEV = "cuda"


def setup_module(module):
    assert torch.cuda.is_available(), "GPU tests need CUDA"
    from stickykv_b200 import _lib
    _lib.lib()


# -- full cache drive against the reference's own run ------------------------------------

@pytest.mark.parametrize("dt", ["f32", "bf16"])
def test_cache_drive_matches_reference_golden(dt):
    z = np.load(os.path.join(G, f"cache_drive_{dt}.npz"))
    B, Hkv, Hq, D, P, M = [int(x) for x in z["meta"]]
    cache = make_cache(dt, B, Hkv, Hq, D, P, M, z["cos"], z["sin"], local=0.25, budget=0.5)
    T = lambda a: torch.from_numpy(a).to(DEV, TORCH_DT[dt])
    cache.update(T(z["k_0"]), T(z["v_0"]), 0)
    for t in range(1, M + 1):
        cache.update(T(z[f"k_{t}"]), T(z[f"v_{t}"]), 0,
                     cache_kwargs={"window_scores": torch.from_numpy(z[f"s_{t - 1}"]).to(DEV)})
        assert cache.get_seq_length(0) == int(z[f"len_{t}"])
        np.testing.assert_array_equal(to_np(cache._states[0].original_window_ids), z[f"ids_{t}"])
    st = cache._states[0]
    np.testing.assert_array_equal(to_np(st.key_states), z["final_k"])
    np.testing.assert_array_equal(to_np(st.value_states), z["final_v"])
    np.testing.assert_allclose(to_np(st.window_scores), z["final_scores"], rtol=1e-6, atol=1e-7)
    assert to_np(st.position_ids).tolist() == z["final_pos"].tolist()


def test_divergent_eviction_kat_on_gpu():
    # reference tests/test_windowed_cache.py:643-724 (head_dim 16: the smallest
    # the kernels take; the KAT only reads which tokens survive)
    D = 16
    cos = np.ones((64, D), np.float32)
    sin = np.zeros((64, D), np.float32)
    rows = {}
    for B in (2, 1):
        cache = make_cache("f32", B, 2, 4, D, 8, 0, cos, sin, ws=1, s=0, local=1, budget=0.375)
        assert cache.resolved.top_k_windows == 2
        s0 = torch.zeros(B, 4, 8)
        s0[0, :, [1, 3]] = 100.0
        if B > 1:
            s0[1, :, [5, 7]] = 100.0
        keys = lambda n, a: torch.arange(a, a + n, dtype=torch.float32).view(1, 1, n, 1).expand(B, 2, n, D).contiguous().to(DEV)
        k = keys(8, 0)
        cache.update(k, k.clone(), 0, cache_kwargs={"window_scores": s0.to(DEV)})
        for i, pos in enumerate((8, 9)):
            k1 = keys(1, pos)
            cache.update(k1, k1.clone(), 0, cache_kwargs={"window_scores": torch.zeros(B, 4, 9 + i, device=DEV)})
        st = cache._states[0]
        rows[B] = st
        if B == 2:
            assert to_np(st.original_window_ids).tolist() == [[1, 3, 9], [5, 7, 9]]
            assert to_np(st.key_states[:, 0, :, 0]).tolist() == [[1.0, 3.0, 9.0], [5.0, 7.0, 9.0]]
            assert to_np(st.position_ids).tolist() == [[0, 1, 2], [0, 1, 2]]
    np.testing.assert_array_equal(to_np(rows[1].key_states[0]), to_np(rows[2].key_states[0]))


# -- decode attention ---------------------------------------------------------------------

@pytest.mark.parametrize("dt", ["f32", "f16"])
def test_decode_matches_reference_eager_golden(dt):
    z = np.load(os.path.join(G, f"eager_decode_{dt}.npz"))
    B, Hq, D = z["q"].shape
    Hkv, S = z["k"].shape[1], z["k"].shape[2]
    cos, sin = rope_tables(1e4, D, 256)
    cache = make_cache(dt, B, Hkv, Hq, D, S, 1, cos, sin)
    T = lambda a: torch.from_numpy(a).to(DEV, TORCH_DT[dt])
    cache.update(T(z["k"]), T(z["v"]), 0)
    st = cache._states[0]
    st.has_scores, st.W = True, 0
    out = cache.decode_attention(0, T(z["q"])[:, :, None, :], D ** -0.5)
    assert_out_close(to_np(out[:, 0]), z["out"], dt, "eager golden")
    np.testing.assert_allclose(to_np(st.window_scores), z["scores"], atol=OUT_TOL[dt], rtol=0)


@pytest.mark.parametrize("dt,D,G,S", [("f32", 64, 2, 300), ("f16", 64, 4, 1000), ("bf16", 128, 4, 777),
                                      ("f16", 128, 8, 64), ("bf16", 64, 1, 2049), ("f16", 32, 4, 5000),
                                      ("f16", 64, 2, 1500), ("bf16", 64, 8, 3001), ("f16", 128, 1, 900),
                                      ("f16", 64, 7, 1100), ("bf16", 128, 3, 600), ("f16", 64, 6, 2500),
                                      ("f32", 64, 7, 500), ("f32", 32, 3, 700), ("f16", 32, 5, 900)])
def test_decode_matches_oracle(dt, D, G, S):
    g = torch.Generator().manual_seed(S + D)
    B, Hkv = 3, 2
    Hq = Hkv * G
    cos, sin = rope_tables(5e5, D, S + 64)
    cache = make_cache(dt, B, Hkv, Hq, D, S, 1, cos, sin)
    k, v = rand((B, Hkv, S, D), dt, g), rand((B, Hkv, S, D), dt, g)
    q = rand((B, Hq, D), dt, g, scale=2.0)
    cache.update(k.to(DEV), v.to(DEV), 0)
    st = cache._states[0]
    before = to_np(st.sides[st.cur].scores[:, :, : math.ceil((S - 4) / 8)])
    out = cache.decode_attention(0, q.to(DEV)[:, :, None, :], D ** -0.5)
    ref_out, ref_mass = O.tiered_decode_attention(
        to_np(q), to_np(k)[:, :, :4], to_np(v)[:, :, :4], None, None, to_np(k)[:, :, 4:],
        to_np(v)[:, :, 4:], 4, 8, D ** -0.5)
    assert_out_close(to_np(out[:, 0]), ref_out, dt, "decode")
    mass = to_np(st.window_scores) - before
    np.testing.assert_allclose(mass, ref_mass, rtol=1e-4, atol=1e-6)
    # the mass of all windows plus the sinks is the whole softmax
    assert np.all(mass.sum(-1) <= 1 + 1e-4)


@pytest.mark.parametrize("dt,ws,G", [("f16", 16, 4), ("bf16", 32, 8), ("f16", 24, 2)])
def test_decode_window_sizes_match_oracle(dt, ws, G):
    """Windows of several 8-token units on the tensor-core path: the kernel
    keeps the mass of every unit, the merge sums a window's units."""
    g = torch.Generator().manual_seed(ws + G)
    B, Hkv, D, S = 2, 2, 64, 1203
    Hq = Hkv * G
    cos, sin = rope_tables(5e5, D, S + 64)
    cache = make_cache(dt, B, Hkv, Hq, D, S, 1, cos, sin, ws=ws)
    k, v = rand((B, Hkv, S, D), dt, g), rand((B, Hkv, S, D), dt, g)
    q = rand((B, Hq, D), dt, g, scale=2.0)
    cache.update(k.to(DEV), v.to(DEV), 0)
    st = cache._states[0]
    nw = math.ceil((S - 4) / ws)
    before = to_np(st.sides[st.cur].scores[:, :, :nw])
    out = cache.decode_attention(0, q.to(DEV)[:, :, None, :], D ** -0.5)
    ref_out, ref_mass = O.tiered_decode_attention(
        to_np(q), to_np(k)[:, :, :4], to_np(v)[:, :, :4], None, None, to_np(k)[:, :, 4:],
        to_np(v)[:, :, 4:], 4, ws, D ** -0.5)
    assert_out_close(to_np(out[:, 0]), ref_out, dt, "decode")
    np.testing.assert_allclose(to_np(st.window_scores) - before, ref_mass, rtol=1e-4, atol=1e-6)


@pytest.mark.parametrize("dt,ws", [("f16", 16), ("bf16", 16)])
def test_int4_tier_window_16(dt, ws):
    """int4 tier with two pages per window: eviction state bit-exact, decode
    output within tolerance, across three evictions."""
    n_checked = 0
    for kind, *rest in _drive_pair(dt, tier=True, P=803, steps=49, seed=5, ws=ws):
        if kind == "evict":
            cache, oc = rest
            st = cache._states[0]
            assert st.tier_pages * 8 == oc.n_tier_tokens
            for a, b in zip(tier_codes(cache), oc.tier_codes):
                np.testing.assert_array_equal(a, b)
            np.testing.assert_array_equal(to_np(st.window_scores), oc.window_scores)
            np.testing.assert_array_equal(to_np(st.original_window_ids), oc.original_window_ids)
            n_checked += 1
        else:
            out, ref_out, t = rest[0][:3]
            assert_out_close(to_np(out[:, 0]), ref_out, dt, f"step {t}")
    assert n_checked == 3


def _random_geometries(n, seed=2024):
    rng = np.random.default_rng(seed)
    out = []
    for _ in range(n):
        out.append((str(rng.choice(["f16", "bf16"])), int(rng.choice([64, 128])), int(rng.integers(1, 9)),
                    int(rng.choice([8, 16])), int(rng.integers(17, 2600)), int(rng.integers(1, 3)),
                    int(rng.integers(1, 3))))
    return out


@pytest.mark.parametrize("dt,D,G,ws,S,B,Hkv", _random_geometries(12))
def test_decode_random_geometries(dt, D, G, ws, S, B, Hkv):
    """Seeded random geometries (dtype, head_dim, GQA 1-8, window 8/16, odd
    lengths, 1-2 rows and kv heads) on the tensor-core decode against the
    oracle: output and window mass."""
    g = torch.Generator().manual_seed(S * 7 + G)
    Hq = Hkv * G
    cos, sin = rope_tables(5e5, D, S + 64)
    cache = make_cache(dt, B, Hkv, Hq, D, S, 1, cos, sin, ws=ws)
    k, v = rand((B, Hkv, S, D), dt, g), rand((B, Hkv, S, D), dt, g)
    q = rand((B, Hq, D), dt, g, scale=2.0)
    cache.update(k.to(DEV), v.to(DEV), 0)
    st = cache._states[0]
    nw = math.ceil((S - 4) / ws)
    before = to_np(st.sides[st.cur].scores[:, :, :nw])
    out = cache.decode_attention(0, q.to(DEV)[:, :, None, :], D ** -0.5)
    ref_out, ref_mass = O.tiered_decode_attention(
        to_np(q), to_np(k)[:, :, :4], to_np(v)[:, :, :4], None, None, to_np(k)[:, :, 4:],
        to_np(v)[:, :, 4:], 4, ws, D ** -0.5)
    assert_out_close(to_np(out[:, 0]), ref_out, dt, "decode")
    np.testing.assert_allclose(to_np(st.window_scores) - before, ref_mass, rtol=1e-4, atol=1e-6)


# -- int4 pages ---------------------------------------------------------------------------

@pytest.mark.parametrize("dt,D", [("f16", 64), ("bf16", 128), ("f32", 32)])
def test_pack_pages_bit_exact(dt, D):
    import ctypes
    from stickykv_b200 import _lib
    g = torch.Generator().manual_seed(7 + D)
    n_pages, s = 37, 4
    first = s + 8 * 11
    cos, sin = rope_tables(5e5, D, first + 8 * n_pages + 8)
    k = rand((n_pages * 8, D), dt, g, scale=3.0)
    v = rand((n_pages * 8, D), dt, g)
    k[5, :32] = 1.25  # a constant group: scale 0
    out = torch.zeros(n_pages, _lib.page_bytes(D), dtype=torch.uint8, device=DEV)
    d = _lib.LayerDesc()
    d.head_dim, d.kv_dtype = D, {"f32": 0, "f16": 1, "bf16": 2}[dt]
    ct = torch.from_numpy(cos[:, : D // 2].copy()).to(DEV)
    stt = torch.from_numpy(sin[:, : D // 2].copy()).to(DEV)
    d.rope_cos, d.rope_sin, d.rope_positions = ct.data_ptr(), stt.data_ptr(), cos.shape[0]
    kd, vd = k.to(DEV), v.to(DEV)
    _lib.check(_lib.lib().skv_pack_pages(ctypes.byref(d), kd.data_ptr(), vd.data_ptr(), first, n_pages,
                                         out.data_ptr(), torch.cuda.current_stream().cuda_stream),
               "skv_pack_pages")
    got = out.cpu().numpy()
    kn, vn = to_np(k), to_np(v)
    for pg in range(n_pages):
        sl = slice(pg * 8, pg * 8 + 8)
        kf = O.to_page_frame(kn[sl], np.arange(first + 8 * pg, first + 8 * pg + 8), cos, sin, s)
        kc, ks, kz = O.quantize_group32(kf)
        vc, vs, vz = O.quantize_group32(vn[sl])
        np.testing.assert_array_equal(got[pg], O.pack_page(kc, ks, kz, vc, vs, vz), err_msg=f"page {pg}")


# -- eviction -----------------------------------------------------------------------------

def _drive_pair(dt, tier, B=3, Hkv=2, G=4, D=64, P=203, steps=30, seed=0, budget=0.4, local=0.25, ws=8):
    """Drive the GPU cache and the oracle cache with identical K/V; scores
    come from the GPU decode kernel each step and are fed to both."""
    g = torch.Generator().manual_seed(seed)
    Hq = Hkv * G
    cos, sin = rope_tables(5e5, D, P + steps + 64)
    cache = make_cache(dt, B, Hkv, Hq, D, P, steps, cos, sin, ws=ws, budget=budget, local=local, tier=tier)
    r = cache.resolved
    oc = O.OracleCache(O.resolve(ws, 4, local, budget, P, Hkv, D, O.DTYPE_SIZES[dt], steps), dt, cos, sin,
                       tier=tier)
    k, v = rand((B, Hkv, P, D), dt, g), rand((B, Hkv, P, D), dt, g)
    cache.update(k.to(DEV), v.to(DEV), 0)
    oc.update(to_np(k), to_np(v), None)
    scores = O.compute_window_scores(np.random.default_rng(seed).random((B, Hq, 1, P)).astype(np.float32), 4, ws)
    st = cache._states[0]
    st.sides[st.cur].scores[:, :, : scores.shape[-1]] = torch.from_numpy(scores).to(DEV)
    st.has_scores, st.W, st.next_window_id = True, scores.shape[-1], scores.shape[-1]
    oc.add_scores(scores)
    evictions = 0
    for t in range(steps):
        k1, v1 = rand((B, Hkv, 1, D), dt, g), rand((B, Hkv, 1, D), dt, g)
        n_before = oc.seq_length
        cache.update(k1.to(DEV), v1.to(DEV), 0)
        evicted = oc.update(to_np(k1), to_np(v1), None)
        evictions += evicted
        assert cache.get_seq_length(0) == oc.seq_length
        if evicted:
            yield "evict", cache, oc
        q = rand((B, Hq, D), dt, g, scale=2.0)
        before = to_np(st.sides[st.cur].scores[:, :, : st.W]) if st.W else None
        out = cache.decode_attention(0, q.to(DEV)[:, :, None, :], D ** -0.5)
        ref_out, ref_mass = oc.decode_attention(to_np(q), D ** -0.5)
        # feed the GPU's step scores to the oracle (identical inputs for selection)
        acc = to_np(st.sides[st.cur].scores[:, :, : st.W])
        step_scores = acc.copy()
        if before is not None:
            step_scores[:, :, : before.shape[-1]] -= before
        yield "decode", (out, ref_out, t, step_scores, ref_mass)
        oc.window_scores = None if oc.window_scores is None else oc.window_scores
        W_new = acc.shape[-1]
        W_old = oc.window_scores.shape[-1]
        if W_new > W_old:
            oc.add_scores(np.zeros(acc.shape[:2] + (W_new,), np.float32))
        oc.window_scores = acc.copy()
    assert evictions == (steps - 1) // ws


@pytest.mark.parametrize("dt,G", [("f32", 4), ("bf16", 4), ("f16", 4), ("f16", 8), ("bf16", 2), ("bf16", 7)])
def test_reference_mode_eviction_bit_exact(dt, G):
    for kind, *rest in _drive_pair(dt, tier=False, G=G):
        if kind == "evict":
            cache, oc = rest
            st = cache._states[0]
            np.testing.assert_array_equal(to_np(st.key_states), oc.k)
            np.testing.assert_array_equal(to_np(st.value_states), oc.v)
            np.testing.assert_array_equal(to_np(st.window_scores), oc.window_scores)
            np.testing.assert_array_equal(to_np(st.original_window_ids), oc.original_window_ids)
        else:
            out, ref_out, t = rest[0][:3]
            assert_out_close(to_np(out[:, 0]), ref_out, dt, f"step {t}")


@pytest.mark.parametrize("dt,G", [("f16", 4), ("bf16", 4), ("f16", 8), ("bf16", 2), ("f16", 1), ("f16", 6)])
def test_int4_tier_eviction_and_decode(dt, G):
    """int4 tier at several GQA ratios (query heads in groups of four MMA
    columns: one group per kv head up to GQA 4, two above; spare columns in
    short groups)."""
    n_checked = 0
    for kind, *rest in _drive_pair(dt, tier=True, G=G, P=403, steps=34, seed=3):
        if kind == "evict":
            cache, oc = rest
            st = cache._states[0]
            assert st.tier_pages * 8 == oc.n_tier_tokens
            sk, sv, rk, rv = fp_parts(cache)
            s = min(4, oc.k.shape[2])
            np.testing.assert_array_equal(sk, oc.k[:, :, :s])
            np.testing.assert_array_equal(sv, oc.v[:, :, :s])
            np.testing.assert_array_equal(rk, oc.k[:, :, s:])
            np.testing.assert_array_equal(rv, oc.v[:, :, s:])
            for a, b in zip(tier_codes(cache), oc.tier_codes):
                np.testing.assert_array_equal(a, b)
            np.testing.assert_array_equal(to_np(st.window_scores), oc.window_scores)
            np.testing.assert_array_equal(to_np(st.original_window_ids), oc.original_window_ids)
            n_checked += 1
        else:
            out, ref_out, t = rest[0][:3]
            assert_out_close(to_np(out[:, 0]), ref_out, dt, f"step {t}")
    assert n_checked == 4



@pytest.mark.parametrize("dt,G,ws,D", [("bf16", 5, 8, 128), ("f16", 3, 16, 64), ("bf16", 6, 8, 64)])
def test_int4_tier_other_geometries(dt, G, ws, D):
    """int4 tier at GQA 3/5/6, head_dim 64/128 and windows of 8/16 tokens:
    tier codes, scores and ids bit-exact after each eviction, decode output
    within tolerance every step."""
    n_checked = 0
    for kind, *rest in _drive_pair(dt, tier=True, G=G, D=D, ws=ws, P=611, steps=2 * ws + 1, seed=G + ws):
        if kind == "evict":
            cache, oc = rest
            st = cache._states[0]
            assert st.tier_pages * 8 == oc.n_tier_tokens
            for a, b in zip(tier_codes(cache), oc.tier_codes):
                np.testing.assert_array_equal(a, b)
            np.testing.assert_array_equal(to_np(st.window_scores), oc.window_scores)
            np.testing.assert_array_equal(to_np(st.original_window_ids), oc.original_window_ids)
            n_checked += 1
        else:
            out, ref_out, t = rest[0][:3]
            assert_out_close(to_np(out[:, 0]), ref_out, dt, f"step {t}")
    assert n_checked == 2


@pytest.mark.parametrize("P", [5000, 6000])
def test_int4_tier_decode_long_single_head(P):
    """One (row, kv head) with thousands of retained tokens: the decode splits
    them into many cost-balanced ranges that a second kernel merges."""
    n = 0
    for kind, *rest in _drive_pair("f16", tier=True, B=1, Hkv=1, P=P, steps=10, seed=P):
        if kind == "decode":
            out, ref_out, t, mass, ref_mass = rest[0]
            assert_out_close(to_np(out[:, 0]), ref_out, "f16", f"step {t}")
            np.testing.assert_allclose(mass, ref_mass, rtol=5e-3, atol=1e-6, err_msg=f"step {t}")
            n += 1
    assert n == 10


# -- prefill ------------------------------------------------------------------------------

def test_prefill_scores_match_reference_golden():
    z = np.load(os.path.join(G, "prefill_scores.npz"))
    B, Hq, T, D = z["q"].shape
    Hkv = z["k"].shape[1]
    cos, sin = rope_tables(1e4, D, 128)
    cache = make_cache("f32", B, Hkv, Hq, D, T, 1, cos, sin)
    k = torch.from_numpy(z["k"]).to(DEV)
    v = torch.randn(B, Hkv, T, D).to(DEV)
    q = torch.from_numpy(z["q"]).to(DEV)
    cache.update(k, v, 0)
    out = cache.prefill_attention(0, q, k, v, D ** -0.5)
    np.testing.assert_allclose(to_np(cache._states[0].window_scores), z["scores"], rtol=1e-5, atol=2e-5)
    ref = torch.nn.functional.scaled_dot_product_attention(
        q, k.repeat_interleave(Hq // Hkv, 1), v.repeat_interleave(Hq // Hkv, 1), is_causal=True)
    np.testing.assert_allclose(to_np(out), to_np(ref.transpose(1, 2)), atol=1e-5)


@pytest.mark.parametrize("dt,D,G,T", [("f16", 64, 4, 333), ("bf16", 64, 4, 333), ("bf16", 128, 2, 700),
                                       ("f16", 128, 8, 129), ("f16", 64, 1, 64), ("f16", 64, 2, 256),
                                       ("bf16", 128, 4, 1100), ("bf16", 64, 7, 300)])
def test_prefill_matches_oracle(dt, D, G, T):
    """Tensor-core prefill (fp16/bf16, head_dim 64/128): output against torch
    fp32 attention, prompt window scores against the oracle; partial last
    tiles, several GQA ratios."""
    g = torch.Generator().manual_seed(5 + T)
    B, Hkv = 2, 2
    Hq = Hkv * G
    cos, sin = rope_tables(5e5, D, T + 64)
    cache = make_cache(dt, B, Hkv, Hq, D, T, 1, cos, sin)
    q, k, v = rand((B, Hq, T, D), dt, g), rand((B, Hkv, T, D), dt, g), rand((B, Hkv, T, D), dt, g)
    cache.update(k.to(DEV), v.to(DEV), 0)
    out = cache.prefill_attention(0, q.to(DEV), k.to(DEV), v.to(DEV), D ** -0.5)
    ref = O.prefill_window_scores(to_np(q), to_np(k), D ** -0.5, 4, 8)
    np.testing.assert_allclose(to_np(cache._states[0].window_scores), ref, rtol=2e-4, atol=1e-4)
    qd, kd, vd = (x.to(DEV).float() for x in (q, k, v))
    sd = torch.nn.functional.scaled_dot_product_attention(
        qd, kd.repeat_interleave(G, 1), vd.repeat_interleave(G, 1), is_causal=True)
    assert_out_close(to_np(out), to_np(sd.transpose(1, 2)), dt, "prefill")


@pytest.mark.parametrize("dt,D,T", [("bf16", 64, 1), ("f16", 128, 5), ("bf16", 64, 127)])
def test_prefill_tiny_prompts_through_the_abi(dt, D, T):
    """Prompts shorter than one 128-row tile (down to one token) straight
    through `skv_prefill_attention` (no window scores): output against torch
    fp32 causal attention."""
    import ctypes as C
    from stickykv_b200 import _lib
    L = _lib.lib()
    g = torch.Generator().manual_seed(11 + T)
    B, Hkv, Hq = 2, 2, 8
    q, k, v = (rand(s_, dt, g).to(DEV) for s_ in ((B, Hq, T, D), (B, Hkv, T, D), (B, Hkv, T, D)))
    out = torch.full((B, T, Hq, D), float("nan"), device=DEV, dtype=TORCH_DT[dt])
    d = _lib.LayerDesc()
    d.batch, d.num_kv_heads, d.num_q_heads, d.head_dim = B, Hkv, Hq, D
    d.kv_dtype = {"f16": 1, "bf16": 2}[dt]
    d.window_size, d.num_sink, d.sink_pad = 8, 4, 8
    d.fp_capacity, d.k_fp, d.v_fp = T, k.data_ptr(), v.data_ptr()
    nb = L.skv_prefill_workspace_size(C.byref(d), T)
    ws = torch.empty(nb, dtype=torch.uint8, device=DEV)
    _lib.check(L.skv_prefill_attention(C.byref(d), T, q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(),
                                       C.c_float(D ** -0.5), None, 0, ws.data_ptr(), nb,
                                       torch.cuda.current_stream().cuda_stream), "prefill")
    qd, kd, vd = (x.float() for x in (q, k, v))
    sd = torch.nn.functional.scaled_dot_product_attention(
        qd, kd.repeat_interleave(Hq // Hkv, 1), vd.repeat_interleave(Hq // Hkv, 1), is_causal=True)
    assert_out_close(to_np(out), to_np(sd.transpose(1, 2)), dt, "prefill tiny")


# -- full-size properties ----------------------------------------------------------------

def test_cfg3_scale_eviction_selection_and_codes():
    """16 rows x 8 kv heads x 16384 tokens (bf16): the kept windows equal the
    oracle's selection on the same scores; spot rows' int4 codes are bit-exact;
    every row keeps 6544 tokens."""
    dt, B, Hkv, Hq, D, P = "bf16", 16, 8, 32, 64, 16384
    g = torch.Generator().manual_seed(2)
    cos, sin = rope_tables(5e5, D, P + 64)
    cache = make_cache(dt, B, Hkv, Hq, D, P, 0, cos, sin, tier=True)
    k = rand((B, Hkv, P, D), dt, g).to(DEV)
    v = rand((B, Hkv, P, D), dt, g).to(DEV)
    cache.update(k, v, 0)
    st = cache._states[0]
    W = math.ceil((P - 4) / 8)
    scores = torch.rand(B, Hq, W, generator=g)
    st.sides[st.cur].scores[:, :, :W] = scores.to(DEV)
    st.has_scores, st.W, st.next_window_id = True, W, W
    for t in range(9):
        cache.update(k[:, :, :1].clone(), v[:, :, :1].clone(), 0)
    r = cache.resolved
    assert (r.top_k_windows, r.local_tokens) == (613, 1640)
    ret = O.retain_window_indices(to_np(scores), r.top_k_windows, r.local_tokens // 8)
    # 16393 tokens at the eviction: the 9 appended tokens past window 2047 are
    # not covered by the scores and drop, as in the reference (6544 + 4)
    assert cache.get_seq_length(0) == O.expand_to_token_indices(ret, 4, 8, P + 9).shape[1] == 6548
    np.testing.assert_array_equal(to_np(st.original_window_ids), ret)
    codes = tier_codes(cache, rows=2)
    kn = to_np(k[:2, :, :])
    for b in range(2):
        for j in (0, 100, 612):
            w = int(ret[b, j])
            pos = 4 + 8 * w + np.arange(8)
            kf = O.to_page_frame(kn[b][:, pos], np.broadcast_to(pos, (Hkv, 8)), cos, sin, 4)
            kc, ks, kz = O.quantize_group32(kf)
            np.testing.assert_array_equal(codes[0][b, :, j * 8:(j + 1) * 8], kc)
            np.testing.assert_array_equal(codes[1][b, :, j * 8:(j + 1) * 8], ks)


@pytest.mark.parametrize("dt,D,G,tier", [("f16", 64, 4, True), ("bf16", 128, 4, False),
                                         ("bf16", 64, 4, True), ("f32", 64, 2, False), ("f16", 64, 8, True),
                                         ("bf16", 128, 2, False)])
def test_fused_append_decode_matches_append_then_decode(dt, D, G, tier):
    """skv_decode_attention_append == skv_append + skv_decode_attention, bit
    for bit: output, window scores and the fp store (tensor-core path for the
    fp16/bf16 cases, the portable path for fp32)."""
    import ctypes as Ct
    from stickykv_b200 import _lib
    L = _lib.lib()
    g = torch.Generator().manual_seed(D + G)
    B, Hkv, P = 2, 2, 611
    Hq = Hkv * G
    cos, sin = rope_tables(5e5, D, P + 64)
    cache = make_cache(dt, B, Hkv, Hq, D, P, 16, cos, sin, tier=tier)
    cache.update(rand((B, Hkv, P, D), dt, g).to(DEV), rand((B, Hkv, P, D), dt, g).to(DEV), 0)
    st = cache._states[0]
    W = math.ceil((P - 4) / 8)
    st.sides[st.cur].scores[:, :, :W] = torch.rand(B, Hq, W, generator=g).to(DEV)
    st.has_scores, st.W, st.next_window_id = True, W, W
    for _ in range(9):  # one eviction
        k1 = rand((B, Hkv, 1, D), dt, g).to(DEV)
        cache.update(k1, k1.clone(), 0)
    if st.pending is not None:
        cache._flush(st)
    assert (st.tier_pages > 0) == tier
    side = st.sides[st.cur]
    d = cache._desc(st, side)
    T0 = st.T
    stream = torch.cuda.current_stream().cuda_stream
    kn = rand((B, Hkv, 1, D), dt, g).to(DEV)
    vn = rand((B, Hkv, 1, D), dt, g).to(DEV)
    q = rand((B, Hq, D), dt, g, scale=2.0).to(DEV)
    nbytes = L.skv_decode_workspace_size(Ct.byref(d), T0 + 1)
    runs = []
    for fused in (False, True):
        k, v, sc = side.k.clone(), side.v.clone(), side.scores.clone()
        dd = _lib.LayerDesc.from_buffer_copy(d)
        dd.k_fp, dd.v_fp = k.data_ptr(), v.data_ptr()
        out = torch.empty(B, Hq, D, dtype=q.dtype, device=DEV)
        ws = torch.empty(nbytes, dtype=torch.uint8, device=DEV)
        if fused:
            rc = L.skv_decode_attention_append(Ct.byref(dd), T0 + 1, st.tier_pages, kn.data_ptr(), vn.data_ptr(),
                                               kn.stride(0), kn.stride(1), q.data_ptr(), q.stride(0), q.stride(1),
                                               out.data_ptr(), out.stride(0), out.stride(1), Ct.c_float(D ** -0.5),
                                               sc.data_ptr(), st.scores_cap, ws.data_ptr(), nbytes, stream)
            assert rc == 0, L.skv_last_cuda_error()
        else:
            assert L.skv_append(Ct.byref(dd), T0, st.tier_pages, kn.data_ptr(), vn.data_ptr(), kn.stride(0),
                                kn.stride(1), kn.stride(2), 1, stream) == 0
            rc = L.skv_decode_attention(Ct.byref(dd), T0 + 1, st.tier_pages, q.data_ptr(), q.stride(0),
                                        q.stride(1), out.data_ptr(), out.stride(0), out.stride(1),
                                        Ct.c_float(D ** -0.5), sc.data_ptr(), st.scores_cap, ws.data_ptr(),
                                        nbytes, stream)
            assert rc == 0, L.skv_last_cuda_error()
        torch.cuda.synchronize()
        runs.append((out, sc, k, v))
    for name, a, b in zip(("out", "scores", "k", "v"), *runs):
        bad = (a != b) & ~(torch.isnan(a) & torch.isnan(b))
        assert not bad.any(), f"{name}: {int(bad.sum())} differ, first at {bad.nonzero()[0].tolist()} (T0={T0})"


@pytest.mark.parametrize("dt,D", [("f16", 64), ("bf16", 128), ("f32", 64)])
def test_int4_tier_key_and_value_states_materialised(dt, D):
    """key_states / value_states of an int4-tier cache (skv_materialize): fp
    tokens as stored, tier tokens dequantised and rotated to their current
    positions, bit-exact against the oracle after each eviction."""
    n = 0
    for kind, *rest in _drive_pair(dt, tier=True, D=D, P=403, steps=18, seed=9):
        if kind != "evict":
            continue
        cache, oc = rest
        st = cache._states[0]
        assert st.tier_pages > 0
        k, v = oc.materialize()
        np.testing.assert_array_equal(to_np(st.key_states), k)
        np.testing.assert_array_equal(to_np(st.value_states), v)
        n += 1
    assert n == 2


@pytest.mark.parametrize("dt,D,tier", [("f16", 64, True), ("bf16", 64, False), ("bf16", 128, True),
                                       ("f32", 64, True)])
def test_fused_append_evict_matches_append_then_evict(dt, D, tier):
    """skv_evict_append (the evicting step's token read by the eviction's move,
    never written to the source store) == skv_append + skv_evict, bit for
    bit over three evictions: fp store, int4 tier, scores and ids."""
    B, Hkv, G, P = 3, 2, 4, 411
    Hq = Hkv * G
    cos, sin = rope_tables(5e5, D, P + 64)
    caches = []
    for fused in (False, True):
        g = torch.Generator().manual_seed(D + 7)
        c = make_cache(dt, B, Hkv, Hq, D, P, 32, cos, sin, tier=tier)
        c.fuse_evict_append = fused
        c.update(rand((B, Hkv, P, D), dt, g).to(DEV), rand((B, Hkv, P, D), dt, g).to(DEV), 0)
        st = c._states[0]
        W = math.ceil((P - 4) / 8)
        st.sides[st.cur].scores[:, :, :W] = torch.rand(B, Hq, W, generator=g).to(DEV)
        st.has_scores, st.W, st.next_window_id = True, W, W
        caches.append((c, g))
    n_ev = 0
    for step in range(25):
        states = []
        for c, g in caches:
            k1 = rand((B, Hkv, 1, D), dt, g).to(DEV)
            v1 = rand((B, Hkv, 1, D), dt, g).to(DEV)
            sc = torch.rand(B, Hq, 1, generator=g)
            before = c._states[0].evictions
            c.update(k1, v1, 0)
            st = c._states[0]
            if st.pending is not None:
                c._flush(st)
            st.sides[st.cur].scores[:, :, : st.W] += sc.to(DEV)  # some mass for the next selection
            states.append(st.evictions > before)
        assert states[0] == states[1]
        if states[0]:
            n_ev += 1
            (a, _), (b, _) = caches
            sa, sb = a._states[0], b._states[0]
            assert (sa.T, sa.tier_pages, sa.W) == (sb.T, sb.tier_pages, sb.W)
            for x, y in zip(fp_parts(a), fp_parts(b)):
                np.testing.assert_array_equal(x, y)
            if tier:
                for x, y in zip(tier_codes(a), tier_codes(b)):
                    np.testing.assert_array_equal(x, y)
            np.testing.assert_array_equal(to_np(sa.window_scores), to_np(sb.window_scores))
            np.testing.assert_array_equal(to_np(sa.original_window_ids), to_np(sb.original_window_ids))
    assert n_ev == 3
