"""Pin the CPU oracle to the reference: golden vectors produced by running the
reference (tests/golden/make_golden.py) and the reference's own known-answer
tests (tests/test_windowed_cache.py in the reference)."""

import json
import math
import os

import numpy as np
import pytest

from oracle import skv_oracle as O

G = os.path.join(os.path.dirname(__file__), "golden")


def load(name):
    return np.load(os.path.join(G, name))


# -- budget resolution --------------------------------------------------------

def test_resolve_matches_reference_on_all_geometries():
    cases = json.load(open(os.path.join(G, "resolve.json")))
    assert len(cases) >= 15
    for c in cases:
        r = O.resolve(c["window_size"], c["num_sink_tokens"], c["local_window_size"],
                      c["cache_budget"], c["prefill_len"], c["num_kv_heads"], c["head_dim"],
                      O.DTYPE_SIZES[c["dtype"]], c["max_tokens"])
        assert r.__dict__ == c["resolved"], c


def test_worked_example_kat():
    # reference tests/test_windowed_cache.py:121-144
    r = O.resolve(8, 4, 16, 0.40, 100, 8, 128, 2, 100)
    assert (r.bytes_per_token, r.total_budget_bytes, r.total_budget_tokens, r.top_k_windows) == \
        (4096, 327680, 80, 7)


def test_local_snapping_kat():
    # reference tests/test_windowed_cache.py:91-115
    assert O.resolve(8, 4, 0.25, 0.50, 100, 8, 128, 2, 128).local_tokens == 32
    assert O.resolve(8, 4, 0.10, 0.50, 100, 8, 128, 2, 128).local_tokens == 16


def test_budget_too_small_raises():
    with pytest.raises(ValueError, match="total_budget_tokens"):
        O.resolve(8, 10, 40, 0.05, 100, 8, 128, 2, 50)


# -- scoring -------------------------------------------------------------------

# float sums: torch and numpy order the additions differently, so the
# reductions agree to a few ulp (rtol 1e-6), not bit for bit.
FSUM = dict(rtol=1e-6, atol=1e-7)


def test_window_scores_match_reference():
    z = load("scorer.npz")
    for (s, ws) in [(4, 5), (0, 8), (4, 8), (3, 1)]:
        got = O.compute_window_scores(z["attn"], s, ws)
        np.testing.assert_allclose(got, z[f"ws_{s}_{ws}"], **FSUM)
    np.testing.assert_allclose(O.reduce_token_scores_to_windows(z["tok"], 4, 8), z["tok_4_8"], **FSUM)


def test_partial_window_count_kat():
    # reference tests/test_windowed_cache.py:587-599: 97 keys, 4 sinks, ws 5 -> 19 windows
    attn = np.random.default_rng(0).random((1, 2, 4, 97)).astype(np.float32)
    assert O.compute_window_scores(attn, 4, 5).shape == (1, 2, math.ceil(93 / 5))


def test_accumulate_three_times_kat():
    # reference tests/test_windowed_cache.py:243-261
    attn = np.random.default_rng(1).random((1, 4, 4, 20)).astype(np.float32)
    s1 = O.compute_window_scores(attn, 4, 8)
    c = O.OracleCache(O.resolve(8, 4, 8, 1.0, 16, 1, 8, 4, 4), "f32",
                      np.ones((64, 8), np.float32), np.zeros((64, 8), np.float32))
    for _ in range(3):
        c.add_scores(s1)
    np.testing.assert_allclose(c.window_scores, 3 * s1, atol=1e-5)


# -- selection -----------------------------------------------------------------

def test_retain_and_expand_match_reference():
    z = load("policy.npz")
    for ci, (k, loc_w, ws, s, total) in enumerate(z["cases"]):
        ret = O.retain_window_indices(z[f"scores_{ci}"], int(k), int(loc_w))
        np.testing.assert_array_equal(ret, z[f"ret_{ci}"])
        tok = O.expand_to_token_indices(ret, int(s), int(ws), int(total))
        np.testing.assert_array_equal(tok, z[f"tok_{ci}"])


def test_scores_survive_compaction_kat():
    # reference tests/test_windowed_cache.py:267-303
    sc = np.broadcast_to(np.array([10.0, 1.0, 2.0, 8.0, 7.0, 5.0], np.float32), (1, 4, 6)).copy()
    ret = O.retain_window_indices(sc, 2, 2)
    assert ret.tolist() == [[0, 3, 4, 5]]
    got = np.take_along_axis(sc, np.broadcast_to(ret[:, None], (1, 4, 4)), axis=-1)
    assert got[0, 0].tolist() == [10.0, 8.0, 7.0, 5.0]


def test_ties_break_to_lowest_index():
    sc = np.ones((2, 3, 10), np.float32)
    sc[1, :, 7] = 2.0
    ret = O.retain_window_indices(sc, 3, 2)
    assert ret[0].tolist() == [0, 1, 2, 8, 9]
    assert ret[1].tolist() == [0, 1, 7, 8, 9]


def test_per_row_independence_kat():
    # reference tests/test_windowed_cache.py:454-471
    sc = np.zeros((2, 4, 5), np.float32)
    sc[0, :, 0] = 100.0
    sc[1, :, 3] = 100.0
    ret = O.retain_window_indices(sc, 1, 1)
    assert 0 in ret[0].tolist() and 3 in ret[1].tolist()


# -- RoPE strip + re-apply -------------------------------------------------------

@pytest.mark.parametrize("dt", ["f32", "bf16", "f16"])
def test_rerotate_bit_exact_vs_reference(dt):
    z = load(f"rerotate_{dt}.npz")
    keep = z["keep"]
    k_sel = np.take_along_axis(z["k"], keep[:, None, :, None], axis=2)
    old = np.take_along_axis(z["pos"], keep, axis=1)
    new = np.broadcast_to(np.arange(keep.shape[1]), keep.shape)
    got = O.rerotate_keys(k_sel, old, new, z["cos"], z["sin"], dt)
    np.testing.assert_array_equal(got, z["k_out"])
    np.testing.assert_array_equal(np.take_along_axis(z["v"], keep[:, None, :, None], axis=2),
                                  z["v_out"])
    assert z["pos_out"].tolist() == new.tolist()


# -- cache orchestration -----------------------------------------------------------

@pytest.mark.parametrize("dt", ["f32", "bf16"])
def test_cache_drive_bit_exact_vs_reference(dt):
    z = load(f"cache_drive_{dt}.npz")
    B, Hkv, Hq, D, P, M = [int(x) for x in z["meta"]]
    r = O.resolve(8, 4, 0.25, 0.5, P, Hkv, D, O.DTYPE_SIZES[dt], M)
    c = O.OracleCache(r, dt, z["cos"], z["sin"])
    c.update(z["k_0"], z["v_0"], None)
    n_evict = 0
    for t in range(1, M + 1):
        n_evict += c.update(z[f"k_{t}"], z[f"v_{t}"], z[f"s_{t - 1}"])
        assert c.seq_length == int(z[f"len_{t}"]), t
        np.testing.assert_array_equal(c.original_window_ids, z[f"ids_{t}"])
    assert n_evict == (M - 1) // 8    # decode steps 0..M-1 evict at 8, 16, 24, 32
    np.testing.assert_array_equal(c.k, z["final_k"])
    np.testing.assert_array_equal(c.v, z["final_v"])
    np.testing.assert_allclose(c.window_scores, z["final_scores"], **FSUM)
    np.testing.assert_array_equal(c.original_window_ids, z["final_ids"])


def _drive_divergent(B):
    # reference tests/test_windowed_cache.py:643-683 geometry
    r = O.resolve(1, 0, 1, 0.375, 8, 8, 128, 4, 0)
    assert (r.top_k_windows, r.local_tokens) == (2, 1)
    D = 8
    cos = np.ones((64, D), np.float32)
    sin = np.zeros((64, D), np.float32)
    c = O.OracleCache(r, "f32", cos, sin)
    s0 = np.zeros((B, 4, 8), np.float32)
    s0[0, :, [1, 3]] = 100.0
    if B > 1:
        s0[1, :, [5, 7]] = 100.0
    scores = [s0, np.zeros((B, 4, 9), np.float32), np.zeros((B, 4, 10), np.float32)]

    def keys(T, start):
        return np.broadcast_to(np.arange(start, start + T, dtype=np.float32)[None, None, :, None],
                               (B, 2, T, D)).copy()
    k = keys(8, 0)
    c.update(k, k.copy(), scores[0])
    for i, pos in enumerate((8, 9)):
        k1 = keys(1, pos)
        c.update(k1, k1.copy(), scores[i + 1])
    return c


def test_divergent_eviction_kat():
    # reference tests/test_windowed_cache.py:689-724
    c = _drive_divergent(2)
    assert c.original_window_ids.tolist() == [[1, 3, 9], [5, 7, 9]]
    kept = c.k[:, 0, :, 0]
    assert kept.tolist() == [[1.0, 3.0, 9.0], [5.0, 7.0, 9.0]]
    c1 = _drive_divergent(1)
    np.testing.assert_array_equal(c1.original_window_ids[0], c.original_window_ids[0])
    np.testing.assert_array_equal(c1.k[0], c.k[0])


# -- attention + scoring -------------------------------------------------------------

@pytest.mark.parametrize("dt,tol", [("f32", 2e-6), ("f16", 2e-3)])
def test_eager_decode_matches_reference(dt, tol):
    z = load(f"eager_decode_{dt}.npz")
    out, sc = O.eager_decode_attention(z["q"], z["k"], z["v"], 64 ** -0.5, 4, 8, dt)
    np.testing.assert_allclose(out, z["out"], atol=tol, rtol=0)
    np.testing.assert_allclose(sc, z["scores"], atol=tol, rtol=0)


def test_tiered_attention_equals_eager_without_tier():
    z = load("eager_decode_f32.npz")
    s = 4
    out, mass = O.tiered_decode_attention(z["q"], z["k"][:, :, :s], z["v"][:, :, :s], None, None,
                                          z["k"][:, :, s:], z["v"][:, :, s:], s, 8, 64 ** -0.5)
    np.testing.assert_allclose(out, z["out"], atol=2e-6)
    np.testing.assert_allclose(mass, z["scores"], atol=2e-6)


def test_prefill_scores_match_reference_chunked_hook_math():
    z = load("prefill_scores.npz")
    got = O.prefill_window_scores(z["q"], z["k"], 16 ** -0.5, 4, 8)
    np.testing.assert_allclose(got, z["scores"], atol=2e-5)


# -- int4 tier restatement ------------------------------------------------------------

def test_int4_roundtrip_and_page_packing():
    rng = np.random.default_rng(3)
    for D in (64, 128):
        x = rng.standard_normal((8, D)).astype(np.float32)
        kc, ks, kz = O.quantize_group32(x)
        vc, vs, vz = O.quantize_group32(-x * 2)
        assert kc.max() <= 15 and ks.dtype == np.float16
        deq = O.dequant_group32(kc, ks, kz)
        # error bounded by half a step (plus fp16 rounding of scale/zero)
        step = ks.astype(np.float32).repeat(32, axis=-1)
        assert np.all(np.abs(deq - x) <= 0.5 * step + 2e-2)
        page = O.pack_page(kc, ks, kz, vc, vs, vz)
        assert page.size == O.page_bytes(D)
        for a, b in zip(O.unpack_page(page, D), (kc, ks, kz, vc, vs, vz)):
            np.testing.assert_array_equal(a, b)


def test_int4_constant_group_gives_zero_scale():
    x = np.full((2, 64), 0.75, np.float32)
    kc, ks, kz = O.quantize_group32(x)
    assert np.all(kc == 0) and np.all(ks == 0)
    np.testing.assert_array_equal(O.dequant_group32(kc, ks, kz), x)


def test_page_frame_rotation_is_consistent():
    """q . R(p) k_pre == R(-P) q . k_frame (page-frame identity) up to fp32."""
    rng = np.random.default_rng(4)
    D = 64
    inv = (1.0 / (500000.0 ** (np.arange(0, D, 2) / D))).astype(np.float32)
    cos, sin = O.rope_tables(inv, 200)
    k_pre = rng.standard_normal((1, 24, D)).astype(np.float32)
    pos = np.arange(37, 61)
    # post-RoPE key at pos
    h = D // 2
    c, s = cos[pos][:, :h], sin[pos][:, :h]
    x, y = k_pre[..., :h], k_pre[..., h:]
    k_post = np.concatenate([x * c - y * s, y * c + x * s], -1)
    sinks = 4
    kf = O.to_page_frame(k_post, pos[None], cos, sin, sinks)
    q = rng.standard_normal(D).astype(np.float32)
    for i, p in enumerate(pos):
        P = sinks + 8 * ((p - sinks) // 8)
        lhs = q @ k_post[0, i]
        rhs = O.rotate_query_to_page(q, P, cos, sin) @ kf[0, i]
        assert abs(lhs - rhs) < 1e-4 * (1 + abs(lhs))


def test_vectorised_page_unpack_equals_scalar_unpack():
    rng = np.random.default_rng(5)
    for D in (64, 128):
        pages = []
        for _ in range(6):
            kc = rng.integers(0, 16, (8, D)).astype(np.uint8)
            vc = rng.integers(0, 16, (8, D)).astype(np.uint8)
            sc = [rng.standard_normal((8, D // 32)).astype(np.float16) for _ in range(4)]
            pages.append(O.pack_page(kc, sc[0], sc[1], vc, sc[2], sc[3]))
        arr = np.stack(pages).reshape(2, 3, -1)
        got = O.unpack_pages(arr, D)
        for i in range(6):
            want = O.unpack_page(pages[i], D)
            for a, b in zip(got, want):
                np.testing.assert_array_equal(a.reshape((6,) + a.shape[2:])[i], b)


def test_grouped_tiered_attention_equals_per_page_loop():
    rng = np.random.default_rng(6)
    B, Hkv, G, D, s, nt, nr = 2, 2, 4, 64, 4, 48, 37
    inv = (1.0 / (500000.0 ** (np.arange(0, D, 2) / D))).astype(np.float32)
    cos, sin = O.rope_tables(inv, 200)
    f = lambda *sh: rng.standard_normal(sh).astype(np.float32)
    args = (f(B, Hkv * G, D), f(B, Hkv, s, D), f(B, Hkv, s, D), f(B, Hkv, nt, D), f(B, Hkv, nt, D),
            f(B, Hkv, nr, D), f(B, Hkv, nr, D), s, 8, D ** -0.5, cos, sin)
    o1, m1 = O.tiered_decode_attention(*args)
    o2, m2 = O.tiered_decode_attention_grouped(*args)
    np.testing.assert_allclose(o2, o1, rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(m2, m1, rtol=1e-5, atol=1e-7)


def test_tie_fixture_puts_equal_means_across_the_threshold():
    """The tie-heavy scores of the GPU tie test (one of a few dyadic levels
    per window, equal across heads) do put several equal head means at the
    top-k threshold, and the oracle keeps the lowest-index ones."""
    rng = np.random.default_rng(21)
    B, Hq, W, k, loc = 4, 8, 150, 37, 10
    per_w = rng.choice(np.asarray((0.25, 0.5, 0.75), np.float32), size=(B, W))
    sc = np.ascontiguousarray(np.broadcast_to(per_w[:, None, :], (B, Hq, W)))
    mean = O.head_mean(sc)
    np.testing.assert_array_equal(mean, per_w)
    ret = O.retain_window_indices(sc, k, loc)
    for b in range(B):
        ev = mean[b, : W - loc]
        kth = np.sort(ev)[::-1][k - 1]
        tied = np.flatnonzero(ev == kth)
        n_above = int((ev > kth).sum())
        assert tied.size > k - n_above  # more tied windows than places left
        kept_tied = [w for w in ret[b, :k] if ev[w] == kth]
        np.testing.assert_array_equal(kept_tied, tied[: k - n_above])


def test_materialized_tier_attends_like_the_page_frame():
    """Attention over the materialised keys and values (tier rotated to its
    current positions) equals the tiered attention that rotates the query to
    each page instead (fp32 cache, so no rounding between the two)."""
    rng = np.random.default_rng(8)
    B, Hkv, G, D, P = 2, 2, 4, 64, 203
    inv = (1.0 / (500000.0 ** (np.arange(0, D, 2) / D))).astype(np.float32)
    cos, sin = O.rope_tables(inv, P + 64)
    oc = O.OracleCache(O.resolve(8, 4, 0.25, 0.4, P, Hkv, D, 4, 16), "f32", cos, sin, tier=True)
    oc.update(rng.standard_normal((B, Hkv, P, D)).astype(np.float32),
              rng.standard_normal((B, Hkv, P, D)).astype(np.float32), None)
    oc.add_scores(rng.random((B, Hkv * G, -(-(P - 4) // 8))).astype(np.float32))
    for _ in range(9):
        kv = rng.standard_normal((B, Hkv, 1, D)).astype(np.float32)
        oc.update(kv, kv, None)
    assert oc.n_tier_tokens > 0
    k, v = oc.materialize()
    assert k.shape[2] == oc.seq_length
    q = rng.standard_normal((B, Hkv * G, D)).astype(np.float32)
    out_frame, mass_frame = oc.decode_attention(q, D ** -0.5)
    out_plain, mass_plain = O.tiered_decode_attention(q, k[:, :, :4], v[:, :, :4], None, None, k[:, :, 4:],
                                                      v[:, :, 4:], 4, 8, D ** -0.5)
    np.testing.assert_allclose(out_plain, out_frame, rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(mass_plain, mass_frame, rtol=1e-4, atol=1e-6)
