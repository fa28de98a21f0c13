"""CPU oracle for StickyKV's windowed-eviction decode path.

TEST INFRASTRUCTURE ONLY.  Nothing in the product (``stickykv_b200``) imports
this module.  It is used as the checker by ``tests/``, ``__graft_entry__.smoke``
and the ``cpu_baseline`` / ``--impl reference`` legs of ``bench.py``.

It restates, in numpy, the algorithm of the reference plugin
(shaswata965-coder/StickyKV) for the hot path, one function per reference
function, each citing the file:line it follows:

* budget resolution          modules/windowed_cache/config.py:155-244
* window scoring             modules/windowed_cache/scorer.py:17-109
* retain selection           modules/windowed_cache/policy.py:81-146
* window -> token expansion  modules/windowed_cache/policy.py:152-209
* compaction                 modules/windowed_cache/state.py:125-159
* RoPE strip + re-apply      modules/windowed_cache/state.py:165-232 together
                             with transformers' ``apply_rotary_pos_emb``
                             (rotate-half convention, elementwise ops rounded
                             to the KV dtype)
* cache orchestration        modules/windowed_cache/cache.py:110-293
* eager decode attention     transformers ``eager_attention_forward`` (softmax
                             in fp32) + scorer.compute_window_scores, as used
                             by modules/windowed_eager_cache/hooks.py:145-180

and it restates the int4 tier that the reference only specifies
(design.md:14-22, :130-187, :335-354), with the group-32 asymmetric format:
per (token, kv head, group of 32 channels), ``scale = fp16((max-min)/15)``,
``zero = fp16(min)``, ``code = clamp(rint((x-zero)/scale), 0, 15)`` (round half
to even; ``scale == 0`` gives code 0), dequant ``code*scale + zero``.

Parity is pinned two ways: the reference's own known-answer tests
(tests/test_windowed_cache.py) are re-run against these functions, and golden
vectors produced by importing the reference (``tests/golden/make_golden.py``)
are compared bit-for-bit.  The int4 tier has no reference implementation; its
parity with the CUDA path is checked bit-exactly (codes, scales, page bytes)
against this restatement.
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Dict, List, Optional, Tuple

import numpy as np

# ---------------------------------------------------------------------------
# dtype helpers (emulate torch's per-op rounding to the KV dtype)
# ---------------------------------------------------------------------------

DTYPE_SIZES = {"f32": 4, "f16": 2, "bf16": 2}


def round_bf16(x: np.ndarray) -> np.ndarray:
    """Round float32 values to bfloat16 (round-to-nearest-even), kept as f32."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    nan = np.isnan(x)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
    out = (r & 0xFFFFFFFF).astype(np.uint32).view(np.float32)
    out = np.where(nan, x, out)
    return out.astype(np.float32)


def round_to(x: np.ndarray, dtype: str) -> np.ndarray:
    """Round float32 values to the KV dtype and return them as float32."""
    x = np.asarray(x, dtype=np.float32)
    if dtype == "f32":
        return x
    if dtype == "f16":
        return x.astype(np.float16).astype(np.float32)
    if dtype == "bf16":
        return round_bf16(x)
    raise ValueError(dtype)


def bf16_bits(x: np.ndarray) -> np.ndarray:
    """uint16 bit pattern of bf16-representable float32 values."""
    return (np.ascontiguousarray(x, dtype=np.float32).view(np.uint32) >> 16).astype(np.uint16)


# ---------------------------------------------------------------------------
# 1. Budget resolution  (config.py:155-244)
# ---------------------------------------------------------------------------


@dataclass(frozen=True)
class Resolved:
    window_size: int
    num_sink_tokens: int
    local_tokens: int
    top_k_windows: int
    bytes_per_token: int
    total_budget_bytes: int
    total_budget_tokens: int


def resolve(window_size: int, num_sink_tokens: int, local_window_size, cache_budget: float,
            prefill_len: int, num_kv_heads: int, head_dim: int, element_size: int,
            max_tokens: int) -> Resolved:
    """Byte budget -> token counts.  Follows config.py:201-244 step for step:
    ``int(budget*(P+M)*bpt) // bpt`` tokens; a float local size is a fraction
    of the *budget*, ceiled then snapped up to a window multiple."""
    bytes_per_token = num_kv_heads * head_dim * element_size * 2          # config.py:203
    total_budget_bytes = int(cache_budget * (prefill_len + max_tokens) * bytes_per_token)  # :206
    total_budget_tokens = total_budget_bytes // bytes_per_token          # :207
    if isinstance(local_window_size, float):                              # :216-222
        ceiled = math.ceil(local_window_size * total_budget_tokens)
        rem = ceiled % window_size
        if rem != 0:
            ceiled += window_size - rem
        local_tokens = ceiled
    else:
        local_tokens = local_window_size
    remaining = total_budget_tokens - num_sink_tokens - local_tokens      # :227
    if remaining < 0:
        raise ValueError(
            f"total_budget_tokens ({total_budget_tokens}) < num_sink_tokens "
            f"({num_sink_tokens}) + local_tokens ({local_tokens}).")
    return Resolved(window_size, num_sink_tokens, local_tokens, remaining // window_size,
                    bytes_per_token, total_budget_bytes, total_budget_tokens)


# ---------------------------------------------------------------------------
# 2. Window scoring  (scorer.py:17-109)
# ---------------------------------------------------------------------------


def reduce_token_scores_to_windows(token_scores: np.ndarray, num_sink: int,
                                   window_size: int) -> np.ndarray:
    """[..., S] per-key received attention -> [..., W] window sums.
    Strip sinks, zero-pad the trailing partial window, sum (scorer.py:51-90)."""
    post = token_scores[..., num_sink:]
    s_post = post.shape[-1]
    rem = s_post % window_size
    if rem:
        pad = np.zeros(post.shape[:-1] + (window_size - rem,), dtype=post.dtype)
        post = np.concatenate([post, pad], axis=-1)
    w = post.shape[-1] // window_size
    return post.reshape(post.shape[:-1] + (w, window_size)).sum(axis=-1, dtype=post.dtype)


def compute_window_scores(attn: np.ndarray, num_sink: int, window_size: int) -> np.ndarray:
    """[B,H,T,S] attention -> [B,H,W] (scorer.py:17-48): sum over query rows."""
    return reduce_token_scores_to_windows(attn.sum(axis=-2, dtype=attn.dtype), num_sink, window_size)


# ---------------------------------------------------------------------------
# 3. Selection  (policy.py:81-209)
# ---------------------------------------------------------------------------


def head_mean(window_scores: np.ndarray) -> np.ndarray:
    """Mean over query heads, fp32, accumulated in head order h=0..Hq-1
    (policy.py:112 ``window_scores.mean(dim=1)``)."""
    ws = np.asarray(window_scores, dtype=np.float32)
    acc = np.zeros((ws.shape[0], ws.shape[2]), dtype=np.float32)
    for h in range(ws.shape[1]):
        acc = (acc + ws[:, h, :]).astype(np.float32)
    return (acc / np.float32(ws.shape[1])).astype(np.float32)


def retain_window_indices(window_scores: np.ndarray, top_k_windows: int,
                          local_windows: int) -> np.ndarray:
    """[B,Hq,W] -> [B, k + local_w] retained window indices (policy.py:81-146).

    Top-k over the evictable prefix ``[0, W - local_w)`` of the head-mean
    scores, ties broken by the lowest window index (``torch.topk`` leaves tie
    order unspecified; this build fixes it), re-sorted chronologically, then
    the local windows appended.  Edge cases k==0 and k>=evictable follow
    policy.py:120-132."""
    B, _, W = window_scores.shape
    local_w = min(local_windows, W)
    evictable = W - local_w
    k = min(top_k_windows, evictable)
    local_idx = np.broadcast_to(np.arange(W - local_w, W, dtype=np.int64), (B, local_w))
    if k == 0 or evictable == 0:
        return np.ascontiguousarray(local_idx)
    if k >= evictable:
        return np.ascontiguousarray(np.broadcast_to(np.arange(W, dtype=np.int64), (B, W)))
    mean = head_mean(window_scores)[:, :evictable]
    out = np.empty((B, k + local_w), dtype=np.int64)
    idx = np.arange(evictable)
    for b in range(B):
        order = np.lexsort((idx, -mean[b].astype(np.float64)))   # score desc, index asc
        out[b, :k] = np.sort(order[:k])
        out[b, k:] = local_idx[b]
    return out


def expand_to_token_indices(retained_window_idx: np.ndarray, num_sink: int, window_size: int,
                            total_tokens: int) -> np.ndarray:
    """Window indices -> token indices: sink prefix + window tokens, tokens at
    or beyond ``total_tokens`` dropped, rows truncated to the minimum valid
    count (policy.py:152-209)."""
    B, Wr = retained_window_idx.shape
    sink = np.broadcast_to(np.arange(num_sink, dtype=np.int64), (B, num_sink))
    tok = (num_sink + retained_window_idx[:, :, None] * window_size
           + np.arange(window_size, dtype=np.int64)).reshape(B, -1)
    all_idx = np.concatenate([sink, tok], axis=1)
    valid = all_idx < total_tokens
    min_valid = int(valid.sum(axis=1).min()) if B else 0
    out = np.empty((B, min_valid), dtype=np.int64)
    for b in range(B):
        order = np.argsort(~valid[b], kind="stable")
        out[b] = all_idx[b][order][:min_valid]
    return out


# ---------------------------------------------------------------------------
# 4. RoPE strip + re-apply in the KV dtype  (state.py:165-232 + HF rotate-half)
# ---------------------------------------------------------------------------


def rope_apply_kdtype(k: np.ndarray, cos: np.ndarray, sin: np.ndarray, dtype: str) -> np.ndarray:
    """transformers ``apply_rotary_pos_emb`` on keys, op by op in ``dtype``:
    ``round(round(k*cos) + round(rotate_half(k)*sin))``.  ``k`` [..., T, D];
    ``cos``/``sin`` broadcastable [..., T, D] already rounded to ``dtype``."""
    D = k.shape[-1]
    h = D // 2
    rot = np.concatenate([-k[..., h:], k[..., :h]], axis=-1)
    t1 = round_to((k * cos).astype(np.float32), dtype)
    t2 = round_to((rot * sin).astype(np.float32), dtype)
    return round_to((t1 + t2).astype(np.float32), dtype)


_POOL = None


def _pool():
    """Host threads for elementwise work on large arrays (numpy's ufuncs
    release the GIL, so slices run in parallel; results are unchanged)."""
    global _POOL
    if _POOL is None:
        import concurrent.futures
        import os
        _POOL = concurrent.futures.ThreadPoolExecutor(max_workers=os.cpu_count() or 1)
    return _POOL


def rerotate_keys(k: np.ndarray, old_pos: np.ndarray, new_pos: np.ndarray,
                  cos_tab: np.ndarray, sin_tab: np.ndarray, dtype: str) -> np.ndarray:
    """Strip RoPE at ``old_pos`` then re-apply at ``new_pos`` (state.py:199-221);
    see :func:`rerotate_keys_serial`.  Large caches are split over kv heads
    and host threads (each head's arithmetic is independent)."""
    B, H = k.shape[0], k.shape[1]
    if k.size < (1 << 20) or H == 1:
        return rerotate_keys_serial(k, old_pos, new_pos, cos_tab, sin_tab, dtype)
    parts = list(_pool().map(lambda h: rerotate_keys_serial(k[:, h:h + 1], old_pos, new_pos, cos_tab,
                                                            sin_tab, dtype), range(H)))
    return np.concatenate(parts, axis=1)


def rerotate_keys_serial(k: np.ndarray, old_pos: np.ndarray, new_pos: np.ndarray,
                         cos_tab: np.ndarray, sin_tab: np.ndarray, dtype: str) -> np.ndarray:
    """Strip RoPE at ``old_pos`` then re-apply at ``new_pos`` (state.py:199-221).

    ``k`` [B,H,T,D] (values representable in ``dtype``), positions [B,T].
    ``cos_tab``/``sin_tab`` are the model rotary module's fp32 output for
    positions 0..N-1, shape [N, D] (HF ``cos = emb.cos()*scaling``); the
    reference rounds them to the KV dtype (``cos.to(x.dtype)``) before use."""
    c_old = round_to(cos_tab[old_pos], dtype)[:, None]      # [B,1,T,D]
    s_old = round_to(sin_tab[old_pos], dtype)[:, None]
    c_new = round_to(cos_tab[new_pos], dtype)[:, None]
    s_new = round_to(sin_tab[new_pos], dtype)[:, None]
    un = rope_apply_kdtype(k, c_old, -s_old, dtype)         # state.py:206-208
    return rope_apply_kdtype(un, c_new, s_new, dtype)       # state.py:219-221


# ---------------------------------------------------------------------------
# 5. int4 tier (design.md:130-187; group-32 asymmetric, fp16 scale/zero)
# ---------------------------------------------------------------------------

QGROUP = 32
PAGE_TOKENS = 8


def quantize_group32(x: np.ndarray) -> Tuple[np.ndarray, np.ndarray, np.ndarray]:
    """x [..., D] fp32 -> (codes uint8 [..., D], scale fp16 [..., D/32], zero fp16 [..., D/32])."""
    x = np.asarray(x, dtype=np.float32)
    D = x.shape[-1]
    g = x.reshape(x.shape[:-1] + (D // QGROUP, QGROUP))
    mn = g.min(axis=-1)
    mx = g.max(axis=-1)
    scale16 = ((mx - mn).astype(np.float32) / np.float32(15.0)).astype(np.float32).astype(np.float16)
    zero16 = mn.astype(np.float16)
    s = scale16.astype(np.float32)[..., None]
    z = zero16.astype(np.float32)[..., None]
    with np.errstate(divide="ignore", invalid="ignore"):
        q = ((g - z).astype(np.float32) / s).astype(np.float32)
    q = np.rint(q)
    q = np.where(s == 0, 0.0, q)
    q = np.clip(q, 0, 15)
    codes = q.astype(np.uint8).reshape(x.shape)
    return codes, scale16, zero16


def dequant_group32(codes: np.ndarray, scale16: np.ndarray, zero16: np.ndarray) -> np.ndarray:
    D = codes.shape[-1]
    c = codes.reshape(codes.shape[:-1] + (D // QGROUP, QGROUP)).astype(np.float32)
    v = c * scale16.astype(np.float32)[..., None] + zero16.astype(np.float32)[..., None]
    return v.reshape(codes.shape).astype(np.float32)


def page_bytes(head_dim: int) -> int:
    """Bytes of one int4 page (8 tokens, K and V, codes + fp16 scale/zero)."""
    return 2 * PAGE_TOKENS * (head_dim // 2 + (head_dim // QGROUP) * 4)


def pack_page(kc, ks, kz, vc, vs, vz) -> np.ndarray:
    """Pack one 8-token page of K and V codes into the device byte layout.

    K codes: [row r][lane t (4)][word w (D/32)] uint32; word w nibble i (0..3)
    holds channel ``2t + 8(4w+i)``, nibble i+4 channel ``2t + 8(4w+i) + 1``.
    K scales: [row r][group][scale, zero] fp16.
    V codes: [pair t (4)][row g (8)][word w] uint32; nibble i holds token 2t
    at channel ``g + 8(4w+i)``, nibble i+4 token 2t+1 at the same channel.
    V scales: [pair t][group][s(2t), s(2t+1), z(2t), z(2t+1)] fp16.
    This is the operand order of an m16n8k16 MMA fragment, so a page is read
    with one vector load per thread and no shuffles."""
    D = kc.shape[-1]
    NW = D // QGROUP
    kwords = np.zeros((PAGE_TOKENS, 4, NW), dtype=np.uint32)
    for r in range(PAGE_TOKENS):
        for t in range(4):
            for w in range(NW):
                word = 0
                for i in range(4):
                    ch = 2 * t + 8 * (4 * w + i)
                    word |= int(kc[r, ch]) << (4 * i)
                    word |= int(kc[r, ch + 1]) << (4 * (i + 4))
                kwords[r, t, w] = word
    kscl = np.zeros((PAGE_TOKENS, NW, 2), dtype=np.float16)
    kscl[:, :, 0] = ks
    kscl[:, :, 1] = kz
    vwords = np.zeros((4, 8, NW), dtype=np.uint32)
    for t in range(4):
        for g in range(8):
            for w in range(NW):
                word = 0
                for i in range(4):
                    ch = g + 8 * (4 * w + i)
                    word |= int(vc[2 * t, ch]) << (4 * i)
                    word |= int(vc[2 * t + 1, ch]) << (4 * (i + 4))
                vwords[t, g, w] = word
    vscl = np.zeros((4, NW, 4), dtype=np.float16)
    for t in range(4):
        vscl[t, :, 0] = vs[2 * t]
        vscl[t, :, 1] = vs[2 * t + 1]
        vscl[t, :, 2] = vz[2 * t]
        vscl[t, :, 3] = vz[2 * t + 1]
    out = np.concatenate([kwords.view(np.uint8).ravel(), kscl.view(np.uint8).ravel(),
                          vwords.view(np.uint8).ravel(), vscl.view(np.uint8).ravel()])
    assert out.size == page_bytes(D)
    return out


def unpack_page(page: np.ndarray, D: int):
    """Inverse of :func:`pack_page` -> (kc, ks, kz, vc, vs, vz)."""
    NW = D // QGROUP
    o = 0
    n = PAGE_TOKENS * 4 * NW * 4
    kwords = page[o:o + n].view(np.uint32).reshape(PAGE_TOKENS, 4, NW); o += n
    n = PAGE_TOKENS * NW * 2 * 2
    kscl = page[o:o + n].view(np.float16).reshape(PAGE_TOKENS, NW, 2); o += n
    n = 4 * 8 * NW * 4
    vwords = page[o:o + n].view(np.uint32).reshape(4, 8, NW); o += n
    n = 4 * NW * 4 * 2
    vscl = page[o:o + n].view(np.float16).reshape(4, NW, 4); o += n
    kc = np.zeros((PAGE_TOKENS, D), dtype=np.uint8)
    vc = np.zeros((PAGE_TOKENS, D), dtype=np.uint8)
    for r in range(PAGE_TOKENS):
        for t in range(4):
            for w in range(NW):
                word = int(kwords[r, t, w])
                for i in range(4):
                    ch = 2 * t + 8 * (4 * w + i)
                    kc[r, ch] = (word >> (4 * i)) & 0xF
                    kc[r, ch + 1] = (word >> (4 * (i + 4))) & 0xF
    for t in range(4):
        for g in range(8):
            for w in range(NW):
                word = int(vwords[t, g, w])
                for i in range(4):
                    ch = g + 8 * (4 * w + i)
                    vc[2 * t, ch] = (word >> (4 * i)) & 0xF
                    vc[2 * t + 1, ch] = (word >> (4 * (i + 4))) & 0xF
    ks, kz = kscl[:, :, 0].copy(), kscl[:, :, 1].copy()
    vs = np.zeros((PAGE_TOKENS, NW), dtype=np.float16)
    vz = np.zeros((PAGE_TOKENS, NW), dtype=np.float16)
    for t in range(4):
        vs[2 * t], vs[2 * t + 1] = vscl[t, :, 0], vscl[t, :, 1]
        vz[2 * t], vz[2 * t + 1] = vscl[t, :, 2], vscl[t, :, 3]
    return kc, ks, kz, vc, vs, vz


def unpack_pages(pages: np.ndarray, D: int):
    """Vectorised :func:`unpack_page` over any leading shape: pages
    [..., page_bytes] uint8 -> (kc, ks, kz, vc, vs, vz) with shapes
    [..., 8, D] / [..., 8, D/32] (same layout rules as :func:`pack_page`)."""
    NW = D // QGROUP
    pages = np.ascontiguousarray(pages, dtype=np.uint8)
    lead = pages.shape[:-1]
    o = 0
    n = PAGE_TOKENS * 4 * NW * 4
    kw = pages[..., o:o + n].copy().view(np.uint32).reshape(lead + (PAGE_TOKENS, 4, NW)); o += n
    n = PAGE_TOKENS * NW * 2 * 2
    ksc = pages[..., o:o + n].copy().view(np.float16).reshape(lead + (PAGE_TOKENS, NW, 2)); o += n
    n = 4 * 8 * NW * 4
    vw = pages[..., o:o + n].copy().view(np.uint32).reshape(lead + (4, 8, NW)); o += n
    n = 4 * NW * 4 * 2
    vsc = pages[..., o:o + n].copy().view(np.float16).reshape(lead + (4, NW, 4))
    shifts = (4 * np.arange(8, dtype=np.uint32))
    knib = ((kw[..., None] >> shifts) & 0xF).astype(np.uint8)   # [..., r, t, w, nibble]
    vnib = ((vw[..., None] >> shifts) & 0xF).astype(np.uint8)   # [..., t, g, w, nibble]
    kc = np.zeros(lead + (PAGE_TOKENS, D), np.uint8)
    vc = np.zeros(lead + (PAGE_TOKENS, D), np.uint8)
    for t in range(4):
        for w in range(NW):
            for i in range(4):
                ch = 2 * t + 8 * (4 * w + i)
                kc[..., ch] = knib[..., t, w, i]
                kc[..., ch + 1] = knib[..., t, w, i + 4]
                c0 = 8 * (4 * w + i)
                vc[..., 2 * t, c0:c0 + 8] = vnib[..., t, :, w, i]
                vc[..., 2 * t + 1, c0:c0 + 8] = vnib[..., t, :, w, i + 4]
    ks, kz = ksc[..., 0].copy(), ksc[..., 1].copy()
    vs = np.zeros(lead + (PAGE_TOKENS, NW), np.float16)
    vz = np.zeros(lead + (PAGE_TOKENS, NW), np.float16)
    for t in range(4):
        vs[..., 2 * t, :], vs[..., 2 * t + 1, :] = vsc[..., t, :, 0], vsc[..., t, :, 1]
        vz[..., 2 * t, :], vz[..., 2 * t + 1, :] = vsc[..., t, :, 2], vsc[..., t, :, 3]
    return kc, ks, kz, vc, vs, vz


def to_page_frame(k: np.ndarray, old_pos: np.ndarray, cos_tab: np.ndarray,
                  sin_tab: np.ndarray, num_sink: int) -> np.ndarray:
    """Post-RoPE key (fp32 of the KV-dtype value) at ``old_pos`` -> the key in
    its page-relative frame ``R(r8) R(-old_pos) k`` with r8 = offset inside its
    8-token page (pages start at ``num_sink + 8m``), in fp32 with the operation order the CUDA path uses (no
    fused multiply-add).  Keys stored this way never change when positions
    are re-based (windows move as units), so the int4 grid stays pinned
    (design.md AMENDMENT 2: the tier is stored position-independent and
    rotated at read)."""
    D = k.shape[-1]
    h = D // 2
    x = k[..., :h].astype(np.float32)
    y = k[..., h:].astype(np.float32)
    c = cos_tab[old_pos][..., :h].astype(np.float32)
    s = sin_tab[old_pos][..., :h].astype(np.float32)
    xs = (x * c).astype(np.float32) + (y * s).astype(np.float32)
    ys = (y * c).astype(np.float32) - (x * s).astype(np.float32)
    r8 = (np.asarray(old_pos) - num_sink) % PAGE_TOKENS
    c8 = cos_tab[r8][..., :h].astype(np.float32)
    s8 = sin_tab[r8][..., :h].astype(np.float32)
    xf = (xs * c8).astype(np.float32) - (ys * s8).astype(np.float32)
    yf = (ys * c8).astype(np.float32) + (xs * s8).astype(np.float32)
    return np.concatenate([xf, yf], axis=-1).astype(np.float32)


def rotate_query_to_page(q: np.ndarray, page_pos: int, cos_tab: np.ndarray,
                         sin_tab: np.ndarray) -> np.ndarray:
    """``R(-P) q`` for a tier page starting at position P (fp32)."""
    D = q.shape[-1]
    h = D // 2
    x, y = q[..., :h].astype(np.float32), q[..., h:].astype(np.float32)
    c, s = cos_tab[page_pos][:h].astype(np.float32), sin_tab[page_pos][:h].astype(np.float32)
    return np.concatenate([(x * c + y * s), (y * c - x * s)], axis=-1).astype(np.float32)


# ---------------------------------------------------------------------------
# 6. Decode attention with per-window mass (eager math, fp32 softmax)
# ---------------------------------------------------------------------------


def eager_decode_attention(q: np.ndarray, k: np.ndarray, v: np.ndarray, scaling: float,
                           num_sink: int, window_size: int, dtype: str):
    """One decode step over an all-fp cache, the reference's eager path:
    ``softmax(q Kᵀ·scale, fp32).to(dtype) @ V`` with GQA by head repetition,
    and the per-window scores of that step (``compute_window_scores`` on the
    weights cast to the model dtype).  q [B,Hq,D]; k,v [B,Hkv,S,D].
    Returns (out [B,Hq,D] fp32, window_scores [B,Hq,W] fp32)."""
    B, Hq, D = q.shape
    Hkv, S = k.shape[1], k.shape[2]
    G = Hq // Hkv
    # query head h reads kv head h // G (repeat_kv); grouped instead of
    # materialised: [B, Hkv, G, D] @ [B, Hkv, D, S]
    qg = q.astype(np.float32, copy=False).reshape(B, Hkv, G, D)
    kf = k.astype(np.float32, copy=False)
    vf = v.astype(np.float32, copy=False)
    logits = np.matmul(qg, kf.transpose(0, 1, 3, 2)).reshape(B, Hq, S) * np.float32(scaling)
    m = logits.max(axis=-1, keepdims=True)
    e = np.exp((logits - m).astype(np.float32))
    p = (e / e.sum(axis=-1, keepdims=True)).astype(np.float32)
    p_d = round_to(p, dtype)
    out = np.matmul(p_d.reshape(B, Hkv, G, S), vf).reshape(B, Hq, D).astype(np.float32, copy=False)
    scores = reduce_token_scores_to_windows(p_d, num_sink, window_size)
    return out, scores


def tiered_decode_attention(q: np.ndarray, sinks_k: np.ndarray, sinks_v: np.ndarray,
                            tier_k: Optional[np.ndarray], tier_v: Optional[np.ndarray],
                            rest_k: np.ndarray, rest_v: np.ndarray, num_sink: int,
                            window_size: int, scaling: float, cos_tab=None, sin_tab=None):
    """Decode attention over [sinks | int4 tier | fp rest] with the window mass
    the scorer would compute from the fp32 weights.

    ``tier_k``/``tier_v`` are the *dequantized* tier keys (page frame) and
    values [B,Hkv,Nt,D] (Nt a multiple of 8); their logits use the query
    rotated to each page's start position.  Other keys are post-RoPE.
    Returns (out [B,Hq,D], mass [B,Hq,W]) in fp32 (mass unrounded)."""
    B, Hq, D = q.shape
    Hkv = rest_k.shape[1]
    G = Hq // Hkv
    qf = q.astype(np.float32)
    parts = []
    vparts = []
    nt = 0 if tier_k is None else tier_k.shape[2]
    s = num_sink
    # sinks
    ks = np.repeat(sinks_k, G, axis=1).astype(np.float32)
    parts.append(np.einsum("bhd,bhsd->bhs", qf, ks))
    vparts.append(np.repeat(sinks_v, G, axis=1).astype(np.float32))
    if nt:
        kt = np.repeat(tier_k, G, axis=1).astype(np.float32)
        lt = np.empty((B, Hq, nt), dtype=np.float32)
        for pg in range(nt // PAGE_TOKENS):
            qr = rotate_query_to_page(qf, s + PAGE_TOKENS * pg, cos_tab, sin_tab)
            sl = slice(PAGE_TOKENS * pg, PAGE_TOKENS * (pg + 1))
            lt[:, :, sl] = np.einsum("bhd,bhsd->bhs", qr, kt[:, :, sl])
        parts.append(lt)
        vparts.append(np.repeat(tier_v, G, axis=1).astype(np.float32))
    kr = np.repeat(rest_k, G, axis=1).astype(np.float32)
    parts.append(np.einsum("bhd,bhsd->bhs", qf, kr))
    vparts.append(np.repeat(rest_v, G, axis=1).astype(np.float32))
    logits = np.concatenate(parts, axis=-1).astype(np.float32) * np.float32(scaling)
    vall = np.concatenate(vparts, axis=2)
    m = logits.max(axis=-1, keepdims=True)
    e = np.exp((logits - m).astype(np.float32))
    p = (e / e.sum(axis=-1, keepdims=True)).astype(np.float32)
    out = np.einsum("bhs,bhsd->bhd", p, vall).astype(np.float32)
    mass = reduce_token_scores_to_windows(p, s, window_size)
    return out, mass


def tiered_decode_attention_grouped(q: np.ndarray, sinks_k: np.ndarray, sinks_v: np.ndarray,
                                    tier_k: Optional[np.ndarray], tier_v: Optional[np.ndarray],
                                    rest_k: np.ndarray, rest_v: np.ndarray, num_sink: int,
                                    window_size: int, scaling: float, cos_tab=None, sin_tab=None):
    """:func:`tiered_decode_attention` for long caches: the same math with the
    query heads grouped per kv head (no ``repeat_kv`` copy of K/V) and the
    per-page query rotation vectorised, so a 32k-token cache of 16 rows fits
    in a few hundred MB.  Same arguments and returns."""
    B, Hq, D = q.shape
    Hkv = rest_k.shape[1]
    G = Hq // Hkv
    h = D // 2
    qg = q.astype(np.float32).reshape(B, Hkv, G, D)
    parts, vparts = [], []
    parts.append(np.einsum("bkgd,bknd->bkgn", qg, sinks_k.astype(np.float32)))
    vparts.append(sinks_v.astype(np.float32))
    nt = 0 if tier_k is None else tier_k.shape[2]
    if nt:
        npg = nt // PAGE_TOKENS
        pos = num_sink + PAGE_TOKENS * np.arange(npg)
        c = cos_tab[pos][:, :h].astype(np.float32)           # [npg, h]
        s = sin_tab[pos][:, :h].astype(np.float32)
        x, y = qg[..., None, :h], qg[..., None, h:]           # [B,Hkv,G,1,h]
        qr = np.concatenate([x * c + y * s, y * c - x * s], axis=-1).astype(np.float32)  # [B,Hkv,G,npg,D]
        kt = tier_k.astype(np.float32).reshape(B, Hkv, npg, PAGE_TOKENS, D)
        lt = np.einsum("bkgpd,bkprd->bkgpr", qr, kt).reshape(B, Hkv, G, nt)
        parts.append(lt)
        vparts.append(tier_v.astype(np.float32))
    parts.append(np.einsum("bkgd,bknd->bkgn", qg, rest_k.astype(np.float32)))
    vparts.append(rest_v.astype(np.float32))
    logits = np.concatenate(parts, axis=-1).astype(np.float32) * np.float32(scaling)
    vall = np.concatenate(vparts, axis=2)
    m = logits.max(axis=-1, keepdims=True)
    e = np.exp((logits - m).astype(np.float32))
    p = (e / e.sum(axis=-1, keepdims=True)).astype(np.float32)
    out = np.einsum("bkgn,bknd->bkgd", p, vall).astype(np.float32).reshape(B, Hq, D)
    mass = reduce_token_scores_to_windows(p.reshape(B, Hq, -1), num_sink, window_size)
    return out, mass


# ---------------------------------------------------------------------------
# 7. Cache orchestration (cache.py:110-293) — reference mode and int4-tier mode
# ---------------------------------------------------------------------------


class OracleCache:
    """Per-layer cache state machine of ``WindowedCache.update`` for one layer.

    Reference mode (``tier=False``) keeps every retained token in the KV dtype
    and re-rotates all kept keys on each eviction, exactly as state.py does.
    Tier mode keeps sinks and the windows after the tier (local + appended)
    in the KV dtype (re-rotated like the reference) and stores kept evictable
    windows as int4 pages in their page-relative frame.

    Scores are supplied per step (what the hook would write); ``add_scores``
    follows cache.py:163-228 (pad on growth, extend original ids from the
    running counter)."""

    def __init__(self, resolved: Resolved, dtype: str, cos_tab: np.ndarray, sin_tab: np.ndarray,
                 tier: bool = False):
        self.r = resolved
        self.dtype = dtype
        self.cos, self.sin = cos_tab, sin_tab
        self.tier = tier
        self.local_windows = resolved.local_tokens // resolved.window_size
        self.k = None            # fp part: [B,H,n_fp,D] logical order minus tier
        self.v = None
        self.n_tier_tokens = 0
        self.tier_codes = None   # (kc, ks, kz, vc, vs, vz) arrays over tier tokens
        self.window_scores = None
        self.original_window_ids = None
        self.next_id = 0
        self.step = 0
        self.prefill_done = False
        self.last_retained = None

    @property
    def seq_length(self) -> int:
        return 0 if self.k is None else self.k.shape[2] + self.n_tier_tokens

    def _fp_positions(self) -> np.ndarray:
        s = self.r.num_sink_tokens
        n = self.k.shape[2]
        pos = np.arange(n)
        return np.where(pos < s, pos, pos + self.n_tier_tokens)

    def append(self, k_new: np.ndarray, v_new: np.ndarray) -> None:
        """state.py:68-119 (positions auto-increment: contiguous)."""
        k_new = round_to(k_new, self.dtype)
        v_new = round_to(v_new, self.dtype)
        if self.k is None:
            self.k, self.v = k_new.copy(), v_new.copy()
        else:
            self.k = np.concatenate([self.k, k_new], axis=2)
            self.v = np.concatenate([self.v, v_new], axis=2)

    def add_scores(self, new: np.ndarray) -> None:
        """cache.py:163-228."""
        new = np.asarray(new, dtype=np.float32)
        if self.window_scores is None:
            self.window_scores = new.copy()
            B, W = new.shape[0], new.shape[-1]
            self.original_window_ids = np.broadcast_to(np.arange(W, dtype=np.int64), (B, W)).copy()
            self.next_id = W
            return
        W_old, W_new = self.window_scores.shape[-1], new.shape[-1]
        if W_new > W_old:
            pad = np.zeros(self.window_scores.shape[:2] + (W_new - W_old,), dtype=np.float32)
            self.window_scores = np.concatenate([self.window_scores, pad], axis=-1)
            extra = np.arange(self.next_id, self.next_id + W_new - W_old, dtype=np.int64)
            self.original_window_ids = np.concatenate(
                [self.original_window_ids,
                 np.broadcast_to(extra, (self.original_window_ids.shape[0], extra.size))], axis=1)
            self.next_id += W_new - W_old
        elif W_new < W_old:
            pad = np.zeros(new.shape[:2] + (W_old - W_new,), dtype=np.float32)
            new = np.concatenate([new, pad], axis=-1)
        self.window_scores = (self.window_scores + new).astype(np.float32)

    def update(self, k_new, v_new, scores=None) -> bool:
        """One ``update()`` call: append, accumulate, maybe evict.  Returns
        True when an eviction ran."""
        self.append(k_new, v_new)
        is_prefill = not self.prefill_done
        self.prefill_done = True
        if scores is not None:
            self.add_scores(scores)
        evicted = False
        if (not is_prefill and self.step > 0 and self.step % self.r.window_size == 0
                and self.window_scores is not None):
            self.evict()
            evicted = True
        if not is_prefill:
            self.step += 1
        return evicted

    def evict(self) -> None:
        r = self.r
        s, ws = r.num_sink_tokens, r.window_size
        T_old = self.seq_length
        retained = retain_window_indices(self.window_scores, r.top_k_windows, self.local_windows)
        tok = expand_to_token_indices(retained, s, ws, T_old)
        self.last_retained = retained
        B = tok.shape[0]
        T_ret = tok.shape[1]
        W = self.window_scores.shape[-1]
        local_w = min(self.local_windows, W)
        kprime = retained.shape[1] - local_w
        new_pos = np.broadcast_to(np.arange(T_ret), (B, T_ret))
        if not self.tier:
            k_sel = np.take_along_axis(self.k, tok[:, None, :, None], axis=2)
            v_sel = np.take_along_axis(self.v, tok[:, None, :, None], axis=2)
            self.k = rerotate_keys(k_sel, tok, new_pos, self.cos, self.sin, self.dtype)
            self.v = v_sel
        else:
            fp_pos = self._fp_positions()
            slot_of = {int(p): i for i, p in enumerate(fp_pos)}
            n_tw_old = self.n_tier_tokens // ws
            # fp tokens kept: sinks + local windows (retained[:, kprime:])
            n_local_tok = T_ret - s - kprime * ws
            fp_keep_pos = np.concatenate([tok[:, :s], tok[:, s + kprime * ws:]], axis=1)
            slots = np.vectorize(lambda p: slot_of[int(p)])(fp_keep_pos)
            k_sel = np.take_along_axis(self.k, slots[:, None, :, None], axis=2)
            v_sel = np.take_along_axis(self.v, slots[:, None, :, None], axis=2)
            newp = np.concatenate([np.broadcast_to(np.arange(s), (B, s)),
                                   np.broadcast_to(np.arange(s + kprime * ws, T_ret),
                                                   (B, n_local_tok))], axis=1)
            new_k = rerotate_keys(k_sel, fp_keep_pos, newp, self.cos, self.sin, self.dtype)
            # tier: kept evictable windows in order
            H, D = self.k.shape[1], self.k.shape[3]
            kc_o = self.tier_codes
            new_codes = [np.zeros((B, H, kprime * ws) + shp, dtype=dt) for shp, dt in
                         [((D,), np.uint8), ((D // QGROUP,), np.float16), ((D // QGROUP,), np.float16),
                          ((D,), np.uint8), ((D // QGROUP,), np.float16), ((D // QGROUP,), np.float16)]]
            for b in range(B):
                for j in range(kprime):
                    w = int(retained[b, j])
                    dst = slice(j * ws, (j + 1) * ws)
                    if w < n_tw_old:
                        src = slice(w * ws, (w + 1) * ws)
                        for a in range(6):
                            new_codes[a][b, :, dst] = kc_o[a][b, :, src]
                    else:
                        p0 = s + w * ws
                        sl = [slot_of[p0 + i] for i in range(ws)]
                        kk = self.k[b][:, sl, :].astype(np.float32)
                        vv = self.v[b][:, sl, :].astype(np.float32)
                        kf = to_page_frame(kk, np.arange(p0, p0 + ws)[None, :].repeat(H, 0),
                                           self.cos, self.sin, s)
                        kc, ks, kz = quantize_group32(kf)
                        vc, vs, vz = quantize_group32(vv)
                        for a, arr in enumerate((kc, ks, kz, vc, vs, vz)):
                            new_codes[a][b, :, dst] = arr
            self.tier_codes = tuple(new_codes)
            self.n_tier_tokens = kprime * ws
            self.k = new_k
            self.v = v_sel
        idx_w = retained[:, None, :]
        self.window_scores = np.take_along_axis(
            self.window_scores, np.broadcast_to(idx_w, (B, self.window_scores.shape[1], retained.shape[1])),
            axis=-1).copy()
        self.original_window_ids = np.take_along_axis(self.original_window_ids, retained, axis=1).copy()

    # -- helpers for tier-mode decode attention ---------------------------
    def tier_dequant(self):
        if self.n_tier_tokens == 0:
            return None, None
        kc, ks, kz, vc, vs, vz = self.tier_codes
        return dequant_group32(kc, ks, kz), dequant_group32(vc, vs, vz)

    def materialize(self):
        """Every retained token as plain keys and values [B,H,T,D] in logical
        order (the reference's ``CacheState.key_states``/``value_states``,
        state.py:20-35): fp tokens as stored; tier tokens dequantised
        (``code*scale + zero`` in fp32) with their keys rotated from the page
        frame to their current position, ``R(P)`` of the stored vector for a
        page starting at P (fp32, no fused multiply-add), then rounded to the
        KV dtype."""
        if self.n_tier_tokens == 0:
            return self.k.copy(), self.v.copy()
        s = self.r.num_sink_tokens
        n_s = min(s, self.k.shape[2])
        tk, tv = self.tier_dequant()
        D = tk.shape[-1]
        h = D // 2
        pos = s + PAGE_TOKENS * (np.arange(self.n_tier_tokens) // PAGE_TOKENS)
        c = self.cos[pos][:, :h].astype(np.float32)
        sn = self.sin[pos][:, :h].astype(np.float32)
        x, y = tk[..., :h], tk[..., h:]
        kx = ((x * c).astype(np.float32) - (y * sn).astype(np.float32)).astype(np.float32)
        ky = ((y * c).astype(np.float32) + (x * sn).astype(np.float32)).astype(np.float32)
        keys = round_to(np.concatenate([kx, ky], axis=-1), self.dtype)
        vals = round_to(tv, self.dtype)
        return (np.concatenate([self.k[:, :, :n_s], keys, self.k[:, :, n_s:]], axis=2),
                np.concatenate([self.v[:, :, :n_s], vals, self.v[:, :, n_s:]], axis=2))

    def decode_attention(self, q: np.ndarray, scaling: float):
        """Attention of a decode query over the current cache -> (out, mass)."""
        s = self.r.num_sink_tokens
        n_s = min(s, self.k.shape[2])
        tk, tv = self.tier_dequant()
        return tiered_decode_attention(q, self.k[:, :, :n_s], self.v[:, :, :n_s], tk, tv,
                                       self.k[:, :, n_s:], self.v[:, :, n_s:], s,
                                       self.r.window_size, scaling, self.cos, self.sin)


# ---------------------------------------------------------------------------
# 8. Prefill column mass (flash hooks.py:245-290, causal, T == S)
# ---------------------------------------------------------------------------


def prefill_window_scores(q: np.ndarray, k: np.ndarray, scaling: float, num_sink: int,
                          window_size: int, dtype: str = "f32") -> np.ndarray:
    """Causal prefill scoring: ``softmax(qKᵀ·scale, causal)`` summed over the
    query rows then reduced to windows.  q [B,Hq,T,D], k [B,Hkv,T,D]."""
    B, Hq, T, D = q.shape
    G = Hq // k.shape[1]
    kx = np.repeat(k, G, axis=1).astype(np.float32)
    tok = np.zeros((B, Hq, T), dtype=np.float32)
    mask = np.triu(np.ones((T, T), dtype=bool), 1)
    for b in range(B):
        for h in range(Hq):
            a = (q[b, h].astype(np.float32) @ kx[b, h].T).astype(np.float32) * np.float32(scaling)
            a[mask] = -np.inf
            a = a - a.max(axis=-1, keepdims=True)
            e = np.exp(a)
            p = round_to((e / e.sum(axis=-1, keepdims=True)).astype(np.float32), dtype)
            tok[b, h] = p.sum(axis=0, dtype=np.float32)
    return reduce_token_scores_to_windows(tok, num_sink, window_size)


def rope_tables(inv_freq: np.ndarray, n_pos: int, scaling: float = 1.0):
    """fp32 cos/sin [n_pos, D] as HF's rotary module builds them
    (``freqs = inv_freq ⊗ pos``; ``emb = cat(freqs, freqs)``)."""
    pos = np.arange(n_pos, dtype=np.float32)
    freqs = (pos[:, None] * inv_freq[None, :].astype(np.float32)).astype(np.float32)
    emb = np.concatenate([freqs, freqs], axis=-1)
    return (np.cos(emb) * np.float32(scaling)).astype(np.float32), \
        (np.sin(emb) * np.float32(scaling)).astype(np.float32)
