"""Shared helpers for the GPU parity tests (oracle = checker)."""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

from oracle import skv_oracle as O

TORCH_DT = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}
# Attention-output tolerance per KV dtype (max-abs vs the fp32 eager restatement).
OUT_TOL = {"f32": 2e-5, "f16": 2e-3, "bf16": 8e-3}
_MANT_BITS = {"f16": 10, "bf16": 7}


def assert_out_close(actual, desired, dt: str, err_msg: str = "") -> None:
    """Attention output against the oracle's fp32 output.

    The reference's eager path returns the model dtype, so the oracle output
    is rounded to the KV dtype first.  The two must then agree within the
    max-abs tolerance OUT_TOL[dt] (2e-3 fp16, 8e-3 bf16, 2e-5 fp32), or within
    one unit in the last place of the dtype where that unit is larger (bf16
    values of magnitude >= 2, fp16 >= 4): two correctly rounded results of
    sums that differ only in summation order can land one ulp apart."""
    a = np.asarray(actual, dtype=np.float32)
    d = O.round_to(np.asarray(desired, dtype=np.float32), dt)
    tol = np.full(d.shape, OUT_TOL[dt], dtype=np.float32)
    if dt in _MANT_BITS:
        mag = np.maximum(np.abs(d), np.float32(1e-30))
        ulp = np.exp2(np.floor(np.log2(mag)) - _MANT_BITS[dt]).astype(np.float32)
        tol = np.maximum(tol, ulp)
    bad = ~(np.abs(a - d) <= tol)
    if bad.any():
        i = np.unravel_index(np.argmax(np.where(bad, np.abs(a - d) - tol, -np.inf)), a.shape)
        raise AssertionError(f"{err_msg}: {int(bad.sum())}/{a.size} outside tolerance; worst at {i}: "
                             f"actual {a[i]!r} desired {d[i]!r} tol {tol[i]!r}")


@dataclass
class ModelCfg:
    num_attention_heads: int
    num_key_value_heads: int
    hidden_size: int
    head_dim: int


class TableRoPE(torch.nn.Module):
    """Rotary module returning fixed fp32 tables (so the cache and the oracle
    see bit-identical cos/sin).  ``cos``/``sin`` are [N, D] numpy arrays."""

    def __init__(self, cos: np.ndarray, sin: np.ndarray):
        super().__init__()
        self.cos = torch.from_numpy(np.ascontiguousarray(cos, np.float32))
        self.sin = torch.from_numpy(np.ascontiguousarray(sin, np.float32))

    def forward(self, x, position_ids):
        # the cache asks for headroom past the last real position; rows past
        # the table repeat its last row and are never read for real tokens
        pos = position_ids.to("cpu").long().clamp(max=self.cos.shape[0] - 1)
        c = self.cos[pos].to(x.device, x.dtype)
        s = self.sin[pos].to(x.device, x.dtype)
        return c, s


def rope_tables(theta: float, D: int, n: int):
    inv = (1.0 / (theta ** (np.arange(0, D, 2, dtype=np.int64).astype(np.float32) / D))).astype(np.float32)
    return O.rope_tables(inv, n)


def to_np(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().cpu().numpy() if t.is_floating_point() else t.detach().cpu().numpy()


def rand(shape, dt, gen, scale=1.0):
    return (torch.randn(*shape, generator=gen) * scale).to(TORCH_DT[dt])


def make_cache(dt, B, Hkv, Hq, D, P, M, cos, sin, ws=8, s=4, local=0.25, budget=0.4, tier=False,
               num_layers=1):
    from stickykv_b200 import WindowedCache, WindowedCacheConfig
    cfg = WindowedCacheConfig(window_size=ws, num_sink_tokens=s, local_window_size=local,
                              cache_budget=budget, int4_tier=tier)
    return WindowedCache(cfg, P, ModelCfg(Hq, Hkv, Hq * D, D), TORCH_DT[dt], TableRoPE(cos, sin),
                         num_layers=num_layers, max_tokens=M)


def tier_codes(cache, layer=0, rows=None):
    """Unpack the logical int4 tier of a cache (first ``rows`` rows) into
    oracle-shaped arrays."""
    st = cache._states[layer]
    side = st.sides[st.cur]
    B = st.B if rows is None else rows
    pages = st.pages[:B].cpu().numpy()
    table = side.table[:B].cpu().numpy()
    H = st.Hkv
    n = st.tier_pages
    D = st.D
    out = [np.zeros((B, H, n * 8, D), np.uint8), np.zeros((B, H, n * 8, D // 32), np.float16),
           np.zeros((B, H, n * 8, D // 32), np.float16), np.zeros((B, H, n * 8, D), np.uint8),
           np.zeros((B, H, n * 8, D // 32), np.float16), np.zeros((B, H, n * 8, D // 32), np.float16)]
    for b in range(B):
        for h in range(H):
            for pg in range(n):
                parts = O.unpack_page(pages[b, h, table[b, pg]], D)
                for a in range(6):
                    out[a][b, h, pg * 8:(pg + 1) * 8] = parts[a]
    return tuple(out)


def fp_parts(cache, layer=0):
    """(sinks_k, sinks_v, rest_k, rest_v) of a cache's fp store as fp32 numpy."""
    st = cache._states[layer]
    side = st.sides[st.cur]
    s = min(st.num_sink, st.T)
    s_pad = (st.num_sink + 7) // 8 * 8
    rest = st.T - s - st.tier_pages * 8
    k = to_np(side.k)
    v = to_np(side.v)
    return k[:, :, :s], v[:, :, :s], k[:, :, s_pad:s_pad + rest], v[:, :, s_pad:s_pad + rest]


def tier_codes_all(cache, layer=0):
    """Vectorised :func:`tier_codes` over every row and kv head: the logical
    int4 tier (pages in table order) as oracle-shaped arrays
    (kc, ks, kz, vc, vs, vz), each [B, Hkv, pages*8, ...]."""
    st = cache._states[layer]
    side = st.sides[st.cur]
    n = st.tier_pages
    pages = st.pages.cpu().numpy()
    table = side.table[:, :n].cpu().numpy().astype(np.int64)
    logical = np.take_along_axis(pages, table[:, None, :, None], axis=2)   # [B, H, n, PB]
    parts = O.unpack_pages(logical, st.D)
    return tuple(a.reshape(a.shape[:2] + (n * 8,) + a.shape[4:]) for a in parts)
