"""Shared helpers for the GPU parity tests (oracle = checker)."""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

from oracle import skv_oracle as O

TORCH_DT = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}
# Attention-output tolerance per KV dtype (max-abs vs the fp32 eager restatement).
OUT_TOL = {"f32": 2e-5, "f16": 2e-3, "bf16": 8e-3}


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
