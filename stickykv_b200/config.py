"""Cache configuration: the user-facing ``WindowedCacheConfig`` and its
resolved integer form ``ResolvedConfig``.

Same fields, validation rules and error messages as the reference plugin
(modules/windowed_cache/config.py:22-244), so reference call sites construct
it unchanged.  One field is added with a default that keeps reference
behaviour: ``int4_tier`` stores the kept evictable windows as group-32 int4
pages instead of the KV dtype (design.md:14-22 of the reference describes
this tier; the reference never implemented it).
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Any, Union

import torch


@dataclass(frozen=True)
class ResolvedConfig:
    """Concrete token counts derived from the byte budget
    (reference modules/windowed_cache/config.py:22-36)."""

    window_size: int
    num_sink_tokens: int
    local_tokens: int
    top_k_windows: int
    bytes_per_token: int
    total_budget_bytes: int
    total_budget_tokens: int


def _is_int(x: Any) -> bool:
    return isinstance(x, int) and not isinstance(x, bool)


@dataclass
class WindowedCacheConfig:
    """User configuration of the windowed KV cache.

    window_size        tokens per scoring window (> 0)
    num_sink_tokens    tokens always kept at the start (>= 0)
    local_window_size  int: local tokens (multiple of window_size);
                       float in (0, 1]: fraction of the *budget*, ceiled and
                       snapped up to a window multiple
    cache_budget       fraction in (0, 1] of full-cache memory to keep (float)
    track_scores       telemetry switch (default False)
    int4_tier          keep the selected evictable windows as int4 pages
                       (default False: every kept token stays in the KV dtype,
                       as in the reference)
    """

    window_size: int
    num_sink_tokens: int
    local_window_size: Union[int, float]
    cache_budget: float
    track_scores: bool = False
    int4_tier: bool = False

    def __post_init__(self) -> None:
        ws = self.window_size
        if not _is_int(ws):
            raise ValueError(f"window_size must be a positive int, got {ws!r}")
        if ws <= 0:
            raise ValueError(f"window_size must be > 0, got {ws}")
        ns = self.num_sink_tokens
        if not _is_int(ns):
            raise ValueError(f"num_sink_tokens must be a non-negative int, got {ns!r}")
        if ns < 0:
            raise ValueError(f"num_sink_tokens must be >= 0, got {ns}")
        cb = self.cache_budget
        if isinstance(cb, bool):
            raise ValueError(
                f"cache_budget must be a float in (0, 1], got bool {cb!r}. "
                f"bool is rejected because it subclasses int.")
        if isinstance(cb, int):
            raise ValueError(
                f"cache_budget must be a float ratio in (0, 1], got int {cb}. "
                f"Use e.g. 0.40 instead of 40.")
        if not isinstance(cb, float):
            raise ValueError(f"cache_budget must be a float in (0, 1], got {type(cb).__name__}")
        if not 0.0 < cb <= 1.0:
            raise ValueError(f"cache_budget must be in (0, 1], got {cb}")
        lw = self.local_window_size
        if isinstance(lw, bool):
            raise ValueError("local_window_size must be int or float, got bool")
        if isinstance(lw, int):
            if lw <= 0:
                raise ValueError(f"local_window_size as int must be > 0, got {lw}")
            if lw % ws:
                raise ValueError(
                    f"local_window_size as int ({lw}) must be a multiple of window_size ({ws})")
        elif isinstance(lw, float):
            if not 0.0 < lw <= 1.0:
                raise ValueError(f"local_window_size as float must be in (0, 1], got {lw}")
        else:
            raise ValueError(f"local_window_size must be int or float, got {type(lw).__name__}")
        if not isinstance(self.int4_tier, bool):
            raise ValueError(f"int4_tier must be a bool, got {self.int4_tier!r}")
        if self.int4_tier and ws % 8:
            raise ValueError(f"int4_tier needs window_size to be a multiple of 8, got {ws}")

    def resolve(self, prefill_len: int, model_config: Any, kv_dtype: torch.dtype,
                max_tokens: int) -> ResolvedConfig:
        """Byte budget -> token counts (reference config.py:155-244).

        Sized against prefill + generation; the byte->token conversion floors,
        so the retained cache never exceeds the budget."""
        hkv = getattr(model_config, "num_key_value_heads",
                      getattr(model_config, "num_attention_heads", None))
        if hkv is None:
            raise ValueError("model_config must have num_key_value_heads or num_attention_heads")
        head_dim = getattr(model_config, "head_dim", None)
        if head_dim is None:
            nh = getattr(model_config, "num_attention_heads", None)
            hidden = getattr(model_config, "hidden_size", None)
            if nh is None or hidden is None:
                raise ValueError(
                    "model_config must provide head_dim or (num_attention_heads + hidden_size)")
            head_dim = hidden // nh
        esize = torch.empty((), dtype=kv_dtype).element_size()
        bpt = hkv * head_dim * esize * 2
        budget_bytes = int(self.cache_budget * (prefill_len + max_tokens) * bpt)
        budget_tokens = budget_bytes // bpt
        if isinstance(self.local_window_size, float):
            local = math.ceil(self.local_window_size * budget_tokens)
            local += (-local) % self.window_size
        else:
            local = self.local_window_size
        remaining = budget_tokens - self.num_sink_tokens - local
        if remaining < 0:
            raise ValueError(
                f"total_budget_tokens ({budget_tokens}) < "
                f"num_sink_tokens ({self.num_sink_tokens}) + local_tokens ({local}). "
                f"Increase cache_budget or reduce sink/local sizes.")
        return ResolvedConfig(
            window_size=self.window_size, num_sink_tokens=self.num_sink_tokens,
            local_tokens=local, top_k_windows=remaining // self.window_size,
            bytes_per_token=bpt, total_budget_bytes=budget_bytes, total_budget_tokens=budget_tokens)
