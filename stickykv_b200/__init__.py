"""stickykv_b200 — B200-native windowed-eviction KV cache (drop-in for StickyKV's
``get_cache_classes`` backends).

Public API (same names as the reference's modules/windowed_cache/__init__.py):
``WindowedCache``, ``WindowedCacheConfig``, ``ResolvedConfig``, ``Telemetry``,
``NullTelemetry``, ``install_score_hooks``, ``HookHandles``, plus
``get_cache_classes`` / ``validate_backend_attn_pairing``; and
``DecodeGraphs`` (CUDA-graph replay of steady-state decode steps).
"""

from .cache import WindowedCache
from .cache_factory import ConfigValidationError, get_cache_classes, validate_backend_attn_pairing
from .config import ResolvedConfig, WindowedCacheConfig
from .graphs import DecodeGraphs
from .hooks import HookHandles, install_score_hooks
from .telemetry import NullTelemetry, Telemetry

__all__ = [
    "WindowedCache", "WindowedCacheConfig", "ResolvedConfig", "Telemetry", "NullTelemetry",
    "install_score_hooks", "HookHandles", "get_cache_classes", "validate_backend_attn_pairing",
    "ConfigValidationError", "DecodeGraphs",
]
