"""Backend selection, same API as the reference's utils/cache_factory.py:110-197.

``get_cache_classes("b200")`` returns ``(WindowedCache, WindowedCacheConfig,
install_score_hooks)`` of this package.  The reference's own backends
(``"flash_attn"``, ``"eager"``) are not provided here: this package only
replaces the hot path.  A reference checkout adds one branch to its
``get_cache_classes`` that imports this package and returns this trio.
"""

from __future__ import annotations

from typing import Callable, Tuple, Type


class ConfigValidationError(ValueError):
    """Raised when a config value is invalid (reference utils/config.py:24)."""


BACKEND = "b200"
_BACKEND_TO_ATTN_IMPL = {BACKEND: ("stickykv_b200",)}


def get_cache_classes(backend: str) -> Tuple[Type, Type, Callable]:
    """Return ``(CacheClass, ConfigClass, install_hooks)`` for ``backend``."""
    if backend == BACKEND:
        try:
            from .cache import WindowedCache
            from .config import WindowedCacheConfig
            from .hooks import install_score_hooks
        except ImportError as e:  # pragma: no cover
            raise ConfigValidationError(f"b200 backend unavailable: {e}") from e
        return WindowedCache, WindowedCacheConfig, install_score_hooks
    raise ConfigValidationError(f"Unknown cache backend: {backend!r}.  Must be 'b200'.")


def validate_backend_attn_pairing(backend: str, attn_implementation: str) -> None:
    """Fail fast on a backend / attention-implementation mismatch."""
    if backend not in _BACKEND_TO_ATTN_IMPL:
        raise ConfigValidationError(f"Unknown cache backend: {backend!r}.  Must be 'b200'.")
    allowed = _BACKEND_TO_ATTN_IMPL[backend]
    if attn_implementation not in allowed:
        raise ConfigValidationError(
            f"Cache backend {backend!r} requires attn_implementation in {allowed!r}, "
            f"but got {attn_implementation!r}.  Fix your config.")
