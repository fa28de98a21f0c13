"""Telemetry hook point of the cache (reference modules/windowed_cache/telemetry.py:18-106).

``NullTelemetry`` (the default) does nothing and costs nothing on the hot
path: the cache only builds the token-level retain indices when the recorder
is a real ``Telemetry``.  ``Telemetry`` keeps host copies of the scores and
retained token indices at every eviction, for parity and faithfulness runs.
"""

from __future__ import annotations

from typing import Any, Dict, List, Optional

from torch import Tensor


class Telemetry:
    """Per-layer list of snapshots; memory grows with layers x windows x evictions."""

    enabled = True

    def __init__(self, num_layers: int) -> None:
        self.num_layers = num_layers
        self._records: Dict[int, List[Dict[str, Any]]] = {i: [] for i in range(num_layers)}

    def record_scores(self, layer_idx: int, step: int, window_scores: Tensor,
                      retain_indices: Optional[Tensor] = None) -> None:
        rec: Dict[str, Any] = {"step": step, "window_scores": window_scores.detach().cpu().clone()}
        if retain_indices is not None:
            rec["retain_indices"] = retain_indices.detach().cpu().clone()
        self._records.setdefault(layer_idx, []).append(rec)

    def record_cache_state(self, layer_idx: int, step: int, key_states: Tensor,
                           value_states: Tensor, position_ids: Tensor) -> None:
        self._records.setdefault(layer_idx, []).append({
            "step": step,
            "key_states": key_states.detach().cpu().clone(),
            "value_states": value_states.detach().cpu().clone(),
            "position_ids": position_ids.detach().cpu().clone(),
        })

    def get_records(self, layer_idx: int) -> List[Dict[str, Any]]:
        return self._records.get(layer_idx, [])

    def clear(self) -> None:
        for recs in self._records.values():
            recs.clear()


class NullTelemetry(Telemetry):
    """No-op recorder (the default)."""

    enabled = False

    def __init__(self, num_layers: int = 0) -> None:
        self.num_layers = num_layers
        self._records = {}

    def record_scores(self, *args: Any, **kwargs: Any) -> None:
        return None

    def record_cache_state(self, *args: Any, **kwargs: Any) -> None:
        return None

    def get_records(self, layer_idx: int) -> List[Dict[str, Any]]:
        return []

    def clear(self) -> None:
        return None
