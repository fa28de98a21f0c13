"""``install_score_hooks`` for the B200 backend.

The reference installs a forward hook that reads (eager,
modules/windowed_eager_cache/hooks.py:80-187) or recomputes (flash,
modules/windowed_cache/hooks.py:125-299) the attention weights after every
attention call.  Here the scoring is fused into the attention kernels, so
instead of a score hook this installs:

1. the query-position pre-hook (same contract as the reference, installed
   first, :160);
2. the ``stickykv_b200`` attention implementation on the model config, which
   routes each ``LlamaAttention``/``Qwen2Attention`` call to the cache's
   native prefill or decode attention (window mass accumulated in the same
   pass).

``HookHandles.remove()`` undoes both and is idempotent.
"""

from __future__ import annotations

import warnings
from dataclasses import dataclass, field
from typing import Any, Dict, List, Optional, Tuple

import torch
import torch.nn as nn

from .position_override import install_position_override_hook

ATTN_IMPLEMENTATION = "stickykv_b200"

try:
    from transformers.models.llama.modeling_llama import LlamaAttention
except ImportError:  # pragma: no cover
    LlamaAttention = None  # type: ignore[assignment,misc]
try:
    from transformers.models.qwen2.modeling_qwen2 import Qwen2Attention
except ImportError:  # pragma: no cover
    Qwen2Attention = None  # type: ignore[assignment,misc]


def _get_attn_classes() -> Tuple:
    return tuple(c for c in (LlamaAttention, Qwen2Attention) if c is not None)


def _extract_arg(args: Tuple, kwargs: Dict[str, Any], name: str, pos: int) -> Optional[Any]:
    """Forward argument by keyword, else by position, else None."""
    if name in kwargs:
        return kwargs[name]
    if len(args) > pos:
        return args[pos]
    return None


@dataclass
class HookHandles:
    """Installed hooks; ``remove()`` is idempotent."""

    _hook_handles: List[Any] = field(default_factory=list)
    _removed: bool = False

    def remove(self) -> None:
        if self._removed:
            return
        for handle in self._hook_handles:
            handle.remove()
        self._hook_handles.clear()
        self._removed = True


class _Restore:
    """Handle that undoes a module/config change on ``remove()``."""

    def __init__(self, fn) -> None:
        self._fn = fn

    def remove(self) -> None:
        if self._fn is not None:
            self._fn()
            self._fn = None


def stickykv_attention(module: nn.Module, query: torch.Tensor, key: torch.Tensor,
                       value: torch.Tensor, attention_mask: Optional[torch.Tensor],
                       scaling: Optional[float] = None, dropout: float = 0.0, **kwargs):
    """HF attention-interface function: prefill or one-token decode through
    the cache's native kernels.  Returns (attn_output [B,T,Hq,D], None)."""
    cache = getattr(module, "_skv_cache", None)
    if cache is None:
        raise RuntimeError(
            "stickykv_b200 attention needs install_score_hooks(model, cache, config) first")
    if attention_mask is not None:
        # the mask function registered with this implementation returns None
        # for every unpadded causal batch, so a mask here means padding
        raise NotImplementedError(
            "stickykv_b200 attends over every cached token of a row: padded batches "
            "(an attention_mask with masked positions) are not supported")
    layer = module.layer_idx
    if scaling is None:
        scaling = getattr(module, "scaling", query.shape[-1] ** -0.5)
    st = cache._states[layer]
    if st.last_update_prefill:
        return cache.prefill_attention(layer, query, key, value, scaling), None
    if query.shape[2] != 1:
        raise NotImplementedError("stickykv_b200 decodes one token per step after the prefill")
    return cache.decode_attention(layer, query, scaling), None


def padding_mask(*args, attention_mask: Optional[torch.Tensor] = None, **kwargs) -> Optional[torch.Tensor]:
    """Mask function of the ``stickykv_b200`` implementation: no mask at all
    for a batch without a 2-D padding mask (the causal pattern is the
    kernels' own, also under CUDA-graph capture, where transformers' sdpa
    function would materialise one), else the sdpa function's answer, which
    is None for an unpadded batch and a 4-D mask for a padded one (that the
    attention then refuses)."""
    if attention_mask is None:
        return None
    from transformers.masking_utils import sdpa_mask
    return sdpa_mask(*args, attention_mask=attention_mask, **kwargs)


def _register_attention() -> None:
    from transformers import AttentionInterface
    from transformers.masking_utils import AttentionMaskInterface
    AttentionInterface.register(ATTN_IMPLEMENTATION, stickykv_attention)
    # transformers builds no mask for an implementation without a mask
    # function, so a padded batch would pass unnoticed
    AttentionMaskInterface.register(ATTN_IMPLEMENTATION, padding_mask)


def install_score_hooks(model: nn.Module, cache: Any, config: Any) -> HookHandles:
    """Install the position override and the fused attention/scoring path.

    ``config`` is accepted for signature compatibility (window size and sink
    count come from the cache's resolved config)."""
    handles = HookHandles()
    install_position_override_hook(model, cache, handles)
    classes = _get_attn_classes()
    if not classes:
        warnings.warn("No LlamaAttention or Qwen2Attention found — no score hooks installed.",
                      RuntimeWarning, stacklevel=2)
        return handles
    _register_attention()
    mods = [m for _, m in model.named_modules() if isinstance(m, classes)]
    for m in mods:
        m._skv_cache = cache

    def detach():
        for m in mods:
            if getattr(m, "_skv_cache", None) is cache:
                del m._skv_cache

    handles._hook_handles.append(_Restore(detach))
    cfg = getattr(model, "config", None)
    if cfg is not None:
        previous = getattr(cfg, "_attn_implementation", None)
        cfg._attn_implementation = ATTN_IMPLEMENTATION

        def restore():
            cfg._attn_implementation = previous

        handles._hook_handles.append(_Restore(restore))
    return handles
