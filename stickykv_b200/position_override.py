"""Decoder pre-hook that places the query at the compacted cache length.

Same contract as the reference's utils/position_override.py:32-99: every
eviction re-bases the kept keys to positions 0..T-1, so at every step the
query must sit at position ``cache.get_seq_length(0)`` (not the monotonic
position ``generate`` would pass), and a 2-D attention mask that no longer
matches the compacted length is dropped for a batch of one.  Rows of a batch
always keep the same token count, so the override holds for any batch size
without padding.
"""

from __future__ import annotations

from typing import Any

import torch


def install_position_override_hook(model: Any, cache: Any, handles: Any) -> None:
    """Register the pre-hook on the decoder and add its handle to ``handles``."""
    decoder = model.get_decoder() if hasattr(model, "get_decoder") else getattr(model, "model", model)

    def pre_hook(module, args, kwargs):
        ids = kwargs.get("input_ids")
        if ids is None and args and torch.is_tensor(args[0]):
            ids = args[0]
        anchor = ids if ids is not None else kwargs.get("inputs_embeds")
        if anchor is None:
            return None
        q_len, device = anchor.shape[1], anchor.device
        past = cache.get_seq_length(0)
        pos = torch.arange(past, past + q_len, device=device, dtype=torch.long)
        kwargs["cache_position"] = pos
        kwargs["position_ids"] = pos.unsqueeze(0)
        mask = kwargs.get("attention_mask")
        if (mask is not None and torch.is_tensor(mask) and mask.dim() == 2 and mask.shape[0] == 1
                and mask.shape[-1] != past + q_len):
            kwargs["attention_mask"] = None
        return args, kwargs

    handles._hook_handles.append(decoder.register_forward_pre_hook(pre_hook, with_kwargs=True))
