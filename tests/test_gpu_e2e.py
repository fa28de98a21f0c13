"""End to end through a transformers model: the 2-layer Llama of _cfg1
generates 50 greedy tokens with this package's backend (prefill scoring,
decode attention with fused window mass, five evictions per layer, query
position override) and must reproduce the reference eager backend's run
recorded in tests/golden/cfg1_e2e.npz: identical tokens, the same kept
windows (original ids) and final length, logits at the reference's top-64
indices within 1e-4 max-abs (fp32 model), window scores within 1e-5 relative
(counting the reference's last-step scores, which it only accumulates at the
next update).
"""

import os

import numpy as np
import pytest
import torch

from tests import _cfg1 as C1

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "cfg1_e2e.npz")


def test_cfg1_greedy_generation_matches_reference():
    from stickykv_b200.cache_factory import get_cache_classes
    z = np.load(GOLDEN)
    model = C1.build_model().cuda()
    Cache, Config, install = get_cache_classes("b200")
    cfg = Config(window_size=C1.WINDOW, num_sink_tokens=C1.SINKS, local_window_size=C1.LOCAL,
                 cache_budget=C1.BUDGET)
    cache = Cache(cfg, C1.PROMPT_LEN, model.config, torch.float32, model.model.rotary_emb, 2, C1.STEPS)
    handles = install(model, cache, cfg)
    try:
        toks, _, logits = C1.greedy(model, cache, C1.prompt().cuda(), at=z["top_i"])
    finally:
        handles.remove()
    assert toks == z["tokens"].tolist()
    np.testing.assert_allclose(logits, z["top_v"], atol=1e-4, rtol=0)
    assert cache.get_seq_length(0) == int(z["seq_len"])
    for li in range(2):
        st = cache._states[li]
        np.testing.assert_array_equal(st.original_window_ids.cpu().numpy(), z[f"ids_{li}"])
        # the reference adds a step's scores at the next update(); this
        # backend adds them in the attention pass itself
        want = z[f"scores_{li}"].copy()
        pend = z[f"pending_{li}"]
        want[..., : pend.shape[-1]] += pend[..., : want.shape[-1]]
        np.testing.assert_allclose(st.window_scores.float().cpu().numpy(), want, rtol=1e-5, atol=1e-6)
    assert model.config._attn_implementation == "eager"  # restored by remove()
