"""CUDA-graph replay of steady-state decode steps (stickykv_b200.DecodeGraphs).

The 2-layer Llama of _cfg1 decodes eagerly until its cache is in steady state
(two evictions behind it, at a period boundary), then one period of 16 steps
is replayed from per-phase CUDA graphs of the whole transformers forward,
then decoding resumes eagerly.  The run must reproduce the reference eager
backend's recording (tests/golden/cfg1_e2e.npz) exactly as the eager loop
does: the same 50 greedy tokens, logits at the reference's top-64 indices
within 1e-4, the same kept windows and final length.
"""

import os

import numpy as np
import pytest
import torch

from tests import _cfg1 as C1

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "cfg1_e2e.npz")


def test_graph_replayed_decode_matches_reference_run():
    from stickykv_b200 import DecodeGraphs
    from stickykv_b200.cache_factory import get_cache_classes
    z = np.load(GOLDEN)
    model = C1.build_model().cuda()
    Cache, Config, install = get_cache_classes("b200")
    cfg = Config(window_size=C1.WINDOW, num_sink_tokens=C1.SINKS, local_window_size=C1.LOCAL,
                 cache_budget=C1.BUDGET)
    cache = Cache(cfg, C1.PROMPT_LEN, model.config, torch.float32, model.model.rotary_emb, 2, C1.STEPS)
    handles = install(model, cache, cfg)
    at = torch.as_tensor(z["top_i"], device="cuda")
    tok = torch.zeros(1, 1, dtype=torch.long, device="cuda")
    toks, logits, replayed = [], [], 0
    try:
        with torch.no_grad():
            def eager(inp, step):
                lg = model(input_ids=inp, past_key_values=cache, use_cache=True).logits[0, -1].float()
                tok.copy_(lg.argmax().view(1, 1))
                toks.append(int(tok))
                logits.append(lg[at[step]].cpu().numpy())

            eager(C1.prompt().cuda(), 0)
            while not DecodeGraphs.ready(cache):
                eager(tok, len(toks))
            first = len(toks)
            period = DecodeGraphs.period_of(cache)
            assert first + period <= C1.STEPS
            hist_tok = torch.zeros(period, dtype=torch.long, device="cuda")
            hist_lg = torch.zeros(period, at.shape[1], device="cuda")

            def graph_step(j):
                lg = model(input_ids=tok, past_key_values=cache, use_cache=True).logits[0, -1].float()
                hist_lg[j].copy_(lg[at[first + j]])
                nxt = lg.argmax()
                hist_tok[j].copy_(nxt)
                tok.copy_(nxt.view(1, 1))

            graphs = DecodeGraphs(cache, graph_step, whole_period=False)
            graphs.replay(period)
            torch.cuda.synchronize()
            assert graphs.in_step
            replayed = period
            toks += hist_tok.tolist()
            logits += list(hist_lg.cpu().numpy())
            del graphs
            while len(toks) < C1.STEPS:
                eager(tok, len(toks))
    finally:
        handles.remove()
    assert replayed == 16 and first == 33  # forwards 33..48 came from the graphs
    assert toks == z["tokens"].tolist()
    np.testing.assert_allclose(np.stack(logits), z["top_v"], atol=1e-4, rtol=0)
    assert cache.get_seq_length(0) == int(z["seq_len"])
    for li in range(2):
        np.testing.assert_array_equal(cache._states[li].original_window_ids.cpu().numpy(), z[f"ids_{li}"])


def test_decode_graphs_refuses_a_cache_that_is_not_steady():
    from stickykv_b200 import DecodeGraphs
    from tests._helpers import make_cache, rope_tables
    cos, sin = rope_tables(1e4, 64, 400)
    cache = make_cache("f16", 1, 2, 4, 64, 300, 40, cos, sin)
    cache.update(torch.randn(1, 2, 300, 64, device="cuda").half(), torch.randn(1, 2, 300, 64, device="cuda").half(), 0)
    assert not DecodeGraphs.ready(cache)
    with pytest.raises(RuntimeError, match="steady state"):
        DecodeGraphs(cache, lambda j: None)
