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


HALF_TOL = {"f16": 2e-3, "bf16": 8e-3}  # max-abs logit tolerance per model dtype


def _b200_cache(model, dtype, steps=C1.STEPS):
    from stickykv_b200.cache_factory import get_cache_classes
    Cache, Config, install = get_cache_classes("b200")
    cfg = Config(window_size=C1.WINDOW, num_sink_tokens=C1.SINKS, local_window_size=C1.LOCAL,
                 cache_budget=C1.BUDGET)
    cache = Cache(cfg, C1.PROMPT_LEN, model.config, dtype, model.model.rotary_emb, 2, steps)
    return cache, install(model, cache, cfg)


@pytest.mark.parametrize("dt", ["f16", "bf16"])
def test_cfg1_half_precision_matches_reference(dt):
    """The cfg1 model cast to fp16 / bf16 against the reference's eager
    backend in the same dtype (tests/golden/cfg1_e2e_<dt>.npz).

    Teacher-forced on one fixed token sequence (so both runs see the same
    inputs): logits at the reference's top-64 indices within max-abs 2e-3
    (fp16) / 8e-3 (bf16) at all 50 steps; the kept windows (original ids) of
    both layers and the final length bit-exact; window scores within the
    rounding of the reference, which accumulates them in the model dtype
    (this backend accumulates in fp32).

    Free-running greedy: every token equal to the reference's own greedy
    token.  At a step where the reference's top two logits are within the
    tolerance of each other the two runs may legitimately pick different
    tokens (the tie is below the numerical contract) and the sequences then
    part; the comparison stops there.  Most such ties in this tiny random
    model are exact ties of the rounded logits."""
    z = np.load(os.path.join(os.path.dirname(__file__), "golden", f"cfg1_e2e_{dt}.npz"))
    tdt = {"f16": torch.float16, "bf16": torch.bfloat16}[dt]
    tol = HALF_TOL[dt]
    model = C1.build_model().to(tdt).cuda()
    cache, handles = _b200_cache(model, tdt)
    try:
        _, logits = C1.teacher_forced(model, cache, C1.prompt().cuda(), z["tf_tokens"], at=z["tf_top_i"])
    finally:
        handles.remove()
    err = np.abs(logits - z["tf_top_v"]).max(axis=1)
    assert err.max() <= tol, f"logits differ by {err.max():.2e} (step {int(err.argmax())})"
    assert cache.get_seq_length(0) == int(z["tf_seq_len"])
    for li in range(2):
        st = cache._states[li]
        np.testing.assert_array_equal(st.original_window_ids.cpu().numpy(), z[f"tf_ids_{li}"], err_msg=f"layer {li}")
        want = z[f"tf_scores_{li}"].astype(np.float32).copy()
        pend = z[f"tf_pending_{li}"]
        want[..., : pend.shape[-1]] += pend[..., : want.shape[-1]]
        # the reference adds each step's mass to a model-dtype accumulator: in
        # bf16 an addend below half an ulp of the running sum (1/16 at 16)
        # is rounded away, so its scores stall (fp16 keeps 3 more bits)
        np.testing.assert_allclose(st.window_scores.float().cpu().numpy(), want,
                                   rtol={"f16": 8 * tol, "bf16": 0.15}[dt], atol=1e-4)
    # free-running greedy
    model = C1.build_model().to(tdt).cuda()
    cache, handles = _b200_cache(model, tdt)
    try:
        toks, _, _ = C1.greedy(model, cache, C1.prompt().cuda())
    finally:
        handles.remove()
    ref = z["greedy_tokens"].tolist()
    for i, (a, b) in enumerate(zip(toks, ref)):
        if a != b:
            assert z["greedy_margin"][i] <= tol, (
                f"step {i}: token {a} vs the reference's {b} with a top-2 margin of "
                f"{z['greedy_margin'][i]:.2e} (above the {tol} tolerance)")
            break


def test_generate_drop_in_matches_the_reference_run():
    """The README usage, model.generate(input_ids, past_key_values=cache,
    max_new_tokens=50), through get_cache_classes("b200"): the same 50 greedy
    tokens, kept windows and final length as the reference's eager backend
    driven step by step (tests/golden/cfg1_e2e.npz)."""
    z = np.load(GOLDEN)
    model = C1.build_model().cuda()
    cache, handles = _b200_cache(model, torch.float32)
    ids = C1.prompt().cuda()
    try:
        with torch.no_grad():
            out = model.generate(ids, past_key_values=cache, max_new_tokens=C1.STEPS, do_sample=False,
                                 min_new_tokens=C1.STEPS, pad_token_id=0)
    finally:
        handles.remove()
    assert out[0, C1.PROMPT_LEN:].tolist() == z["tokens"].tolist()
    assert cache.get_seq_length(0) == int(z["seq_len"])
    for li in range(2):
        np.testing.assert_array_equal(cache._states[li].original_window_ids.cpu().numpy(), z[f"ids_{li}"])


def test_qwen2_gqa7_matches_transformers_attention_without_eviction():
    """A 2-layer Qwen2-shaped fp16 model with 14 query and 2 kv heads (GQA 7,
    head_dim 64, the tensor-core decode's head groups of 4 + 3) through this
    package's hooks, with a budget that never evicts, against transformers'
    own cache and eager attention on the same tokens.

    Its logits reach |3|, where one fp16 ulp (1/512) already exceeds the 2e-3
    contract, so both fp16 paths are measured against the same model in fp32
    (teacher-forced on the same tokens): at every step this backend's largest
    logit error may exceed the fp16 eager path's own by at most 2e-3."""
    from transformers import Qwen2Config, Qwen2ForCausalLM

    from stickykv_b200.cache_factory import get_cache_classes
    cfg = Qwen2Config(vocab_size=32000, hidden_size=896, intermediate_size=1024, num_hidden_layers=2,
                      num_attention_heads=14, num_key_value_heads=2, max_position_embeddings=4096,
                      rope_theta=1e6, tie_word_embeddings=True)
    cfg._attn_implementation = "eager"
    torch.manual_seed(0)
    model32 = Qwen2ForCausalLM(cfg).float().cuda().eval()
    model = Qwen2ForCausalLM(cfg).cuda().eval()
    model.load_state_dict(model32.state_dict())
    model = model.half()
    P, steps = 512, 16
    ids = torch.randint(0, 32000, (2, P), generator=torch.Generator().manual_seed(1)).cuda()

    def hf_run(m, toks=None):
        out = m(input_ids=ids, use_cache=True)
        past = out.past_key_values
        own, lg = [out.logits[:, -1:].argmax(-1)], [out.logits[:, -1].float()]
        for t in range(steps - 1):
            out = m(input_ids=(toks or own)[t], past_key_values=past, use_cache=True)
            past = out.past_key_values
            own.append(out.logits[:, -1:].argmax(-1))
            lg.append(out.logits[:, -1].float())
        return own, lg

    with torch.no_grad():
        toks, ref = hf_run(model)
        _, exact = hf_run(model32, toks)
    Cache, Config, install = get_cache_classes("b200")
    wcfg = Config(window_size=8, num_sink_tokens=4, local_window_size=0.25, cache_budget=1.0)
    cache = Cache(wcfg, P, model.config, torch.float16, model.model.rotary_emb, 2, steps)
    handles = install(model, cache, wcfg)
    try:
        with torch.no_grad():
            out = model(input_ids=ids, past_key_values=cache, use_cache=True)
            got = [out.logits[:, -1].float()]
            for t in range(steps - 1):
                out = model(input_ids=toks[t], past_key_values=cache, use_cache=True)
                got.append(out.logits[:, -1].float())
    finally:
        handles.remove()
    for t, (a, b, x) in enumerate(zip(got, ref, exact)):
        ours, theirs = float((a - x).abs().max()), float((b - x).abs().max())
        assert ours <= theirs + HALF_TOL["f16"], f"step {t}: error {ours:.2e} vs eager fp16 {theirs:.2e}"
    assert cache.get_seq_length(0) == P + steps - 1
