"""Generate golden vectors by running the reference StickyKV code on seeded inputs.

Run in a container where the reference checkout is available:

    python tests/golden/make_golden.py --ref <path of the reference checkout>

It imports the reference read-only (``sys.path``) and writes small ``.npz`` /
``.json`` fixtures next to this script.  The fixtures are committed; nothing at
test time reads the reference tree.

Fixtures:
  resolve.json         WindowedCacheConfig.resolve on the reference KAT
                       geometries and on the five benchmark geometries
  scorer.npz           compute_window_scores / reduce_token_scores_to_windows
  policy.npz           EvictionPolicy.compute_retain_window_indices +
                       expand_to_token_indices on tie-free fp32 scores
  rerotate_<dt>.npz    CacheState.slice_and_keep + rerotate_keys with a HF
                       LlamaRotaryEmbedding (theta 5e5), dt in f32/bf16/f16
  cache_drive_<dt>.npz WindowedCache.update driven through prefill + 40 decode
                       steps (5 evictions) with hook-style scores each step
  eager_decode_<dt>.npz transformers eager_attention_forward +
                       compute_window_scores for one decode query
  prefill_scores.npz   the flash hook's chunked causal scoring math
  cfg1_e2e.npz         the 2-layer Llama of tests/_cfg1.py generating 50 greedy
                       tokens through the reference's eager backend (tokens,
                       top-64 logits per step, final per-layer window ids,
                       window scores, the last step's not yet accumulated
                       scores, and seq length)
  cfg1_e2e_<dt>.npz    the same model cast to fp16 / bf16: teacher-forced on
                       the fp32 tokens (logits, window ids, scores) and
                       free-running greedy (tokens, top-2 margins)
  cfg1_runner.npz      the parity runner's per-step capture on the fp32 cfg1
                       model, teacher-forced: eviction flags, effective window
                       scores and ids per layer, and the runner's
                       _extract_row_retained of them (ragged arrays stored
                       flat with per-step shapes)
"""

from __future__ import annotations

import argparse
import contextlib
import json
import math
import os
import sys
from dataclasses import dataclass

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
DT = {"f32": torch.float32, "bf16": torch.bfloat16, "f16": torch.float16}


@dataclass
class FakeModelConfig:
    num_attention_heads: int = 32
    num_key_value_heads: int = 8
    hidden_size: int = 4096
    head_dim: int = 128
    num_hidden_layers: int = 32


def to_np(t: torch.Tensor) -> np.ndarray:
    return t.detach().to(torch.float32).cpu().numpy() if t.is_floating_point() else t.cpu().numpy()


def rope_module(theta: float, head_dim: int, max_pos: int = 40000):
    from transformers import LlamaConfig
    from transformers.models.llama.modeling_llama import LlamaRotaryEmbedding
    cfg = LlamaConfig(hidden_size=head_dim * 4, num_attention_heads=4, num_key_value_heads=2,
                      head_dim=head_dim, rope_theta=theta, max_position_embeddings=max_pos)
    return LlamaRotaryEmbedding(config=cfg)


def rope_table(rope, n_pos: int, head_dim: int):
    cos, sin = rope(torch.zeros(1, 1, 1, head_dim), torch.arange(n_pos)[None])
    return to_np(cos[0]), to_np(sin[0])


def gen_resolve(WindowedCacheConfig):
    cases = []
    # reference KATs (tests/test_windowed_cache.py:91-188)
    for (ws, s, loc, bud, P, M, mc, dt) in [
        (8, 4, 0.25, 0.50, 100, 128, FakeModelConfig(), "f16"),
        (8, 4, 0.10, 0.50, 100, 128, FakeModelConfig(), "f16"),
        (8, 4, 16, 0.40, 100, 100, FakeModelConfig(32, 8, 4096, 128), "f16"),
        (8, 4, 8, 0.20, 200, 128, FakeModelConfig(), "f32"),
        (8, 4, 8, 0.60, 200, 128, FakeModelConfig(), "f16"),
        (8, 4, 8, 1.0, 200, 128, FakeModelConfig(), "f32"),
        (8, 4, 8, 0.12, 100, 50, FakeModelConfig(), "f16"),
        (1, 0, 1, 0.375, 8, 0, FakeModelConfig(), "f32"),
        # the five benchmark geometries
        (8, 4, 0.25, 0.40, 512, 50, FakeModelConfig(4, 2, 256, 64), "f32"),
        (8, 4, 0.25, 0.40, 4096, 0, FakeModelConfig(32, 8, 2048, 64), "f16"),
        (8, 4, 0.25, 0.40, 8192, 0, FakeModelConfig(32, 8, 2048, 64), "f16"),
        (8, 4, 0.25, 0.40, 16384, 0, FakeModelConfig(32, 8, 2048, 64), "f16"),
        (8, 4, 0.25, 0.40, 32768, 0, FakeModelConfig(32, 8, 2048, 64), "f16"),
        (8, 4, 0.25, 0.40, 16384, 0, FakeModelConfig(32, 8, 2048, 64), "bf16"),
        (8, 4, 0.25, 0.40, 8192, 256, FakeModelConfig(32, 8, 2048, 64), "bf16"),
        (8, 4, 0.25, 0.25, 32768, 128, FakeModelConfig(32, 8, 4096, 128), "bf16"),
        (5, 3, 0.33, 0.7, 97, 13, FakeModelConfig(6, 3, 96, 16), "f32"),
    ]:
        r = WindowedCacheConfig(window_size=ws, num_sink_tokens=s, local_window_size=loc,
                                cache_budget=bud).resolve(P, mc, DT[dt], M)
        cases.append(dict(window_size=ws, num_sink_tokens=s, local_window_size=loc,
                          cache_budget=bud, prefill_len=P, max_tokens=M,
                          num_kv_heads=mc.num_key_value_heads, head_dim=mc.head_dim,
                          dtype=dt, resolved=r.__dict__))
    with open(os.path.join(HERE, "resolve.json"), "w") as f:
        json.dump(cases, f, indent=1)


def gen_scorer(scorer):
    g = torch.Generator().manual_seed(11)
    attn = torch.randn(2, 4, 3, 37, generator=g).softmax(-1)
    out = {"attn": to_np(attn)}
    for (s, ws) in [(4, 5), (0, 8), (4, 8), (3, 1)]:
        out[f"ws_{s}_{ws}"] = to_np(scorer.compute_window_scores(attn, s, ws))
    tok = torch.rand(3, 5, 29, generator=g)
    out["tok"] = to_np(tok)
    out["tok_4_8"] = to_np(scorer.reduce_token_scores_to_windows(tok, 4, 8))
    np.savez_compressed(os.path.join(HERE, "scorer.npz"), **out)


def gen_policy(ResolvedConfig, EvictionPolicy):
    g = torch.Generator().manual_seed(12)
    out = {}
    cases = []
    for ci, (B, Hq, W, k, loc_w, ws, s, extra) in enumerate([
            (3, 4, 20, 5, 3, 8, 4, 0), (2, 8, 9, 0, 2, 8, 4, 3), (2, 4, 6, 9, 2, 8, 4, 5),
            (4, 32, 64, 17, 10, 8, 4, 1), (1, 4, 7, 2, 1, 5, 3, 2)]):
        scores = torch.rand(B, Hq, W, generator=g)
        res = ResolvedConfig(window_size=ws, num_sink_tokens=s, local_tokens=loc_w * ws,
                             top_k_windows=k, bytes_per_token=4, total_budget_bytes=0,
                             total_budget_tokens=0)
        pol = EvictionPolicy(res)
        total = s + (W - 1) * ws + extra if extra else s + W * ws
        pol.initialize_after_prefill(total)
        ret = pol.compute_retain_window_indices(scores)
        tok = pol.expand_to_token_indices(ret)
        out[f"scores_{ci}"] = to_np(scores)
        out[f"ret_{ci}"] = to_np(ret)
        out[f"tok_{ci}"] = to_np(tok)
        cases.append([k, loc_w, ws, s, total])
    out["cases"] = np.array(cases, dtype=np.int64)
    np.savez_compressed(os.path.join(HERE, "policy.npz"), **out)


def gen_rerotate(CacheState):
    rope = rope_module(500000.0, 64)
    cos, sin = rope_table(rope, 1000, 64)
    for dt in ("f32", "bf16", "f16"):
        g = torch.Generator().manual_seed(13)
        B, H, T, D = 2, 3, 40, 64
        k = torch.randn(B, H, T, D, generator=g).to(DT[dt])
        v = torch.randn(B, H, T, D, generator=g).to(DT[dt])
        pos = torch.stack([torch.sort(torch.randperm(1000, generator=g)[:T])[0] for _ in range(B)])
        keep = torch.stack([torch.sort(torch.randperm(T, generator=g)[:25])[0] for _ in range(B)])
        st = CacheState()
        st.key_states, st.value_states, st.position_ids = k.clone(), v.clone(), pos.clone()
        old = st.position_ids.gather(1, keep).clone()
        st.slice_and_keep(keep)
        st.rerotate_keys(rope, old)
        np.savez_compressed(os.path.join(HERE, f"rerotate_{dt}.npz"), k=to_np(k), v=to_np(v),
                            pos=to_np(pos), keep=to_np(keep), cos=cos, sin=sin,
                            k_out=to_np(st.key_states), v_out=to_np(st.value_states),
                            pos_out=to_np(st.position_ids))


def gen_cache_drive(WindowedCache, WindowedCacheConfig):
    rope = rope_module(10000.0, 64)
    cos, sin = rope_table(rope, 512, 64)
    for dt in ("f32", "bf16"):
        g = torch.Generator().manual_seed(14)
        B, Hkv, Hq, D, P, M = 2, 2, 4, 64, 100, 40
        mc = FakeModelConfig(Hq, Hkv, Hq * D, D)
        cfg = WindowedCacheConfig(window_size=8, num_sink_tokens=4, local_window_size=0.25,
                                  cache_budget=0.5)
        cache = WindowedCache(config=cfg, prefill_len=P, model_config=mc, kv_dtype=DT[dt],
                              rope_module=rope, num_layers=1, max_tokens=M)
        rec = {"cos": cos, "sin": sin}
        k = torch.randn(B, Hkv, P, D, generator=g).to(DT[dt])
        v = torch.randn(B, Hkv, P, D, generator=g).to(DT[dt])
        rec["k_0"], rec["v_0"] = to_np(k), to_np(v)
        cache.update(k, v, 0)
        n = cache.get_seq_length(0)
        sc = torch.rand(B, Hq, math.ceil((n - 4) / 8), generator=g)
        rec["s_0"] = to_np(sc)
        cache.cache_kwargs[0]["window_scores"] = sc
        for t in range(1, M + 1):
            k = torch.randn(B, Hkv, 1, D, generator=g).to(DT[dt])
            v = torch.randn(B, Hkv, 1, D, generator=g).to(DT[dt])
            rec[f"k_{t}"], rec[f"v_{t}"] = to_np(k), to_np(v)
            cache.update(k, v, 0)
            n = cache.get_seq_length(0)
            st = cache._states[0]
            rec[f"len_{t}"] = np.array(n)
            rec[f"ids_{t}"] = to_np(st.original_window_ids)
            sc = torch.rand(B, Hq, math.ceil((n - 4) / 8), generator=g)
            rec[f"s_{t}"] = to_np(sc)
            cache.cache_kwargs[0]["window_scores"] = sc
        st = cache._states[0]
        rec["final_k"], rec["final_v"] = to_np(st.key_states), to_np(st.value_states)
        rec["final_scores"] = to_np(st.window_scores)
        rec["final_ids"] = to_np(st.original_window_ids)
        rec["final_pos"] = to_np(st.position_ids)
        rec["meta"] = np.array([B, Hkv, Hq, D, P, M])
        np.savez_compressed(os.path.join(HERE, f"cache_drive_{dt}.npz"), **rec)


def gen_eager_decode(scorer):
    from transformers.models.llama.modeling_llama import eager_attention_forward

    class Mod(torch.nn.Module):
        num_key_value_groups = 4

    for dt in ("f32", "f16"):
        g = torch.Generator().manual_seed(15)
        B, Hq, Hkv, S, D = 2, 8, 2, 77, 64
        q = torch.randn(B, Hq, 1, D, generator=g).to(DT[dt])
        k = torch.randn(B, Hkv, S, D, generator=g).to(DT[dt])
        v = torch.randn(B, Hkv, S, D, generator=g).to(DT[dt])
        out, w = eager_attention_forward(Mod().eval(), q, k, v, None, scaling=D ** -0.5)
        sc = scorer.compute_window_scores(w, 4, 8)
        np.savez_compressed(os.path.join(HERE, f"eager_decode_{dt}.npz"), q=to_np(q[:, :, 0]),
                            k=to_np(k), v=to_np(v), out=to_np(out[:, 0]), scores=to_np(sc))


def gen_prefill_scores(scorer):
    import torch.nn.functional as F
    g = torch.Generator().manual_seed(16)
    B, Hq, Hkv, T, D = 1, 4, 2, 45, 16
    q = torch.randn(B, Hq, T, D, generator=g)
    k = torch.randn(B, Hkv, T, D, generator=g)
    kx = k.repeat_interleave(Hq // Hkv, dim=1)
    scaling = D ** -0.5
    # modules/windowed_cache/hooks.py:258-289 with chunk 16
    token_scores = torch.zeros(B, Hq, T)
    for start in range(0, T, 16):
        end = min(start + 16, T)
        aw = torch.matmul(q[:, :, start:end], kx.transpose(-2, -1)) * scaling
        causal = torch.triu(torch.ones(end - start, T, dtype=torch.bool), diagonal=T - T + start + 1)
        aw = aw.masked_fill(causal, float("-inf"))
        token_scores += F.softmax(aw, dim=-1, dtype=torch.float32).sum(dim=-2)
    sc = scorer.reduce_token_scores_to_windows(token_scores, 4, 8)
    np.savez_compressed(os.path.join(HERE, "prefill_scores.npz"), q=to_np(q), k=to_np(k),
                        scores=to_np(sc))


@contextlib.contextmanager
def _cfg1_env(ref_eager):
    """The cfg1 model's module and the transformers 5.5 harness shim around
    the reference eager backend.  The shim changes no reference arithmetic:
    the Cache mask-size API (``layers``, ``is_compileable``,
    ``get_mask_sizes``) and an eager attention wrapper that trims the mask to
    the compacted key length (the 4.47 behaviour)."""
    import transformers.models.llama.modeling_llama as LM
    import importlib.util
    spec = importlib.util.spec_from_file_location("skv_cfg1", os.path.join(os.path.dirname(HERE), "_cfg1.py"))
    C1 = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(C1)

    class Shim(ref_eager.WindowedCache):
        layers = []
        is_compileable = False

        def get_mask_sizes(self, q_len, layer_idx=0):
            q = int(q_len.shape[0]) if torch.is_tensor(q_len) else int(q_len)
            return self.get_seq_length(layer_idx) + q, 0

    eager = LM.eager_attention_forward

    def eager_trimmed(module, q, k, v, mask, *a, **kw):
        if mask is not None:
            mask = mask[..., : k.shape[-2]]
        return eager(module, q, k, v, mask, *a, **kw)

    LM.eager_attention_forward = eager_trimmed
    try:
        yield C1, Shim
    finally:
        LM.eager_attention_forward = eager


def _cfg1_cache(ref_eager, C1, Shim, model, dt):
    wcfg = ref_eager.WindowedCacheConfig(window_size=C1.WINDOW, num_sink_tokens=C1.SINKS,
                                         local_window_size=C1.LOCAL, cache_budget=C1.BUDGET)
    cache = Shim(config=wcfg, prefill_len=C1.PROMPT_LEN, model_config=model.config, kv_dtype=dt,
                 rope_module=model.model.rotary_emb, num_layers=2, max_tokens=C1.STEPS)
    return cache, ref_eager.install_score_hooks(model, cache, wcfg)


def gen_cfg1_e2e(ref_eager):
    """Reference eager backend on the cfg1 model (harness: :func:`_cfg1_env`)."""
    with _cfg1_env(ref_eager) as (C1, Shim):
        model = C1.build_model()
        cache, handles = _cfg1_cache(ref_eager, C1, Shim, model, torch.float32)
        toks, top_i, top_v = C1.greedy(model, cache, C1.prompt(), output_attentions=True)
        handles.remove()
    rec = dict(tokens=np.array(toks, np.int64), top_i=top_i.astype(np.int64), top_v=top_v.astype(np.float32),
               seq_len=np.array(cache.get_seq_length(0)))
    for li in range(2):
        st = cache._states[li]
        rec[f"ids_{li}"] = to_np(st.original_window_ids)
        rec[f"scores_{li}"] = to_np(st.window_scores)
        # the last step's scores wait in cache_kwargs for the next update()
        rec[f"pending_{li}"] = to_np(cache.cache_kwargs[li]["window_scores"])
    np.savez_compressed(os.path.join(HERE, "cfg1_e2e.npz"), **rec)


def gen_cfg1_e2e_half(ref_eager):
    """The cfg1 model cast to fp16 and to bf16 through the reference's eager
    backend (harness: :func:`_cfg1_env`; matmuls accumulate in fp32, the
    softmax runs in fp32 and is cast to the model dtype, window scores
    accumulate in the model dtype).  Two runs per dtype: teacher-forced on the
    fp32 run's greedy tokens (top-64 logits per step, final per-layer window
    ids, scores, the last step's pending scores, seq length) and free-running
    greedy (tokens and the top-1/top-2 logit margin of every step)."""
    fp32 = np.load(os.path.join(HERE, "cfg1_e2e.npz"))
    with _cfg1_env(ref_eager) as (C1, Shim):
        for name, dt in (("f16", torch.float16), ("bf16", torch.bfloat16)):
            rec = {"tf_tokens": fp32["tokens"]}
            for mode in ("tf", "greedy"):
                model = C1.build_model().to(dt)
                cache, handles = _cfg1_cache(ref_eager, C1, Shim, model, dt)
                if mode == "tf":
                    top_i, top_v = C1.teacher_forced(model, cache, C1.prompt(), fp32["tokens"],
                                                     output_attentions=True)
                    rec.update(tf_top_i=top_i.astype(np.int64), tf_top_v=top_v.astype(np.float32),
                               tf_seq_len=np.array(cache.get_seq_length(0)))
                    for li in range(2):
                        st = cache._states[li]
                        rec[f"tf_ids_{li}"] = to_np(st.original_window_ids)
                        rec[f"tf_scores_{li}"] = to_np(st.window_scores)
                        rec[f"tf_pending_{li}"] = to_np(cache.cache_kwargs[li]["window_scores"])
                else:
                    toks, _, top_v = C1.greedy(model, cache, C1.prompt(), output_attentions=True)
                    rec.update(greedy_tokens=np.array(toks, np.int64),
                               greedy_margin=(top_v[:, 0] - top_v[:, 1]).astype(np.float32))
                handles.remove()
            np.savez_compressed(os.path.join(HERE, f"cfg1_e2e_{name}.npz"), **rec)


def _effective_scores(cache, li):
    """[1, H, W] window scores of layer ``li`` including the step's scores
    that the reference keeps pending in ``cache_kwargs`` until the next
    update() (which may already cover a window the state does not list yet),
    and the [1, W] original window ids: identity before the first eviction,
    and a window that only the pending scores cover takes the id after the
    newest one (windows are numbered in order of creation)."""
    st = cache._states[li]
    pend = cache.cache_kwargs[li].get("window_scores") if li in cache.cache_kwargs else None
    ids = st.original_window_ids
    W = max(ids.shape[-1] if ids is not None else 0,
            st.window_scores.shape[-1] if st.window_scores is not None else 0,
            pend.shape[-1] if pend is not None else 0)
    if ids is None:
        ids = torch.arange(W, dtype=torch.long).unsqueeze(0)
    elif ids.shape[-1] < W:
        extra = ids[:, -1:] + torch.arange(1, W - ids.shape[-1] + 1, dtype=ids.dtype).unsqueeze(0)
        ids = torch.cat([ids, extra], dim=-1)
    H = (st.window_scores if st.window_scores is not None else pend).shape[1]
    eff = torch.zeros(1, H, W, dtype=torch.float32)
    for part in (st.window_scores, pend):
        if part is not None:
            n = min(W, part.shape[-1])
            eff[..., :n] += part[..., :n].float()
    return eff, ids.long()


def gen_cfg1_runner(ref_eager, extract_row_retained):
    """The parity runner's per-step capture (modules/evaluation/
    ours_parity_runner.py:312-402) on the fp32 cfg1 model through the
    reference eager backend, teacher-forced on the fp32 greedy tokens: per
    step the eviction flag, and per layer the effective window scores, the
    original window ids and the runner's own ``_extract_row_retained`` of
    them (its top-K window ids, fp16 scores, retained ids and retained fp16
    scores)."""
    fp32 = np.load(os.path.join(HERE, "cfg1_e2e.npz"))
    with _cfg1_env(ref_eager) as (C1, Shim):
        model = C1.build_model()
        cache, handles = _cfg1_cache(ref_eager, C1, Shim, model, torch.float32)
        tk = cache.resolved.top_k_windows
        rec = {"tokens": fp32["tokens"], "top_k": np.array(tk)}
        steps = {k: [] for k in ("evicted", "W")}
        per = {}
        inp = C1.prompt()
        with torch.no_grad():
            for step in range(C1.STEPS):
                model(input_ids=inp, past_key_values=cache, use_cache=True, return_dict=True,
                      output_attentions=True)
                gs = cache._generation_step
                steps["evicted"].append(any((gs[li] - 1) > 0 and (gs[li] - 1) % C1.WINDOW == 0 for li in range(2)))
                for li in range(2):
                    eff, ids = _effective_scores(cache, li)
                    a_tk, a_ws, a_rid, a_rsc = extract_row_retained(eff[0], ids[0], tk, C1.WINDOW, C1.LOCAL)
                    for key, val in (("scores", eff[0].numpy()), ("ids", ids[0].numpy()), ("tk", a_tk),
                                     ("ws16", a_ws), ("ret_ids", a_rid), ("ret_sc16", a_rsc)):
                        per.setdefault(f"{key}_{li}", []).append(val)
                if step + 1 < C1.STEPS:
                    inp = torch.tensor([[int(fp32["tokens"][step])]])
        handles.remove()
    rec["evicted"] = np.array(steps["evicted"], bool)
    for key, vals in per.items():  # ragged over steps: concatenated with per-step lengths
        rec[key] = np.concatenate([np.asarray(v).reshape(-1) for v in vals])
        rec[key + "_shape"] = np.array([np.asarray(v).shape + (0,) * (2 - np.asarray(v).ndim) for v in vals],
                                       np.int64)
    np.savez_compressed(os.path.join(HERE, "cfg1_runner.npz"), **rec)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", required=True, help="path of the reference checkout (imported read-only)")
    args = ap.parse_args()
    sys.path.insert(0, args.ref)
    from modules.windowed_cache import scorer
    from modules.windowed_cache.cache import WindowedCache
    from modules.windowed_cache.config import ResolvedConfig, WindowedCacheConfig
    from modules.windowed_cache.policy import EvictionPolicy
    from modules.windowed_cache.state import CacheState
    torch.set_num_threads(1)
    gen_resolve(WindowedCacheConfig)
    gen_scorer(scorer)
    gen_policy(ResolvedConfig, EvictionPolicy)
    gen_rerotate(CacheState)
    gen_cache_drive(WindowedCache, WindowedCacheConfig)
    gen_eager_decode(scorer)
    gen_prefill_scores(scorer)
    import modules.windowed_eager_cache as ref_eager
    gen_cfg1_e2e(ref_eager)
    gen_cfg1_e2e_half(ref_eager)
    from modules.evaluation.ours_parity_runner import _extract_row_retained
    gen_cfg1_runner(ref_eager, _extract_row_retained)
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    main()
