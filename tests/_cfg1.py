"""The end-to-end plumbing model: a 2-layer Llama (hidden 256, 4 query heads,
2 KV heads, head_dim 64, SwiGLU 688, RoPE theta 1e4, vocab 32000, fp32) with
seeded N(0, 0.02) matrices and unit norms, a seeded 512-token prompt, and a
50-step greedy loop through a windowed cache (window 8, 4 sinks, local 0.25,
budget 0.40).  Shared by the golden generator (reference backend) and the GPU
test (this package's backend) so both run the identical model."""

from __future__ import annotations

from typing import List, Tuple

import numpy as np
import torch

PROMPT_LEN, STEPS = 512, 50
WINDOW, SINKS, LOCAL, BUDGET = 8, 4, 0.25, 0.40
TOPK_LOGITS = 64


def build_model() -> torch.nn.Module:
    from transformers import LlamaConfig, LlamaForCausalLM
    cfg = LlamaConfig(vocab_size=32000, hidden_size=256, intermediate_size=688, num_hidden_layers=2,
                      num_attention_heads=4, num_key_value_heads=2, head_dim=64, rope_theta=1e4,
                      max_position_embeddings=2048, tie_word_embeddings=False)
    cfg._attn_implementation = "eager"
    model = LlamaForCausalLM(cfg).float().eval()
    g = torch.Generator().manual_seed(0)
    with torch.no_grad():
        for _, p in model.named_parameters():  # fixed order, CPU generator: same values everywhere
            if p.dim() >= 2:
                p.copy_(torch.randn(p.shape, generator=g) * 0.02)
            else:
                p.fill_(1.0)
    return model


def prompt() -> torch.Tensor:
    return torch.randint(0, 32000, (1, PROMPT_LEN), generator=torch.Generator().manual_seed(0))


def greedy(model, cache, ids: torch.Tensor, at=None, **fwd) -> Tuple[List[int], np.ndarray, np.ndarray]:
    """Prefill then STEPS-1 one-token steps, feeding back the argmax.  Returns
    (tokens, top-k logit indices [STEPS, K], their logits [STEPS, K]); with
    ``at`` ([STEPS, K] indices) the logits are read at those indices instead."""
    toks, top_i, top_v = [], [], []
    inp = ids
    with torch.no_grad():
        for step in range(STEPS):
            out = model(input_ids=inp, past_key_values=cache, use_cache=True, return_dict=True, **fwd)
            lg = out.logits[0, -1].float()
            v, i = torch.topk(lg, TOPK_LOGITS)
            toks.append(int(i[0]))
            if at is not None:
                i = torch.as_tensor(at[step], device=lg.device)
                v = lg[i]
            top_i.append(i.cpu().numpy())
            top_v.append(v.cpu().numpy())
            inp = torch.tensor([[toks[-1]]], device=ids.device)
    return toks, np.stack(top_i), np.stack(top_v)


def teacher_forced(model, cache, ids: torch.Tensor, tokens, at=None, **fwd) -> Tuple[np.ndarray, np.ndarray]:
    """Prefill then STEPS-1 one-token steps feeding ``tokens[step-1]`` (a fixed
    sequence, so two implementations see the same inputs whatever their own
    argmax).  Returns (top-k logit indices [STEPS, K], their logits [STEPS,
    K]); with ``at`` the logits are read at those indices instead."""
    top_i, top_v = [], []
    inp = ids
    with torch.no_grad():
        for step in range(STEPS):
            out = model(input_ids=inp, past_key_values=cache, use_cache=True, return_dict=True, **fwd)
            lg = out.logits[0, -1].float()
            v, i = torch.topk(lg, TOPK_LOGITS)
            if at is not None:
                i = torch.as_tensor(at[step], device=lg.device)
                v = lg[i]
            top_i.append(i.cpu().numpy())
            top_v.append(v.cpu().numpy())
            if step + 1 < STEPS:
                inp = torch.tensor([[int(tokens[step])]], device=ids.device)
    return np.stack(top_i), np.stack(top_v)
