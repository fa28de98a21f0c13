"""Time the reference's own CPU path against the oracle port on the bench's
decode-step workload (one row of the 32k-context geometry, all-fp16 tiers,
budget 0.40, an eviction every 8 steps): the reference's
``WindowedCache.update`` (append, score accumulation, eviction with
``EvictionPolicy`` + ``CacheState.slice_and_keep`` + ``rerotate_keys`` and a
transformers rotary module, theta 5e5), transformers'
``eager_attention_forward`` and the reference's ``compute_window_scores``, in
fp16 on the host cores.  Build container only: the reference is imported
from its checkout and does not travel with this repository.

    python oracle/time_reference_cpu.py --ref <path of the reference checkout> [--steps 16]
"""

from __future__ import annotations

import argparse
import math
import os
import sys
import time

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", required=True)
    ap.add_argument("--steps", type=int, default=16)
    ap.add_argument("--threads", type=int, default=os.cpu_count() or 1)
    args = ap.parse_args()
    sys.path.insert(0, args.ref)
    sys.path.insert(0, ROOT)
    import torch
    from transformers import LlamaConfig
    from transformers.models.llama.modeling_llama import LlamaRotaryEmbedding, eager_attention_forward

    import bench
    from modules.windowed_cache import scorer
    from modules.windowed_cache.cache import WindowedCache
    from modules.windowed_cache.config import WindowedCacheConfig

    torch.set_num_threads(args.threads)
    B, HQ, HKV, D, CTX, WS = 1, bench.HQ, bench.HKV, bench.D, bench.CTX, bench.WS

    class MC:
        num_attention_heads, num_key_value_heads, hidden_size, head_dim = HQ, HKV, HQ * D, D
        num_hidden_layers = 1

    class Mod(torch.nn.Module):
        num_key_value_groups = HQ // HKV

    rope = LlamaRotaryEmbedding(config=LlamaConfig(hidden_size=HQ * D, num_attention_heads=HQ,
                                                   num_key_value_heads=HKV, head_dim=D, rope_theta=5e5,
                                                   max_position_embeddings=CTX + 256))
    cfg = WindowedCacheConfig(window_size=WS, num_sink_tokens=bench.SINKS, local_window_size=bench.LOCAL,
                              cache_budget=bench.BUDGET)
    cache = WindowedCache(config=cfg, prefill_len=CTX, model_config=MC(), kv_dtype=torch.float16,
                          rope_module=rope, num_layers=1, max_tokens=0)
    g = torch.Generator().manual_seed(0)
    cache.update(torch.randn(B, HKV, CTX, D, generator=g).half(), torch.randn(B, HKV, CTX, D, generator=g).half(), 0)
    W = math.ceil((CTX - bench.SINKS) / WS)
    cache.cache_kwargs[0]["window_scores"] = torch.rand(B, HQ, W, generator=g)
    mod = Mod().eval()

    def step():
        kn = torch.randn(B, HKV, 1, D, generator=g).half()
        k, v = cache.update(kn, kn.clone(), 0)
        q = torch.randn(B, HQ, 1, D, generator=g).half()
        _, w = eager_attention_forward(mod, q, k, v, None, scaling=D ** -0.5)
        cache.cache_kwargs[0]["window_scores"] = scorer.compute_window_scores(w, bench.SINKS, WS)

    for _ in range(WS + 1):  # the first eviction, to the steady state
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    ref_ms = (time.perf_counter() - t0) * 1e3 / args.steps
    import threadpoolctl
    with threadpoolctl.threadpool_limits(args.threads):
        oc, rng = bench.cpu_reference_setup(1)
        bench.cpu_step(oc, rng)
        t0 = time.perf_counter()
        for _ in range(args.steps):
            bench.cpu_step(oc, rng)
        port_ms = (time.perf_counter() - t0) * 1e3 / args.steps
    print(f"threads {args.threads}, {args.steps} steps ({args.steps // WS} evictions), retained {cache.get_seq_length(0)}: "
          f"reference {ref_ms:.1f} ms/step, oracle port {port_ms:.1f} ms/step")


if __name__ == "__main__":
    main()
