"""CPU tests of the host side: the C-ABI library loads and exports every
declared symbol, the host-only eviction plan agrees with the oracle, and the
config / factory / hook plumbing behaves like the reference's
(tests/test_windowed_cache.py of the reference)."""

import json
import os
import re
import subprocess
from dataclasses import dataclass

import numpy as np
import pytest
import torch

from oracle import skv_oracle as O
from stickykv_b200 import (ConfigValidationError, HookHandles, NullTelemetry, WindowedCacheConfig,
                           get_cache_classes, validate_backend_attn_pairing)
from stickykv_b200 import _lib
from stickykv_b200.position_override import install_position_override_hook

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
G = os.path.join(ROOT, "tests", "golden")


@dataclass
class FakeModelConfig:
    num_attention_heads: int = 32
    num_key_value_heads: int = 8
    hidden_size: int = 4096
    head_dim: int = 128


def _cfg(**kw):
    d = dict(window_size=8, num_sink_tokens=4, local_window_size=16, cache_budget=0.40)
    d.update(kw)
    return WindowedCacheConfig(**d)


# -- native library ---------------------------------------------------------------------

def test_library_exports_every_declared_symbol():
    L = _lib.lib()
    header = open(os.path.join(ROOT, "include", "stickykv_b200.h")).read()
    declared = set(re.findall(r"^\s*(?:int|int32_t|size_t|const char\*)\s+(skv_\w+)\(", header, re.M))
    assert declared == set(_lib.EXPORTS), declared ^ set(_lib.EXPORTS)
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True,
                         text=True, check=True).stdout
    exported = set(re.findall(r" T (skv_\w+)$", out, re.M))
    assert declared <= exported, declared - exported
    for name in declared:
        assert hasattr(L, name)


def test_abi_struct_layout_and_constants():
    L = _lib.lib()
    assert L.skv_abi_version() == 1
    import ctypes
    assert L.skv_struct_size(0) == ctypes.sizeof(_lib.LayerDesc)
    assert L.skv_struct_size(1) == ctypes.sizeof(_lib.EvictPlan)
    assert L.skv_struct_size(2) == ctypes.sizeof(_lib.EvictArgs)
    for D in (32, 64, 128):
        assert L.skv_page_bytes(D) == O.page_bytes(D) == _lib.page_bytes(D)
    assert L.skv_page_bytes(48) == 0
    assert L.skv_status_string(4) == b"buffer capacity exceeded"


def test_null_arguments_are_rejected_without_a_gpu():
    L = _lib.lib()
    assert L.skv_append(None, 0, 0, None, None, 0, 0, 0, 1, None) == 1
    assert L.skv_decode_attention(None, 1, 0, None, 0, 0, None, 0, 0, 1.0, None, 0, None, 0, None) == 1
    assert L.skv_evict(None, None, None, None, 0, None) == 1
    import ctypes
    d = _lib.LayerDesc()
    d.batch, d.num_kv_heads, d.num_q_heads, d.head_dim = 1, 1, 4, 64
    d.kv_dtype, d.window_size, d.sink_pad = 0, 8, 0
    d.fp_capacity, d.k_fp, d.v_fp = 64, 16, 16   # never dereferenced: checks fail first
    assert L.skv_append(ctypes.byref(d), 0, 0, None, None, 0, 0, 0, 1, None) == 1  # null k/v
    assert L.skv_append(ctypes.byref(d), 60, 0, 16, 16, 0, 0, 64, 8, None) == 4    # past capacity
    assert L.skv_append(ctypes.byref(d), 0, 0, 16, 24, 0, 0, 64, 8, None) == 3     # misaligned v
    d.num_q_heads = 12                                                             # G=12: no kernel
    assert L.skv_decode_attention(ctypes.byref(d), 8, 0, 16, 0, 0, 16, 0, 0, 1.0, None, 0, None, 0,
                                  None) == 2
    d.num_q_heads, d.sink_pad, d.num_sink = 4, 0, 3                                # sink_pad != 8
    assert L.skv_decode_attention(ctypes.byref(d), 8, 0, 16, 0, 0, 16, 0, 0, 1.0, None, 0, None, 0,
                                  None) == 1
    # the fused append + decode runs every check of both halves before any launch
    assert L.skv_decode_attention_append(None, 1, 0, 16, 16, 0, 0, 16, 0, 0, 16, 0, 0, 1.0, None, 0,
                                         None, 0, None) == 1
    d.sink_pad = 8
    assert L.skv_decode_attention_append(ctypes.byref(d), 8, 0, 16, 16, 0, 0, 16, 0, 0, 16, 0, 0, 1.0,
                                         None, 0, None, 0, None) == 6              # no workspace
    assert L.skv_decode_attention_append(ctypes.byref(d), 80, 0, 16, 16, 0, 0, 16, 0, 0, 16, 0, 0, 1.0,
                                         None, 0, 256, 1 << 20, None) == 4         # past capacity
    assert L.skv_decode_attention_append(ctypes.byref(d), 8, 0, None, 16, 0, 0, 16, 0, 0, 16, 0, 0,
                                         1.0, None, 0, 256, 1 << 20, None) == 1    # null k_new
    assert L.skv_decode_attention_append(ctypes.byref(d), 8, 0, 24, 16, 0, 0, 16, 0, 0, 16, 0, 0, 1.0,
                                         None, 0, 256, 1 << 20, None) == 3         # misaligned k_new
    # the eviction with this step's token: its buffers are checked before the eviction's own checks
    assert L.skv_evict_append(None, None, None, 16, 16, 0, 0, None, 0, None) == 1
    a = _lib.EvictArgs()
    a.seq_len, a.local_windows = 9, 1
    assert L.skv_evict_append(ctypes.byref(d), ctypes.byref(d), None, 16, 16, 0, 0, None, 0, None) == 1
    assert L.skv_evict_append(ctypes.byref(d), ctypes.byref(d), ctypes.byref(a), None, 16, 0, 0, None, 0,
                              None) == 1                                            # null k_new
    assert L.skv_evict_append(ctypes.byref(d), ctypes.byref(d), ctypes.byref(a), 16, 24, 0, 0, None, 0,
                              None) == 3                                            # misaligned v_new
    assert L.skv_evict_append(ctypes.byref(d), ctypes.byref(d), ctypes.byref(a), 16, 16, 3, 0, None, 0,
                              None) == 3                                            # row stride not 16 B
    assert L.skv_evict_append(ctypes.byref(d), ctypes.byref(d), ctypes.byref(a), 16, 16, 64, 64, None, 0,
                              None) == 1                                            # src == dst stores
    d.rope_cos, d.rope_sin = 16, 8                                                 # rope rows are vector-read
    assert L.skv_decode_attention(ctypes.byref(d), 8, 0, 16, 0, 0, 16, 0, 0, 1.0, None, 0, 256, 1 << 20,
                                  None) == 3
    assert L.skv_decode_workspace_size(ctypes.byref(d), 8) == 0
    d.rope_cos, d.rope_sin = None, None
    # prefill: null and misaligned buffers are refused before any launch
    assert L.skv_prefill_attention(ctypes.byref(d), 8, None, 16, 16, 16, 1.0, None, 0, 256, 1 << 20,
                                   None) == 1                                       # null q
    assert L.skv_prefill_attention(ctypes.byref(d), 8, 16, 16, 16, 24, 1.0, None, 0, 256, 1 << 20,
                                   None) == 3                                       # misaligned out


@pytest.mark.parametrize("seed", range(6))
def test_evict_plan_matches_oracle_expansion(seed):
    rng = np.random.default_rng(seed)
    for _ in range(200):
        ws = int(rng.choice([1, 4, 5, 8, 16]))
        s = int(rng.integers(0, 9))
        post = int(rng.integers(0, 400))
        T = s + post
        Wmax = -(-post // ws)
        W = int(rng.integers(max(0, Wmax - 1), Wmax + 1)) if Wmax else 0
        k = int(rng.integers(0, 30))
        Lw = int(rng.integers(1, 12))
        tier = bool(rng.integers(0, 2)) and ws % 8 == 0
        p = _lib.evict_plan(T, W, s, ws, k, Lw, tier)
        scores = rng.random((2, 3, W)).astype(np.float32)
        ret = O.retain_window_indices(scores, k, Lw)
        tok = O.expand_to_token_indices(ret, s, ws, T)
        assert p.retained_windows == ret.shape[1]
        assert p.seq_len_new == tok.shape[1]
        assert p.local_windows == min(Lw, W)
        assert p.tier_pages_new == (p.kept_evictable * ws // 8 if tier else 0)


# -- config (reference config.py semantics) -----------------------------------------------

def test_config_resolve_matches_reference_goldens():
    for c in json.load(open(os.path.join(G, "resolve.json"))):
        mc = FakeModelConfig(num_key_value_heads=c["num_kv_heads"], head_dim=c["head_dim"])
        dt = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}[c["dtype"]]
        cfg = WindowedCacheConfig(c["window_size"], c["num_sink_tokens"], c["local_window_size"],
                                  c["cache_budget"])
        r = cfg.resolve(c["prefill_len"], mc, dt, c["max_tokens"])
        assert r.__dict__ == c["resolved"]


def test_config_validation_messages():
    with pytest.raises(ValueError, match="float"):
        _cfg(cache_budget=1)
    with pytest.raises(ValueError, match="bool"):
        _cfg(cache_budget=True)
    with pytest.raises(ValueError, match="must be > 0"):
        _cfg(window_size=0)
    with pytest.raises(ValueError, match="multiple of window_size"):
        _cfg(local_window_size=12)
    with pytest.raises(ValueError, match="in \\(0, 1\\]"):
        _cfg(local_window_size=1.5)
    with pytest.raises(ValueError, match="int4_tier needs window_size"):
        _cfg(window_size=5, local_window_size=10, int4_tier=True)
    with pytest.raises(ValueError, match="total_budget_tokens"):
        _cfg(cache_budget=0.05, num_sink_tokens=10, local_window_size=40).resolve(
            100, FakeModelConfig(), torch.float16, 50)


def test_gqa_byte_accounting():
    r = _cfg(cache_budget=0.5, local_window_size=8).resolve(100, FakeModelConfig(), torch.float16, 128)
    assert r.bytes_per_token == 8 * 128 * 2 * 2


# -- factory ----------------------------------------------------------------------------------

def test_factory_returns_trio_and_rejects_unknown():
    C, Cfg, hook = get_cache_classes("b200")
    assert C.__name__ == "WindowedCache" and Cfg is WindowedCacheConfig and callable(hook)
    with pytest.raises(ConfigValidationError):
        get_cache_classes("eager_v2")
    validate_backend_attn_pairing("b200", "stickykv_b200")
    with pytest.raises(ConfigValidationError):
        validate_backend_attn_pairing("b200", "eager")


def test_cache_construction_needs_no_gpu_and_refuses_beam_search():
    C, Cfg, _ = get_cache_classes("b200")
    cache = C(_cfg(), 100, FakeModelConfig(), torch.float16, None, num_layers=2, max_tokens=10)
    assert cache.get_seq_length(0) == 0 and cache.get_max_length() is None
    assert cache.resolved.top_k_windows == 3   # int(0.4*110*4096)//4096 = 44; (44-4-16)//8
    with pytest.raises(NotImplementedError):
        cache.reorder_cache(torch.tensor([0]))
    with pytest.raises(RuntimeError, match="CUDA"):
        cache.update(torch.zeros(1, 8, 4, 128, dtype=torch.float16),
                     torch.zeros(1, 8, 4, 128, dtype=torch.float16), 0)


# -- hooks / telemetry --------------------------------------------------------------------------

def test_hook_handles_idempotent_and_null_telemetry():
    h = HookHandles()
    h.remove()
    h.remove()
    assert h._removed
    t = NullTelemetry()
    t.record_scores(0, 0, torch.zeros(1, 4, 8))
    assert t.get_records(0) == []


def test_padded_batches_are_refused():
    """transformers builds no mask for an unknown attention implementation;
    this package registers a mask function with its own that builds no mask
    without a 2-D padding mask and otherwise defers to the sdpa one (None for
    an unpadded batch), so a mask reaching the attention means padding, and
    the attention refuses it."""
    from transformers.masking_utils import ALL_MASK_ATTENTION_FUNCTIONS
    from stickykv_b200.hooks import ATTN_IMPLEMENTATION, _register_attention, stickykv_attention
    _register_attention()
    assert ATTN_IMPLEMENTATION in ALL_MASK_ATTENTION_FUNCTIONS
    from stickykv_b200.hooks import padding_mask
    assert padding_mask(1, 1, 5, attention_mask=None) is None  # no padding mask: no mask, even when capturing

    class Attn(torch.nn.Module):
        layer_idx = 0
        _skv_cache = object()

    q = torch.zeros(2, 4, 6, 16)
    k = torch.zeros(2, 2, 6, 16)
    mask = torch.ones(2, 1, 6, 6, dtype=torch.bool)
    with pytest.raises(NotImplementedError, match="padded"):
        stickykv_attention(Attn(), q, k, k, mask)


def _install(seq_len):
    captured = {}

    class Dec(torch.nn.Module):
        def forward(self, **kw):
            captured.update(kw)

    dec = Dec()

    class Model:
        def get_decoder(self):
            return dec

    class Cache:
        def get_seq_length(self, layer_idx=0):
            return seq_len

    handles = HookHandles()
    install_position_override_hook(Model(), Cache(), handles)
    return dec, captured, handles


def test_position_override_prefill_and_decode():
    # reference tests/test_windowed_cache.py:770-816
    dec, cap, h = _install(0)
    dec(input_ids=torch.zeros(1, 8, dtype=torch.long), position_ids=torch.arange(8)[None],
        cache_position=torch.arange(8), attention_mask=torch.ones(1, 8, dtype=torch.long))
    assert cap["cache_position"].tolist() == list(range(8)) and cap["attention_mask"] is not None
    h.remove()
    dec, cap, h = _install(5)
    dec(input_ids=torch.zeros(1, 1, dtype=torch.long), position_ids=torch.tensor([[42]]),
        cache_position=torch.tensor([42]), attention_mask=torch.ones(1, 43, dtype=torch.long))
    assert cap["cache_position"].tolist() == [5] and cap["position_ids"].tolist() == [[5]]
    assert cap["attention_mask"] is None
    h.remove()
    dec(input_ids=torch.zeros(1, 1, dtype=torch.long), position_ids=torch.tensor([[42]]),
        cache_position=torch.tensor([42]), attention_mask=torch.ones(1, 43, dtype=torch.long))
    assert cap["cache_position"].tolist() == [42]


def test_no_per_token_python_loops_in_host_hot_path():
    """The reference bans for-loops over batch/head/token/window in its hot
    path (tests/test_windowed_cache.py:605-624); the host side here has none."""
    import ast
    import inspect
    from stickykv_b200 import cache, config, hooks
    banned = {"batch", "b", "head", "h", "token", "tok", "t", "window", "w", "n"}
    for mod in (cache, config, hooks):
        for node in ast.walk(ast.parse(inspect.getsource(mod))):
            if isinstance(node, ast.For) and isinstance(node.target, ast.Name):
                assert node.target.id.lower() not in banned, (mod.__name__, node.target.id)


def test_cfg1_model_and_prompt_reproduce_the_golden_prefill():
    """The end-to-end fixture's model is rebuilt from seeds on every machine:
    its plain-transformers prefill (no cache, full attention) must give the
    first-step logits the reference recorded."""
    import numpy as np
    import torch

    from tests import _cfg1 as C1
    z = np.load(os.path.join(os.path.dirname(__file__), "golden", "cfg1_e2e.npz"))
    model = C1.build_model()
    with torch.no_grad():
        lg = model(input_ids=C1.prompt(), use_cache=False).logits[0, -1].float()
    assert int(lg.argmax()) == int(z["tokens"][0])
    np.testing.assert_allclose(lg[torch.as_tensor(z["top_i"][0])].numpy(), z["top_v"][0], atol=1e-5, rtol=0)
