"""``WindowedCache`` for B200: the HF ``Cache`` drop-in of the reference's
modules/windowed_cache/cache.py:30-300, driving the native kernels.

Host orchestration only (Python ints, no device syncs).  Per layer the device
state lives in preallocated buffers:

* two fp stores (ping-pong) ``[B, Hkv, cap, D]`` in the KV dtype: sinks at
  slots ``[0, s)``, then the tokens after the int4 tier in logical order;
* with ``int4_tier``: one pool of int4 pages ``[B, Hkv, pages, page_bytes]``
  and two page tables (ping-pong) ``[B, pages]``;
* two fp32 window-score accumulators ``[B, Hq, Wcap]`` and two original-id
  tables ``[B, Wcap]`` (ping-pong), so compaction never races with itself.

Counts (tokens, pages, windows) are identical for every row and tracked on
the host; eviction counts come from ``skv_evict_plan_compute`` so the host
never reads device memory.
"""

from __future__ import annotations

import contextlib
import ctypes as C
import math
from typing import Any, Dict, List, Optional, Tuple

import torch
from torch import Tensor

from . import _lib
from ._lib import EvictArgs, LayerDesc, check, lib
from .config import ResolvedConfig, WindowedCacheConfig
from .telemetry import NullTelemetry, Telemetry

try:
    from transformers import Cache as _HFCacheBase
except ImportError:  # pragma: no cover
    _HFCacheBase = object  # type: ignore[assignment,misc]

_DT = {torch.float32: _lib.SKV_F32, torch.float16: _lib.SKV_F16, torch.bfloat16: _lib.SKV_BF16}
TAIL_WINDOWS = 8  # score/id slots the eviction kernel seeds past the retained windows


def _ptr(t: Optional[Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


# torch's own accessors of the current device and of a device's current raw
# stream (what torch.cuda.current_device / current_stream(...).cuda_stream
# return, without building a Stream object: they run on every native call)
_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)
_cur_dev = getattr(torch._C, "_cuda_getDevice", None)


def _stream(device: torch.device) -> int:
    if _raw_stream is not None and _cur_dev is not None:
        return _raw_stream(device.index if device.index is not None else _cur_dev())
    return torch.cuda.current_stream(device).cuda_stream


def _on(device: torch.device):
    """Make ``device`` current for a native call (kernels launch on the
    current device; the stream passed with them belongs to ``device``).
    Layers of one model may sit on different GPUs (``device_map``)."""
    if device.index is None or device.index == (_cur_dev() if _cur_dev is not None else torch.cuda.current_device()):
        return contextlib.nullcontext()
    return torch.cuda.device(device)


class _Side:
    """One half of the ping-pong state."""

    __slots__ = ("k", "v", "table", "scores", "ids", "desc", "desc_key")

    def __init__(self) -> None:
        self.k: Optional[Tensor] = None
        self.v: Optional[Tensor] = None
        self.table: Optional[Tensor] = None
        self.scores: Optional[Tensor] = None
        self.ids: Optional[Tensor] = None
        self.desc: Optional[LayerDesc] = None   # ABI descriptor of this side, rebuilt when
        self.desc_key: Optional[tuple] = None   # its buffers, the page pool or the rope table change


class LayerState:
    """Device buffers and host counters of one layer.

    Exposes the reference ``CacheState`` view used by its runners
    (``window_scores [B,Hq,W]``, ``original_window_ids [B,W]``,
    ``position_ids [B,T]``, ``key_states``/``value_states``)."""

    def __init__(self) -> None:
        self.sides: List[_Side] = [_Side(), _Side()]
        self.cur = 0
        self.pages: Optional[Tensor] = None
        self.T = 0
        self.tier_pages = 0
        self.W = 0
        self.has_scores = False
        self.next_window_id = 0
        self.last_update_prefill = False
        self.allocated = False
        self.evictions = 0  # evictions run so far (steady state after the second)
        # one decode token whose append is fused into the next decode call
        self.pending: Optional[Tuple[Tensor, Tensor]] = None
        self.flush = None  # writes a pending token (set by the cache)
        self.materialize = None  # (keys, values) of an int4-tier cache (set by the cache)
        self.decode_ws, self.decode_ws_T = 0, 0  # decode workspace bytes, valid up to decode_ws_T
        # geometry copied at allocation
        self.B = self.Hkv = self.Hq = self.D = 0
        self.dtype: Optional[torch.dtype] = None
        self.device: Optional[torch.device] = None
        self.scores_cap = 0
        self.page_cap = 0
        self.num_sink = 0

    # -- reference-compatible views --------------------------------------------
    def _fp_view(self, which: str) -> Optional[Tensor]:
        if not self.allocated:
            return None
        if self.pending is not None:
            self.flush(self)
        if self.tier_pages:
            return self.materialize(self)[0 if which == "k" else 1]
        side = self.sides[self.cur]
        buf = side.k if which == "k" else side.v
        s = min(self.num_sink, self.T)
        s_pad = (self.num_sink + 7) // 8 * 8
        rest = self.T - s
        return torch.cat([buf[:, :, :s], buf[:, :, s_pad:s_pad + rest]], dim=2)

    @property
    def key_states(self) -> Optional[Tensor]:
        """[B, Hkv, T, D] post-RoPE keys in logical order (a copy; int4 tier
        tokens dequantised and rotated to their current positions)."""
        return self._fp_view("k")

    @property
    def value_states(self) -> Optional[Tensor]:
        return self._fp_view("v")

    @property
    def seq_length(self) -> int:
        return self.T

    @property
    def window_scores(self) -> Optional[Tensor]:
        if not self.has_scores:
            return None
        return self.sides[self.cur].scores[:, :, : self.W]

    @property
    def original_window_ids(self) -> Optional[Tensor]:
        if not self.has_scores:
            return None
        return self.sides[self.cur].ids[:, : self.W]

    @property
    def position_ids(self) -> Optional[Tensor]:
        if not self.allocated:
            return None
        return torch.arange(self.T, device=self.device).unsqueeze(0).expand(self.B, -1)


class WindowedCache(_HFCacheBase):
    """Windowed KV cache with H2O-style cumulative eviction, B200 kernels.

    Constructor and methods follow the reference (cache.py:53-300):
    ``WindowedCache(config, prefill_len, model_config, kv_dtype, rope_module,
    num_layers, max_tokens, telemetry=None)``.  Attention must run through the
    ``stickykv_b200`` attention implementation that ``install_score_hooks``
    selects: decode attention, score accumulation and eviction all happen in
    the native library.
    """

    def __init__(self, config: WindowedCacheConfig, prefill_len: int, model_config: Any,
                 kv_dtype: torch.dtype, rope_module: torch.nn.Module, num_layers: int,
                 max_tokens: int, telemetry: Optional[Telemetry] = None) -> None:
        if isinstance(_HFCacheBase, type) and _HFCacheBase is not object:
            try:
                super().__init__(layers=[])
            except (TypeError, ValueError):
                pass
        self.config = config
        self.resolved: ResolvedConfig = config.resolve(prefill_len, model_config, kv_dtype, max_tokens)
        self.rope_module = rope_module
        self.num_layers = num_layers
        self.prefill_len = prefill_len
        self.max_tokens = max_tokens
        self.kv_dtype = kv_dtype
        self.model_config = model_config
        self.telemetry = telemetry if telemetry is not None else NullTelemetry()
        self.tier = bool(config.int4_tier)
        self.local_windows = self.resolved.local_tokens // self.resolved.window_size
        # an evicting one-token step appends inside the eviction (skv_evict_append)
        # instead of a separate skv_append launch before it
        self.fuse_evict_append = True
        self._states: List[LayerState] = [self._new_state() for _ in range(num_layers)]
        self._generation_step: List[int] = [0] * num_layers
        self._prefill_done: List[bool] = [False] * num_layers
        self.cache_kwargs: Dict[int, Dict[str, Any]] = {i: {} for i in range(num_layers)}
        # per device: layers placed on several GPUs each use their own
        self._rope: Dict[torch.device, Tuple[Tensor, Tensor]] = {}
        self._rope_positions: Dict[torch.device, int] = {}
        self._ws: Dict[torch.device, Tensor] = {}
        self._retained: Dict[torch.device, Tensor] = {}
        self.layers = []

    # -- HF Cache surface ---------------------------------------------------------------
    def get_seq_length(self, layer_idx: int = 0) -> int:
        return self._states[layer_idx].T

    def get_max_length(self) -> Optional[int]:
        return None

    def get_max_cache_shape(self, layer_idx: int = 0) -> int:
        return -1

    def get_mask_sizes(self, query_length, layer_idx: int = 0) -> Tuple[int, int]:
        q = int(query_length.shape[0]) if torch.is_tensor(query_length) else int(query_length)
        return self.get_seq_length(layer_idx) + q, 0

    @property
    def is_compileable(self) -> bool:
        return False

    @property
    def is_initialized(self) -> bool:
        return any(s.allocated for s in self._states)

    @property
    def is_sliding(self) -> List[bool]:
        return [False] * self.num_layers

    @property
    def max_batch_size(self) -> int:
        return self._states[0].B

    @property
    def max_cache_len(self) -> int:
        return -1

    def has_previous_state(self, layer_idx: Optional[int] = None) -> bool:
        return self._states[0 if layer_idx is None else layer_idx].T > 0

    def __len__(self) -> int:
        return self.num_layers

    def reorder_cache(self, beam_idx: Tensor) -> None:
        raise NotImplementedError(
            "WindowedCache does not support beam search (reorder_cache). "
            "Use greedy or sampling decoding.")

    def crop(self, max_length: int) -> None:
        raise NotImplementedError("WindowedCache cannot be cropped: eviction already compacts it")

    def reset(self) -> None:
        for i in range(self.num_layers):
            self._states[i] = self._new_state()
            self._generation_step[i] = 0
            self._prefill_done[i] = False
            self.cache_kwargs[i] = {}

    def _new_state(self) -> LayerState:
        st = LayerState()
        st.flush = self._flush
        st.materialize = self._materialize
        return st

    def _materialize(self, st: LayerState) -> Tuple[Tensor, Tensor]:
        """Keys and values of every retained token, tier included, as plain
        [B, Hkv, T, D] tensors in the KV dtype (skv_materialize)."""
        k = torch.empty(st.B, st.Hkv, st.T, st.D, dtype=st.dtype, device=st.device)
        v = torch.empty_like(k)
        d = self._desc(st, st.sides[st.cur])
        with _on(st.device):
            check(lib().skv_materialize(C.byref(d), st.T, st.tier_pages, k.data_ptr(), v.data_ptr(),
                                        _stream(st.device)), "skv_materialize")
        return k, v

    # -- allocation ------------------------------------------------------------------------
    def _caps(self, P: int) -> Tuple[int, int, int, int]:
        r = self.resolved
        s, ws = r.num_sink_tokens, r.window_size
        s_pad = (s + 7) // 8 * 8
        budget = r.total_budget_tokens
        steady = s_pad + budget + 2 * ws + 16
        first = s_pad + P + ws + 16
        cap_a = -(-max(first, steady) // 8) * 8
        cap_b = -(-steady // 8) * 8
        max_T = max(P + ws + 2, budget + 2 * ws + 2)
        wcap = -(-(max_T + ws) // ws) + TAIL_WINDOWS + 2
        return cap_a, cap_b, wcap, max_T

    def _allocate(self, st: LayerState, key: Tensor, P: int) -> None:
        if key.device.type != "cuda":
            raise RuntimeError("stickykv_b200 needs CUDA tensors (no CPU path)")
        if key.dtype not in _DT:
            raise NotImplementedError(f"KV dtype {key.dtype} is not supported")
        lib()  # fail loudly now if the library is missing
        B, Hkv, _, D = key.shape
        mc = self.model_config
        Hq = getattr(mc, "num_attention_heads", Hkv)
        dev, dt = key.device, key.dtype
        cap_a, cap_b, wcap, max_T = self._caps(P)
        st.B, st.Hkv, st.Hq, st.D, st.dtype, st.device = B, Hkv, Hq, D, dt, dev
        st.num_sink = self.resolved.num_sink_tokens
        st.scores_cap = wcap
        for side, cap in zip(st.sides, (cap_a, cap_b)):
            side.k = torch.empty(B, Hkv, cap, D, dtype=dt, device=dev)
            side.v = torch.empty(B, Hkv, cap, D, dtype=dt, device=dev)
            side.scores = torch.zeros(B, Hq, wcap, dtype=torch.float32, device=dev)
            side.ids = torch.arange(wcap, device=dev, dtype=torch.int64).unsqueeze(0).repeat(B, 1)
        if self.tier:
            ppw = self.resolved.window_size // _lib.PAGE_TOKENS
            st.page_cap = max(1, self.resolved.top_k_windows * ppw + 2 * ppw)
            st.pages = torch.empty(B, Hkv, st.page_cap, _lib.page_bytes(D), dtype=torch.uint8, device=dev)
            for side in st.sides:
                side.table = torch.zeros(B, st.page_cap, dtype=torch.int32, device=dev)
        self._ensure_rope(max_T + 64, D, dev)
        st.allocated = True

    def _ensure_rope(self, n: int, D: int, dev: torch.device) -> None:
        have = self._rope_positions.get(dev, 0)
        if have >= n:
            return
        n = max(n, 2 * have)
        x = torch.zeros(1, 1, 1, D, dtype=torch.float32, device=dev)
        pos = torch.arange(n, device=dev).unsqueeze(0)
        with torch.no_grad():
            cos, sin = self.rope_module(x, pos)
        cos = cos.reshape(-1, cos.shape[-1])[:n].float()
        sin = sin.reshape(-1, sin.shape[-1])[:n].float()
        # the layout check reads the table back (a device sync): only when the
        # table is first built, not when it grows during decoding
        if cos.shape[-1] != D or (have == 0 and (not torch.equal(cos[:, : D // 2], cos[:, D // 2:]) or
                                                not torch.equal(sin[:, : D // 2], sin[:, D // 2:]))):
            raise NotImplementedError("rotary module must use the rotate-half layout cat(f, f)")
        self._rope[dev] = (cos[:, : D // 2].contiguous(), sin[:, : D // 2].contiguous())
        self._rope_positions[dev] = n

    def _grow_side(self, st: LayerState, side: _Side, need_slots: int) -> None:
        cap = side.k.shape[2]
        if need_slots <= cap:
            return
        new_cap = -(-max(need_slots, 2 * cap) // 8) * 8
        for name in ("k", "v"):
            old = getattr(side, name)
            new = torch.empty(st.B, st.Hkv, new_cap, st.D, dtype=st.dtype, device=st.device)
            new[:, :, :cap].copy_(old)
            setattr(side, name, new)

    def _desc(self, st: LayerState, side: _Side) -> LayerDesc:
        rope = self._rope[st.device]
        key = side.desc_key
        # the key holds the buffers themselves: identity checks cost nothing
        # per call, and a held buffer cannot be freed and its address reused
        if (key is not None and key[0] is side.k and key[1] is side.v and key[2] is side.table
                and key[3] is rope[0] and key[4] is st.pages):
            return side.desc
        r = self.resolved
        d = LayerDesc()
        d.batch, d.num_kv_heads, d.num_q_heads, d.head_dim = st.B, st.Hkv, st.Hq, st.D
        d.kv_dtype = _DT[st.dtype]
        d.window_size, d.num_sink = r.window_size, r.num_sink_tokens
        d.sink_pad = (r.num_sink_tokens + 7) // 8 * 8
        d.fp_capacity = side.k.shape[2]
        d.k_fp, d.v_fp = side.k.data_ptr(), side.v.data_ptr()
        if self.tier:
            d.tier_page_capacity = st.page_cap
            d.tier_pages = st.pages.data_ptr()
            d.tier_table = side.table.data_ptr()
        d.rope_cos, d.rope_sin = rope[0].data_ptr(), rope[1].data_ptr()
        d.rope_positions = self._rope_positions[st.device]
        side.desc, side.desc_key = d, (side.k, side.v, side.table, rope[0], st.pages)
        return d

    def _fp_slots(self, T: int, tier_pages: int) -> int:
        s = self.resolved.num_sink_tokens
        if T <= s:
            return T
        return (s + 7) // 8 * 8 + (T - s - tier_pages * _lib.PAGE_TOKENS)

    def _workspace(self, nbytes: int, device: torch.device) -> Tensor:
        ws = self._ws.get(device)
        if ws is None or ws.numel() < nbytes:
            ws = torch.empty(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
            self._ws[device] = ws
        return ws

    # -- update (reference cache.py:110-293) ------------------------------------------------
    def update(self, key_states: Tensor, value_states: Tensor, layer_idx: int,
               cache_kwargs: Optional[Dict[str, Any]] = None) -> Tuple[Tensor, Tensor]:
        """Append this step's keys/values, accumulate external window scores,
        evict every ``window_size`` decode steps.  Returns the step's own
        key/value states: the ``stickykv_b200`` attention reads the cache
        directly.  A one-token decode step that does not evict defers its
        append to the attention call, which fuses it into the same launch
        (``skv_decode_attention_append``); the length already counts it."""
        st = self._states[layer_idx]
        n_new = key_states.shape[2]
        if not st.allocated:
            self._allocate(st, key_states, max(n_new, self.prefill_len))
        if st.pending is not None:
            self._flush(st)
        is_prefill = not self._prefill_done[layer_idx]
        self._prefill_done[layer_idx] = True
        st.last_update_prefill = is_prefill

        lk = self.cache_kwargs.get(layer_idx)
        if cache_kwargs or lk:
            merged: Dict[str, Any] = dict(cache_kwargs or {})
            merged.update(lk or {})
            ext = merged.get("window_scores")
            if lk is not None and "window_scores" in lk:
                del lk["window_scores"]
            if ext is not None:
                self._add_scores(st, ext)

        step = self._generation_step[layer_idx]
        ws = self.resolved.window_size
        evict = not is_prefill and step > 0 and step % ws == 0 and st.has_scores
        fresh = None
        if not is_prefill and n_new == 1 and not evict:
            self._defer_append(st, key_states, value_states)
        elif evict and n_new == 1 and self.fuse_evict_append:  # the token rides in the eviction
            fresh = self._append(st, key_states, value_states, launch=False)
        else:
            self._append(st, key_states, value_states)
        if evict:
            self._evict(st, layer_idx, step, fresh)
        if not is_prefill:
            self._generation_step[layer_idx] = step + 1
        return key_states, value_states

    @staticmethod
    def _kv_ok(k: Tensor, v: Tensor) -> bool:
        es, ks = k.element_size(), k.stride()
        return (ks == v.stride() and ks[3] == 1 and k.data_ptr() % 16 == 0 and v.data_ptr() % 16 == 0
                and (ks[0] * es) % 16 == 0 and (ks[1] * es) % 16 == 0 and (ks[2] * es) % 16 == 0)

    def _defer_append(self, st: LayerState, k: Tensor, v: Tensor) -> None:
        if not self._kv_ok(k, v):
            k, v = k.contiguous(), v.contiguous()
        self._grow_side(st, st.sides[st.cur], self._fp_slots(st.T + 1, st.tier_pages))
        self._ensure_rope(st.T + 67, st.D, st.device)
        st.pending = (k, v)
        st.T += 1

    def _flush(self, st: LayerState) -> None:
        """Write a deferred decode token with a plain append."""
        k, v = st.pending
        st.pending = None
        d = self._desc(st, st.sides[st.cur])
        with _on(st.device):
            check(lib().skv_append(C.byref(d), st.T - 1, st.tier_pages, k.data_ptr(), v.data_ptr(),
                                   k.stride(0), k.stride(1), k.stride(2), 1, _stream(st.device)),
                  "skv_append")

    def _append(self, st: LayerState, k: Tensor, v: Tensor, launch: bool = True):
        """Append n tokens; with ``launch=False`` only the bookkeeping (capacity,
        rotary rows, length) and return the (k, v) that the eviction's
        ``skv_evict_append`` reads the one token from."""
        n_new = k.shape[2]
        if not self._kv_ok(k, v):
            k, v = k.contiguous(), v.contiguous()
        side = st.sides[st.cur]
        need = self._fp_slots(st.T + n_new, st.tier_pages)
        self._grow_side(st, side, need)
        max_T = st.T + n_new + 2
        self._ensure_rope(max_T + 64, st.D, st.device)
        if launch:
            d = self._desc(st, side)
            with _on(st.device):
                check(lib().skv_append(C.byref(d), st.T, st.tier_pages, k.data_ptr(), v.data_ptr(),
                                       k.stride(0), k.stride(1), k.stride(2), n_new, _stream(st.device)),
                      "skv_append")
        st.T += n_new
        return None if launch else (k, v)

    def _add_scores(self, st: LayerState, new: Tensor) -> None:
        """Accumulate externally computed window scores (reference cache.py:163-228)."""
        W_new = new.shape[-1]
        if W_new > st.scores_cap:
            raise MemoryError(f"{W_new} windows exceed the score capacity {st.scores_cap}")
        acc = st.sides[st.cur].scores
        if not st.has_scores:
            acc.zero_()
            st.sides[st.cur].ids.copy_(torch.arange(st.scores_cap, device=st.device).unsqueeze(0))
            st.has_scores = True
            st.W = 0
            st.next_window_id = 0
        acc[:, :, :W_new] += new.to(device=st.device, dtype=torch.float32)
        if W_new > st.W:
            st.next_window_id += W_new - st.W
            st.W = W_new

    def _note_windows(self, st: LayerState) -> None:
        s, ws = self.resolved.num_sink_tokens, self.resolved.window_size
        W_now = -(-(st.T - s) // ws) if st.T > s else 0
        if not st.has_scores:
            st.has_scores = True
            st.W = W_now
            st.next_window_id = W_now
        elif W_now > st.W:
            st.next_window_id += W_now - st.W
            st.W = W_now

    # -- eviction (reference cache.py:230-286) ------------------------------------------------
    def _evict(self, st: LayerState, layer_idx: int, step: int, fresh=None) -> None:
        r = self.resolved
        plan = _lib.evict_plan(st.T, st.W, r.num_sink_tokens, r.window_size, r.top_k_windows,
                               self.local_windows, self.tier)
        src, dst = st.sides[st.cur], st.sides[1 - st.cur]
        need = self._fp_slots(plan.seq_len_new, plan.tier_pages_new) + r.window_size + 2
        cap_dst = dst.k.shape[2]
        if cap_dst < need:
            self._grow_side(st, dst, need)
        elif cap_dst > 4 * need + 4096:  # the prefill-sized store is no longer needed
            dst.k = torch.empty(st.B, st.Hkv, -(-2 * need // 8) * 8, st.D, dtype=st.dtype, device=st.device)
            dst.v = torch.empty_like(dst.k)
        want_tel = bool(getattr(self.telemetry, "enabled", False))
        retained = self._retained.get(st.device)
        if want_tel:
            if retained is None or retained.shape != (st.B, st.scores_cap):
                retained = torch.zeros(st.B, st.scores_cap, dtype=torch.int32, device=st.device)
                self._retained[st.device] = retained
            pre = src.scores[:, :, : st.W].clone()
        a = EvictArgs()
        a.seq_len, a.tier_pages, a.num_windows = st.T, st.tier_pages, st.W
        a.top_k_windows, a.local_windows = r.top_k_windows, self.local_windows
        a.scores_capacity = st.scores_cap
        a.scores_src, a.scores_dst = src.scores.data_ptr(), dst.scores.data_ptr()
        a.ids_src, a.ids_dst = src.ids.data_ptr(), dst.ids.data_ptr()
        a.retained_out = retained.data_ptr() if want_tel else None
        a.next_window_id = st.next_window_id
        ds, dd = self._desc(st, src), self._desc(st, dst)
        nbytes = lib().skv_evict_workspace_size(C.byref(ds), st.W)
        ws = self._workspace(nbytes, st.device)
        with _on(st.device):
            if fresh is None:
                check(lib().skv_evict(C.byref(ds), C.byref(dd), C.byref(a), ws.data_ptr(), ws.numel(),
                                      _stream(st.device)), "skv_evict")
            else:  # this step's token, never written to src, moves into dst with the eviction
                k, v = fresh
                check(lib().skv_evict_append(C.byref(ds), C.byref(dd), C.byref(a), k.data_ptr(), v.data_ptr(),
                                             k.stride(0), k.stride(1), ws.data_ptr(), ws.numel(),
                                             _stream(st.device)), "skv_evict_append")
        if want_tel:
            ret = retained[:, : plan.retained_windows].long()
            self.telemetry.record_scores(layer_idx, step, pre, self._token_indices(ret, st.T))
        st.cur ^= 1
        st.T = plan.seq_len_new
        st.tier_pages = plan.tier_pages_new
        st.W = plan.retained_windows
        st.evictions += 1

    def _token_indices(self, retained: Tensor, total: int) -> Tensor:
        """Retained windows -> token indices (reference policy.py:152-209); telemetry only."""
        r = self.resolved
        B = retained.shape[0]
        dev = retained.device
        sink = torch.arange(r.num_sink_tokens, device=dev).unsqueeze(0).expand(B, -1)
        tok = (r.num_sink_tokens + retained.unsqueeze(-1) * r.window_size
               + torch.arange(r.window_size, device=dev)).reshape(B, -1)
        idx = torch.cat([sink, tok], dim=1)
        return idx[:, : int((idx[0] < total).sum())]

    # -- attention entry points (called by the stickykv_b200 attention function) ----------
    def decode_attention(self, layer_idx: int, query: Tensor, scaling: float) -> Tensor:
        """One-token attention over the retained cache; accumulates window mass.
        query [B, Hq, 1, D] -> out [B, 1, Hq, D].  A deferred append of this
        step's token runs in the same native call."""
        st = self._states[layer_idx]
        if query.stride(-1) != 1:
            query = query.contiguous()
        out = torch.empty(st.B, 1, st.Hq, st.D, dtype=st.dtype, device=st.device)
        side = st.sides[st.cur]
        d = self._desc(st, side)
        L = lib()
        if st.T > st.decode_ws_T:  # workspace sized for twice the length, re-queried rarely
            st.decode_ws_T = 2 * st.T
            st.decode_ws = L.skv_decode_workspace_size(C.byref(d), st.decode_ws_T)
        ws = self._workspace(st.decode_ws, st.device)
        # q[:, :, 0, :] and out[:, 0] by strides (no views)
        qst, ost = query.stride(), out.stride()
        qs_b, qs_h, os_b, os_h = qst[0], qst[1], ost[0], ost[2]
        with _on(st.device):
            if st.pending is not None:
                k, v = st.pending
                st.pending = None
                check(L.skv_decode_attention_append(
                    C.byref(d), st.T, st.tier_pages, k.data_ptr(), v.data_ptr(), k.stride(0), k.stride(1),
                    query.data_ptr(), qs_b, qs_h, out.data_ptr(), os_b, os_h, float(scaling),
                    side.scores.data_ptr(), st.scores_cap, ws.data_ptr(), ws.numel(), _stream(st.device)),
                    "skv_decode_attention_append")
            else:
                check(L.skv_decode_attention(
                    C.byref(d), st.T, st.tier_pages, query.data_ptr(), qs_b, qs_h, out.data_ptr(), os_b,
                    os_h, float(scaling), side.scores.data_ptr(), st.scores_cap, ws.data_ptr(), ws.numel(),
                    _stream(st.device)), "skv_decode_attention")
        self._note_windows(st)
        return out

    def prefill_attention(self, layer_idx: int, query: Tensor, key: Tensor, value: Tensor,
                          scaling: float) -> Tensor:
        """Causal attention over the prompt; seeds the window scores with the
        prompt's column mass.  query [B,Hq,P,D], key/value [B,Hkv,P,D] ->
        out [B, P, Hq, D]."""
        st = self._states[layer_idx]
        P = query.shape[2]
        q, k, v = query.contiguous(), key.contiguous(), value.contiguous()
        out = torch.empty(st.B, P, st.Hq, st.D, dtype=st.dtype, device=st.device)
        side = st.sides[st.cur]
        side.scores.zero_()
        d = self._desc(st, side)
        L = lib()
        nbytes = L.skv_prefill_workspace_size(C.byref(d), P)
        ws = self._workspace(nbytes, st.device)
        with _on(st.device):
            check(L.skv_prefill_attention(C.byref(d), P, q.data_ptr(), k.data_ptr(), v.data_ptr(),
                                          out.data_ptr(), float(scaling), side.scores.data_ptr(),
                                          st.scores_cap, ws.data_ptr(), ws.numel(), _stream(st.device)),
                  "skv_prefill_attention")
        st.has_scores = False
        self._note_windows(st)
        return out
