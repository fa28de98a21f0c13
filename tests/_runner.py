"""The reference parity runner's per-step capture, restated for the tests.

The reference's Suite-A runner (modules/evaluation/ours_parity_runner.py)
drives a windowed cache teacher-forced and, after every model call, reads
``cache._states[li].window_scores`` ([B, H_q, W]), ``original_window_ids``
([B, W]) and ``cache._generation_step`` (lines 312-402), turns each (row,
layer) into top-K window ids, fp16 scores, retained ids and retained fp16
scores (``_extract_row_retained``, lines 35-101), pads the per-step arrays
and writes one npz (lines 408-476 and 521-537).  These helpers do the same
for one sample so a test can run the capture against this package's cache
and compare it with the reference's own capture (tests/golden/cfg1_runner.npz).
"""

from __future__ import annotations

import json
import math
from typing import Dict, List, Optional, Sequence, Tuple, Union

import numpy as np
import torch

RUNNER_KEYS = ("top_window_indices", "window_scores", "eviction_step_mask", "generated_tokens",
               "retained_window_ids", "retained_window_scores", "metadata_json")


def local_windows(W: int, ws: int, lws: Union[int, float]) -> int:
    """Windows at the end of the row that the runner counts as local
    (ours_parity_runner.py:61-71): a float ``lws`` is a fraction of the W
    windows' tokens, rounded up to whole windows."""
    if isinstance(lws, float):
        tokens = math.ceil(lws * max(W * ws, 1))
        tokens += (-tokens) % ws
        n = tokens // ws
    else:
        n = lws // ws
    return min(n, W)


def extract_row_retained(scores: torch.Tensor, orig: Optional[torch.Tensor], tk: int, ws: int,
                         lws: Union[int, float]) -> Tuple[np.ndarray, np.ndarray, np.ndarray, np.ndarray]:
    """One (row, layer)'s runner arrays from its [H_q, W] window scores and
    [W] original ids (None: identity), after ours_parity_runner.py:35-101:
    the top-K evictable windows by head mean (score order), the fp16 scores,
    the retained ids (top-K evictable and local, by original id) and their
    fp16 scores [H_q, M]."""
    scores = scores.detach().float().cpu()
    W = scores.shape[-1]
    ids = torch.arange(W) if orig is None else orig.detach().long().cpu()
    eW = W - local_windows(W, ws, lws)
    if eW > 0 and tk > 0:
        top = scores[:, :eW].mean(dim=0).topk(min(tk, eW)).indices
        top_ids = ids[top]
        tk_arr = top_ids.numpy()
    else:
        top = torch.zeros(0, dtype=torch.long)
        top_ids = torch.zeros(0, dtype=torch.long)
        tk_arr = np.zeros(min(tk, max(W, 1)), dtype=np.int64)
    loc = torch.arange(eW, W)
    compact = torch.cat([top, loc])
    orig_all = torch.cat([top_ids, ids[loc]])
    order = torch.argsort(orig_all)
    ret_sc = scores[:, compact[order]].to(torch.float16).numpy()
    return tk_arr, scores.to(torch.float16).numpy(), orig_all[order].numpy(), ret_sc


class RunnerCapture:
    """Per-step capture of one sample (batch row ``row``) over ``n_layers``
    layers, as the runner's loop body does after each model call."""

    def __init__(self, n_layers: int, tk: int, ws: int, lws: Union[int, float], row: int = 0):
        self.n_layers, self.tk, self.ws, self.lws, self.row = n_layers, tk, ws, lws, row
        self.evicted: List[bool] = []
        self.steps: List[Dict[str, list]] = []

    def step(self, cache) -> None:
        gs = cache._generation_step
        # update() advances the generation step after its eviction check
        # (ours_parity_runner.py:322-328)
        self.evicted.append(any((gs[li] - 1) > 0 and (gs[li] - 1) % self.ws == 0 for li in range(self.n_layers)))
        rec: Dict[str, list] = {k: [] for k in ("scores", "ids", "tk", "ws16", "ret_ids", "ret_sc16")}
        for li in range(self.n_layers):
            st = cache._states[li]
            sc, ids = st.window_scores, st.original_window_ids
            if sc is None:
                raise AssertionError(f"layer {li} has no window scores after a model call")
            row_ids = None if ids is None else ids[self.row]
            out = extract_row_retained(sc[self.row], row_ids, self.tk, self.ws, self.lws)
            rec["scores"].append(sc[self.row].float().cpu().numpy())
            rec["ids"].append(np.arange(sc.shape[-1]) if ids is None else ids[self.row].cpu().numpy())
            for key, val in zip(("tk", "ws16", "ret_ids", "ret_sc16"), out):
                rec[key].append(val)
        self.steps.append(rec)


def golden_steps(z, n_layers: int) -> Tuple[List[bool], List[Dict[str, list]]]:
    """Per-step records of tests/golden/cfg1_runner.npz (stored flat with
    per-step shapes) in :class:`RunnerCapture`'s layout."""
    two_d = {"scores", "ws16", "ret_sc16"}
    steps: List[Dict[str, list]] = [dict() for _ in range(len(z["evicted"]))]
    for key in ("scores", "ids", "tk", "ws16", "ret_ids", "ret_sc16"):
        for li in range(n_layers):
            flat, shapes = z[f"{key}_{li}"], z[f"{key}_{li}_shape"]
            off = 0
            for t, shp in enumerate(shapes):
                shp = tuple(int(x) for x in (shp if key in two_d else shp[:1]))
                n = int(np.prod(shp))
                steps[t].setdefault(key, []).append(flat[off:off + n].reshape(shp))
                off += n
            assert off == flat.size
    return [bool(x) for x in z["evicted"]], steps


def runner_arrays(evicted: Sequence[bool], steps: Sequence[Dict[str, list]], tokens: np.ndarray,
                  meta: dict) -> Dict[str, np.ndarray]:
    """The npz arrays of one sample with the runner's padding
    (ours_parity_runner.py:391-402 per step, 408-430 over steps, 521-537):
    top-K ids pad -1, scores pad 0 over heads and windows, retained ids pad -1
    and retained scores pad 0, all with a leading sample axis of 1."""
    topk, ws, rid, rsc = [], [], [], []
    for rec in steps:
        topk.append(np.stack(rec["tk"], 0))
        ws.append(np.stack(rec["ws16"], 0))
        m = max(len(x) for x in rec["ret_ids"])
        h = max(x.shape[0] for x in rec["ret_sc16"])
        rid.append(np.stack([np.pad(x, [(0, m - len(x))], constant_values=-1) for x in rec["ret_ids"]], 0))
        rsc.append(np.stack([np.pad(x, [(0, h - x.shape[0]), (0, m - x.shape[1])]) for x in rec["ret_sc16"]], 0))
    mW, mK = max(x.shape[-1] for x in ws), max(x.shape[-1] for x in topk)
    mH = max(x.shape[-2] for x in ws)
    ws = [np.pad(x, [(0, 0), (0, mH - x.shape[-2]), (0, mW - x.shape[-1])]) for x in ws]
    topk = [np.pad(x, [(0, 0), (0, mK - x.shape[-1])], constant_values=-1) for x in topk]
    mM, mHr = max(x.shape[-1] for x in rid), max(x.shape[-2] for x in rsc)
    rid = [np.pad(x, [(0, 0), (0, mM - x.shape[-1])], constant_values=-1) for x in rid]
    rsc = [np.pad(x, [(0, 0), (0, mHr - x.shape[-2]), (0, mM - x.shape[-1])]) for x in rsc]
    return {
        "top_window_indices": np.stack(topk, 0)[None],
        "window_scores": np.stack(ws, 0)[None],
        "eviction_step_mask": np.array(evicted, dtype=bool)[None],
        "generated_tokens": np.asarray(tokens)[None],
        "retained_window_ids": np.stack(rid, 0)[None],
        "retained_window_scores": np.stack(rsc, 0)[None],
        "metadata_json": np.array([json.dumps(meta)], dtype=object),
    }
