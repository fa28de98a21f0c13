"""The reference parity runner's npz (Suite A, modules/evaluation/
ours_parity_runner.py:312-537) produced against this package's cache.

CPU: the restated per-row extraction (tests/_runner.py) reproduces the
reference runner's own ``_extract_row_retained`` outputs recorded in
tests/golden/cfg1_runner.npz, and the padded npz arrays carry the runner's
keys, dtypes and shapes.

GPU: the fp32 cfg1 model (tests/_cfg1.py) runs teacher-forced through the
b200 backend with the runner's capture after every model call; every step's
window ids, eviction flag, top-K ids and retained ids equal the reference
eager backend's run, its window scores match within 1e-5 relative (the
reference holds a step's scores pending until the next update(); the
recorded reference state includes them, and a window they cover before the
state lists it), and the npz written from the
capture equals the one written from the reference's capture.
"""

import os

import numpy as np
import pytest
import torch

from tests import _cfg1 as C1
from tests import _runner as R

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "cfg1_runner.npz")


def _golden():
    z = np.load(GOLDEN)
    evicted, steps = R.golden_steps(z, 2)
    return z, evicted, steps


def test_restated_extraction_matches_reference_runner():
    z, _, steps = _golden()
    tk = int(z["top_k"])
    for t, rec in enumerate(steps):
        for li in range(2):
            out = R.extract_row_retained(torch.from_numpy(rec["scores"][li]), torch.from_numpy(rec["ids"][li]),
                                         tk, C1.WINDOW, C1.LOCAL)
            for key, got in zip(("tk", "ws16", "ret_ids", "ret_sc16"), out):
                want = rec[key][li]
                assert got.dtype == want.dtype and got.shape == want.shape, (t, li, key)
                np.testing.assert_array_equal(got, want, err_msg=f"step {t} layer {li} {key}")


def test_local_window_count_follows_runner_rounding():
    # 34 windows of 8 tokens, local 0.25: ceil(0.25 * 272) = 68 -> 72 tokens -> 9 windows
    assert R.local_windows(34, 8, 0.25) == 9
    assert R.local_windows(34, 8, 64) == 8
    assert R.local_windows(3, 8, 0.99) == 3
    assert R.local_windows(0, 8, 0.25) == 0


def test_runner_npz_schema(tmp_path):
    z, evicted, steps = _golden()
    arr = R.runner_arrays(evicted, steps, z["tokens"], {"cache_backend": "windowed"})
    assert tuple(arr) == R.RUNNER_KEYS
    T = len(steps)
    assert arr["top_window_indices"].shape[:3] == (1, T, 2) and arr["top_window_indices"].dtype == np.int64
    assert arr["window_scores"].shape[:4] == (1, T, 2, 4) and arr["window_scores"].dtype == np.float16
    assert arr["eviction_step_mask"].shape == (1, T) and arr["eviction_step_mask"].dtype == bool
    assert arr["retained_window_ids"].shape[:3] == (1, T, 2)
    assert arr["retained_window_scores"].shape[:4] == (1, T, 2, 4)
    assert arr["retained_window_scores"].shape[-1] == arr["retained_window_ids"].shape[-1]
    path = tmp_path / "parity_ours.npz"
    np.savez_compressed(path, **arr)
    back = np.load(path, allow_pickle=True)
    assert sorted(back.files) == sorted(R.RUNNER_KEYS)
    for k in R.RUNNER_KEYS[:-1]:
        np.testing.assert_array_equal(back[k], arr[k])
    # every retained id list is sorted, padded with -1 only at the end
    rid = arr["retained_window_ids"][0]
    for t in range(T):
        for li in range(2):
            row = rid[t, li]
            n = int((row >= 0).sum())
            assert (row[n:] == -1).all() and (np.diff(row[:n]) > 0).all()


@pytest.mark.gpu
def test_runner_capture_matches_reference_on_b200_backend(tmp_path):
    from stickykv_b200.cache_factory import get_cache_classes, validate_backend_attn_pairing
    z, evicted_ref, steps_ref = _golden()
    tokens = z["tokens"]
    model = C1.build_model().cuda()
    Cache, Config, install = get_cache_classes("b200")
    cfg = Config(window_size=C1.WINDOW, num_sink_tokens=C1.SINKS, local_window_size=C1.LOCAL,
                 cache_budget=C1.BUDGET)
    cache = Cache(cfg, C1.PROMPT_LEN, model.config, torch.float32, model.model.rotary_emb, 2, C1.STEPS)
    tk = cache.resolved.top_k_windows
    assert tk == int(z["top_k"])
    handles = install(model, cache, cfg)
    validate_backend_attn_pairing("b200", model.config._attn_implementation)
    cap = R.RunnerCapture(2, tk, C1.WINDOW, C1.LOCAL)
    try:
        inp = C1.prompt().cuda()
        with torch.no_grad():
            for step in range(C1.STEPS):
                model(input_ids=inp, past_key_values=cache, use_cache=True, return_dict=True)
                cap.step(cache)
                if step + 1 < C1.STEPS:
                    inp = torch.tensor([[int(tokens[step])]], device="cuda")
    finally:
        handles.remove()
    assert cap.evicted == evicted_ref
    for t, (got, want) in enumerate(zip(cap.steps, steps_ref)):
        for li in range(2):
            msg = f"step {t} layer {li}"
            np.testing.assert_array_equal(got["ids"][li], want["ids"][li], err_msg=msg)
            np.testing.assert_allclose(got["scores"][li], want["scores"][li], rtol=1e-5, atol=1e-6, err_msg=msg)
            np.testing.assert_array_equal(got["tk"][li], want["tk"][li], err_msg=msg)
            np.testing.assert_array_equal(got["ret_ids"][li], want["ret_ids"][li], err_msg=msg)
            # fp16 copies of scores equal within 1e-5 relative: at most one fp16 ulp apart
            np.testing.assert_allclose(got["ret_sc16"][li].astype(np.float32),
                                       want["ret_sc16"][li].astype(np.float32), rtol=2 ** -10, atol=0)
    ours = R.runner_arrays(cap.evicted, cap.steps, tokens, {"cache_backend_package": "b200"})
    ref = R.runner_arrays(evicted_ref, steps_ref, tokens, {"cache_backend_package": "eager"})
    np.savez_compressed(tmp_path / "parity_ours_b200.npz", **ours)
    for k in ("top_window_indices", "eviction_step_mask", "generated_tokens", "retained_window_ids"):
        np.testing.assert_array_equal(ours[k], ref[k], err_msg=k)
    for k in ("window_scores", "retained_window_scores"):
        assert ours[k].shape == ref[k].shape
        np.testing.assert_allclose(ours[k].astype(np.float32), ref[k].astype(np.float32), rtol=2 ** -10, atol=0)
