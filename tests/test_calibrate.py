"""The cap controller and cost-curve reading on the CPU (src/mlx_dspark/calibrate.py:157-297):
knee detection, interpolation, the acceptance EWMA, the rate-maximising cap with hysteresis,
the per-batch-width cap and the disk cache."""
import pytest

import importlib

cal = importlib.import_module("mlx_dspark_b200.calibrate")


def test_knee_width():
    # cheap marginal cost ~1 ms per row, then a jump at width 5
    convex = {2: 10.0, 3: 11.0, 4: 12.0, 5: 20.0, 6: 21.0}
    assert cal.knee_width(convex) == 5
    flat = {w: 3.0 + 0.01 * w for w in range(2, 10)}   # the B200 shape: no knee below 64 rows
    assert cal.knee_width(flat) == 9
    assert cal.knee_width({2: 1.0, 3: 2.0}) == 3
    rec = cal.drafter_recommendation(flat, dflash_block=16)
    assert rec == {"knee_width": 9, "dflash_full_block_viable": False, "recommend": "dspark"}
    assert cal.drafter_recommendation(flat, dflash_block=9)["recommend"] == "dflash-on-structured"


def test_interp():
    c = {2: 10.0, 4: 14.0, 8: 30.0}
    assert cal._interp(c, 2) == 10.0
    assert cal._interp(c, 3) == 12.0
    assert cal._interp(c, 6) == 22.0
    assert cal._interp(c, 1) == 10.0
    assert cal._interp(c, 10) == 38.0        # last segment's slope (4 ms per width)
    assert cal._interp({5: 7.0}, 9) == 7.0


def test_expected_committed_and_updates():
    ctl = cal.CapController({2: 1.0, 3: 1.0}, 0.5, max_cap=4, prior_p=0.5, alpha=0.1,
                            repick_every=1000)
    assert ctl.expected_committed(3) == pytest.approx(1 + 0.5 + 0.25 + 0.125)
    ctl.update(2, 3)          # two successes, then one failure
    p = 0.5
    p += 0.1 * (1 - p)
    p += 0.1 * (1 - p)
    p -= 0.1 * p
    assert ctl.p == pytest.approx(p)
    ctl.update(3, 3)          # a fully accepted block: successes only (censored)
    for _ in range(3):
        p += 0.1 * (1 - p)
    assert ctl.p == pytest.approx(p) and ctl.rounds == 2


def test_flat_curve_picks_full_block():
    """A flat verify curve (every width streams the same weights) makes the whole block the
    best cap at the prior acceptance, so the controller moves there from its initial cap 2."""
    verify = {w: 3.9 for w in range(2, 10)}
    drafter = {c: 0.40 + 0.02 * c for c in range(1, 9)}
    ctl = cal.CapController(verify, drafter, max_cap=8, init_cap=2, repick_every=4)
    assert max(range(1, 9), key=ctl.rate) == 8
    for _ in range(4):
        ctl.update(5, ctl.cap)
    assert ctl.cap == 8
    # a steep curve (convex knee at 3) keeps short caps
    steep = {2: 5.0, 3: 10.0, 4: 30.0, 5: 50.0, 6: 70.0, 7: 90.0, 8: 110.0, 9: 130.0}
    ctl2 = cal.CapController(steep, 0.5, max_cap=8, init_cap=8, repick_every=1)
    ctl2.update(1, 8)
    assert ctl2.cap == 1


def test_hysteresis_keeps_near_ties():
    verify = {w: 10.0 for w in range(2, 6)}
    # cap 2 vs 3 differ by under 3 % in rate at p = 0.05
    ctl = cal.CapController(verify, {1: 0.0, 2: 0.0, 3: 0.0, 4: 0.0}, max_cap=4, init_cap=2,
                            prior_p=0.05, repick_every=1, alpha=0.0)
    r2, r3 = ctl.rate(2), ctl.rate(3)
    assert r3 > r2 and r3 < 1.03 * r2
    ctl.update(0, 2)
    assert ctl.cap == 2


def test_cap_for_batch_grid():
    verify = {w: 4.0 for w in range(2, 10)}
    grid = {4: {2: 4.0, 3: 4.1, 4: 9.0, 5: 14.0, 6: 19.0, 7: 24.0, 8: 29.0, 9: 34.0}}
    ctl = cal.CapController(verify, 0.3, max_cap=8, init_cap=8, verify_grid=grid)
    assert ctl.cap_for(1) == 8
    assert ctl.cap_for(3) == ctl.cap_for(4) == 2     # nearest measured B >= width
    assert ctl.cap_for(16) == 2                      # past the grid: its largest B
    info = ctl.info()
    assert info["batch_caps"] == {4: 2} and set(info["predicted_rates"]) == set(range(1, 9))


def test_disk_cache_round_trip(tmp_path):
    key = cal.cache_key("dspark", "/models/Qwen3-8B-8bit/", "x/dspark-qwen3", 512, 8,
                        device_name="NVIDIA B200")
    assert "|dspark|Qwen3-8B-8bit|dspark-qwen3|ctx512|kv8" in key and "NVIDIA B200" in key
    assert cal.load_cached(key, str(tmp_path)) is None
    entry = {"verify": {"2": 3.5}, "drafter": {"1": 0.4}}
    cal.save_cached(key, entry, str(tmp_path))
    cal.save_cached("other", {"verify": {}}, str(tmp_path))
    assert cal.load_cached(key, str(tmp_path)) == entry
    (tmp_path / cal.CACHE_FILE).write_text("{not json")
    assert cal.load_cached(key, str(tmp_path)) is None     # a corrupt file reads as empty
