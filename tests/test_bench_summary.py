"""bench.py's training summary on a synthetic kernel-timer report (host only): per-kernel
HBM fractions, the roofline object on the largest kernel with an HBM byte model, and the
sort's share of the step."""
import pytest

from gsplat_tt_b200 import train_bench as tb

PEAKS = {"hbm_gbs": 6541.5, "source": "measured"}


def test_summary_picks_largest_hbm_kernel_and_scales_traffic():
    n, views, pairs, px = 6_000_000, 32, 46_000_000.0, 1920 * 1080
    ksteps = 2
    rep = {  # name: (total ms over ksteps steps, launches)
        "train_project": (12.4, 2),
        "radix_pass32": (14.8, 256),
        "tile_sort_emit": (16.0, 64),
        "tile_sort_pass": (8.8, 64),
        "tile_filter": (6.0, 64),
        "raster_fwd": (33.2, 64),
        "raster_bwd": (74.2, 64),
        "loss": (11.7, 64),
        "param_bwd": (11.7, 2),
        "sparse_adam": (3.4, 2),
    }
    per_kernel, roof, sort = tb.summarize_kernels(rep, ksteps, n, views, pairs, px, PEAKS)
    assert roof["kernel"] == "radix_pass32"            # raster_bwd is larger but issue-bound
    assert "achieved_gbs" not in per_kernel["raster_bwd"]
    assert "achieved_gbs" not in per_kernel["tile_sort_emit"]   # per super-tile item bytes
    e = per_kernel["radix_pass32"]
    assert e["ms_per_step"] == pytest.approx(7.4)
    assert e["algorithmic_bytes"] == pytest.approx(n * 16)
    assert roof["achieved"] == pytest.approx(e["algorithmic_bytes"] / (14.8 / 256 / 1e3) / 1e9)
    assert roof["frac"] == pytest.approx(roof["achieved"] / 6541.5)
    assert roof["traffic"] is None
    assert "raster_bwd 37.1 ms" in roof["note"]
    assert per_kernel["tile_filter"]["algorithmic_bytes"] == pytest.approx(pairs * 4)
    assert sort["ms_per_step"] == pytest.approx((14.8 + 16.0 + 8.8 + 6.0) / 2)
    assert per_kernel["train_project"]["algorithmic_bytes"] == pytest.approx(n * 236 + views * n * 48)


def test_summary_without_traffic_entry():
    rep = {"sparse_adam": (2.0, 1), "raster_bwd": (30.0, 1)}
    per_kernel, roof, sort = tb.summarize_kernels(rep, 1, 1000, 1, 5000.0, 100, PEAKS)
    assert roof["kernel"] == "sparse_adam" and roof["traffic"] is None and sort is None


def test_chunked_and_owner_sharded_launches_are_charged_their_own_rows():
    """At N > 1 the projection backward runs once per row chunk and the multicast update
    moves link bytes, not HBM bytes: no kernel may read above the peak."""
    n, views, world, q, chunks = 6_000_000, 4, 8, 187_500, 4
    rep = {"param_bwd": (2.41 * 2, 4 * 2), "sparse_adam_mc": (3.28 * 2, 4 * 2),
           "tile_filter": (2.0, 8), "train_project": (1.6 * 2, 4 * 2)}
    per_kernel, roof, _ = tb.summarize_kernels(rep, 2, n, views, 4.6e7, 1920 * 1080, PEAKS,
                                               adam_rows=chunks * q, world=world, q=q)
    pb = per_kernel["param_bwd"]
    assert pb["algorithmic_bytes"] == pytest.approx((n * 472.0 + views * n * 36.0) / 4)
    assert pb["frac_hbm"] < 1.0
    # the next step's projection, one launch per row chunk behind the update
    tp = per_kernel["train_project"]
    assert tp["algorithmic_bytes"] == pytest.approx((n * 236.0 + views * n * 48.0) / 4)
    assert tp["frac_hbm"] < 1.0
    mc = per_kernel["sparse_adam_mc"]
    assert "frac_hbm" not in mc
    assert mc["link_bytes_per_direction"] == pytest.approx(q * (world * 240 + 236))
    assert mc["frac_nvlink"] == pytest.approx(mc["achieved_link_gbs"] / tb.NVLINK_GBS)
    assert roof["kernel"] in ("param_bwd", "tile_filter")
    # NCCL owner-sharded update: the rank's own rows
    per_kernel, _, _ = tb.summarize_kernels({"sparse_adam": (1.0, 1)}, 1, n, views, 1.0, 1,
                                            PEAKS, adam_rows=n // world, world=world)
    assert per_kernel["sparse_adam"]["algorithmic_bytes"] == pytest.approx(n // world * 59 * 28)


def test_sort_byte_model_counts_the_narrowed_passes():
    """The sort line's own-bytes model: six passes for 45 key bits, the first on 64-bit
    keys, the second writing keys narrowed to 32 bits, three on 32-bit keys, the last
    writing values only; up to 32 key bits every pass moves 64-bit keys."""
    import bench
    assert bench.sort_pass_bytes(45) == [24, 20, 16, 16, 16, 12]
    assert bench.sort_pass_bytes(64) == [24, 24, 24, 20, 16, 16, 16, 12]
    assert bench.sort_pass_bytes(33) == [20, 16, 16, 16, 12]
    assert bench.sort_pass_bytes(32) == [24, 24, 24, 16]
    per_launch, per_sort = bench.sort_algorithmic_bytes(1 << 24, 45)
    assert per_sort == (104 + 8) * (1 << 24)
    assert per_launch == 104 * (1 << 24) / 6
    assert bench.SORT_PASS_BYTES_PER_PAIR * 6 + 8 == 152
