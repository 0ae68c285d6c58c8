"""bench.py's roofline arithmetic on the CPU: visible and distinct KV positions of the scheduled
steps (one position per slot, or prompt chunks under an item budget), the dominant class, the
committed steady-state traffic attached only to the configuration it was captured in, and the
latency bound of k_layer."""
import bench


def test_visible_positions_one_position_per_slot():
    slots = [(0, 10, 1), (1, 300, 1), (2, 5, 0)]  # (sequence, position, busy)
    prompts = [list(range(40)), list(range(500)), list(range(7))]
    visible, distinct = bench.visible_positions(slots, prompts, 0, 0, 2)
    # step 1: positions 10 and 300 see 11 and 256; step 2: 12 and 256
    assert visible == distinct == (11 + 256 + 12 + 256) / 2


def test_visible_positions_with_chunks():
    slots = [(0, 10, 1), (1, 300, 1), (2, 5, 1)]
    prompts = [list(range(40)), list(range(500)), list(range(7))]
    visible, distinct = bench.visible_positions(slots, prompts, 8, 6, 2)
    # budget 6 - 3 = 3 extra items per step: slot 0 takes 4 positions, the others one each
    step1 = (11 + 12 + 13 + 14) + 256 + 6
    step2 = (15 + 16 + 17 + 18) + 256 + 7
    assert visible == (step1 + step2) / 2
    assert distinct == ((14 + 256 + 6) + (18 + 256 + 7)) / 2


def test_roofline_traffic_and_bounds():
    peaks = {"hbm_gbs": 6554.9}
    prof = {"attention": (19.0, 270), "layer": (14.0, 280), "gemv_qkvg": (18.0, 270)}  # 10 profiled steps
    line = bench.roofline_for(prof, 380, peaks, visible=77000, unique=60000, sm_mhz=1965.0, state_chunk=8)
    assert line["kernel"] == "attention" and line["traffic"] == bench.STEADY_TRAFFIC["attention"]["bytes"]
    assert line["algorithmic_bytes_per_launch"] == 4 * 60000 * 136 + 380 * (1536 * 4 + 512 * 4)
    assert 0 < line["fp64"]["frac"] < 1
    # another chunk setting, or no config-4 state: the capture does not apply
    assert bench.roofline_for(prof, 380, peaks, visible=77000, unique=60000, state_chunk=12)["traffic"] is None
    assert bench.roofline_for(prof, 380, peaks)["traffic"] is None
    layer = bench.roofline_for({"layer": (20.0, 280)}, 380, peaks, sm_mhz=1965.0, state_chunk=8)
    assert layer["latency"]["chain_adds_per_item"] == 512 + 512 + 2048 + 512
    assert abs(layer["latency"]["floor_ms"] - 3584 * 11 / 1965e3) < 1e-5  # rounded to 5 decimals
