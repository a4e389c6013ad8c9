"""The sm_100a tile table keeps the reference's lookup surface (autotune_configs.py:17-85:
PRESETS, get_preset(seq_len, arch), _detect_arch) and answers from measured entries."""
import pytest

from inkling_fa4 import autotune_configs as ac


def test_reference_keys_for_every_arch_and_length():
    for arch in (None, "sm86", "sm90", "sm100"):
        for n in (64, 4096, 32768, 1 << 20):
            cfg = ac.get_preset(n, arch)
            assert set(cfg) == {"BLOCK_Q", "BLOCK_K", "num_warps", "num_stages", "tile_config"}
            assert cfg["tile_config"] in ac.TILE_CONFIGS
    assert ac.get_preset(1)["BLOCK_Q"] == 1  # decode
    assert ac.get_config is ac.get_preset


def test_workload_entries_pick_their_measured_best_within_noise():
    for name, entry in ac.WORKLOAD_TABLE.items():
        tc = ac.get_preset(32768, workload=name)["tile_config"]
        assert tc == entry["tile_config"]
        best = max(entry["tflops"].values())
        chosen = entry["tflops"][tc]
        # within the run-to-run noise of two repetitions (up to about 5 % on the local-window
        # shape, whose tiles are all band tiles that no variant changes)
        assert chosen >= 0.95 * best, (name, tc, chosen, best)
    with pytest.raises(KeyError):
        ac.get_preset(32768, workload="no-such-workload")
