"""The YGG1 writer/reader and the generator (CPU only)."""
import numpy as np
import pytest

from yggdrasil_b200 import synth, ygg1


def test_header_round_trip(tmp_path):
    p = tmp_path / "m.bin"
    shape = synth.ModelShape(128, 16, 5, 27, 3, 16, 20, input_rank=8, group=True)
    synth.write_random_model(shape, p, seed=3)
    h = ygg1.read_header(p)
    assert (h["n_layers"], h["d_state"], h["block_size"], h["vocab"], h["router_depth"], h["readout_rank"],
            h["layer_input_rank"], h["input_rank"], h["shift"]) == (3, 128, 16, 27, 5, 16, 20, 8, 14)
    table, start = ygg1.array_table(p.read_bytes())
    assert start % 64 == 0 and "head_b" in table and "l2_vt" in table and "l1_r2b" in table
    assert all(off % 64 == 0 for off, _ in table.values())


def test_writer_enforces_limits(tmp_path):
    with pytest.raises(ValueError, match="d_state"):
        synth.write_random_model(synth.ModelShape(96, 16, 4, 5, 2, 8, 16), tmp_path / "m.bin")
    with pytest.raises(ValueError, match="readout_rank"):
        synth.write_random_model(synth.ModelShape(64, 16, 4, 5, 2, 12, 16), tmp_path / "m.bin")


def test_extension_d96(tmp_path):
    """d_state 96 with readout rank 12 is written only when asked; the readout then takes the rank-16 layout with zero
    rows 12-15 and the group scales stay 12 per expert."""
    shape = synth.ModelShape(96, 16, 4, 5, 3, 12, 24, group=True)
    assert shape.extended and not synth.WORKLOADS["c3"].extended and synth.WORKLOADS["c3n96"].extended
    p = tmp_path / "m.bin"
    layers = synth.write_random_model(shape, p, seed=2, extended=True)
    h = ygg1.read_header(p)
    assert (h["d_state"], h["readout_rank"], h["layer_input_rank"]) == (96, 12, 24)
    data = p.read_bytes()
    table, start = ygg1.array_table(data)
    meta = np.frombuffer(data, np.int32, 5, start + table["l1_meta"][0])
    rec = np.frombuffer(data, np.uint8, table["l1_rec"][1], start + table["l1_rec"][0]).reshape(2 ** 4, meta[0])
    ro = rec[:, meta[3]:meta[3] + 16 * 96].reshape(16, 96 // 4, 16, 4).astype(np.int64) - 128
    np.testing.assert_array_equal(ro[:, :, 12:], 0)
    np.testing.assert_array_equal(ro[:, :, :12].transpose(0, 2, 1, 3).reshape(16, 12, 96), layers[1].readout)
    assert table["l1_mzl"][1] == 4 * 16 * 12


def test_read_header_rejects_other_files(tmp_path):
    with pytest.raises(ValueError):
        ygg1.read_header(b"GGUF" + bytes(60))


def test_gathered_bytes_match_the_scope_table():
    # algorithmic bytes per token of the benchmark shapes (table storage), as tabulated for the roofline
    assert synth.gathered_bytes_per_token(synth.WORKLOADS["c1"].shape) == 8364
    assert synth.gathered_bytes_per_token(synth.WORKLOADS["c3"].shape) == 44084
    assert synth.gathered_bytes_per_token(synth.WORKLOADS["c4"].shape) == 45088


def test_dna_tokens_distribution():
    w = synth.WORKLOADS["c3"]
    x = synth.workload_tokens(w, 512, 512, seed=0)
    freq = np.bincount(x.ravel(), minlength=5) / x.size
    np.testing.assert_allclose(freq, synth.DNA_P, atol=3e-3)
