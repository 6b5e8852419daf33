"""CPU tests of the GGUF v3 reader (lc_gguf_*, host code of the library) against
files written by tests/gguf_writer.py, and the reference's gguf.rs unit tests
(src/gguf.rs:655-759)."""
import os

import numpy as np
import pytest

from gguf_writer import write_gguf
from laguna_raw_halo_strix_b200 import lc, synth
from laguna_raw_halo_strix_b200.model import Gguf


def test_type_sizes():
    L = lc.lib()
    # src/gguf.rs:659-708
    assert L.lc_type_block_elements(lc.F32) == 1 and L.lc_type_block_elements(lc.Q8_0) == 32
    assert L.lc_type_block_elements(lc.Q4_K) == 256
    assert [L.lc_type_block_bytes(t) for t in (lc.F32, lc.F16, lc.BF16, lc.Q8_0, lc.Q4_K)] == [4, 2, 2, 34, 144]
    # n_bytes cases (src/gguf.rs:696-732)
    assert L.lc_tensor_bytes(lc.BF16, 100 * 200) == 40000
    assert L.lc_tensor_bytes(lc.F32, 100 * 200) == 80000
    assert L.lc_tensor_bytes(lc.Q8_0, 1024) == 1088
    assert L.lc_tensor_bytes(lc.Q4_K, 256 * 10 * 3) == 30 * 144
    assert L.lc_type_block_bytes(6) == 0  # unsupported


def test_roundtrip(tmp_path):
    rng = np.random.default_rng(0)
    w4 = synth.q4k_blocks(8, 512, rng)
    w8 = synth.q8_0_blocks(3, 64, rng)
    nf = rng.standard_normal(37).astype(np.float32)
    meta = {"general.architecture": "dflash", "dflash.block_count": 2, "dflash.embedding_length": 512,
            "dflash.feed_forward_length": 768, "dflash.attention.head_count": 4,
            "dflash.attention.head_count_kv": 2, "dflash.attention.key_length": 128,
            "dflash.rope.dimension_count": 128, "dflash.rope.freq_base": 10000.0,
            "dflash.target_layers": [1, 5, 9]}
    path = str(tmp_path / "m.gguf")
    write_gguf(path, meta, [("a.weight", lc.Q4_K, (512, 8), w4), ("b.weight", lc.Q8_0, (64, 3), w8),
                            ("blk.0.attn_norm.weight", lc.F32, (37,), nf)])
    g = Gguf(path)
    ts = g.tensors()
    assert [t["name"] for t in ts] == ["a.weight", "b.weight", "blk.0.attn_norm.weight"]
    assert ts[0]["dtype"] == lc.Q4_K and ts[0]["shape"] == (512, 8) and ts[0]["n_bytes"] == w4.nbytes
    assert ts[1]["n_bytes"] == 3 * 68
    assert all(t["offset"] % 32 == 0 for t in ts)
    assert np.array_equal(g.read("a.weight"), w4.ravel())
    assert np.array_equal(g.read("b.weight"), w8.ravel())
    assert np.array_equal(g.read("blk.0.attn_norm.weight").view(np.float32), nf)
    assert g.meta_str("general.architecture") == "dflash"
    assert g.meta_u64("dflash.block_count") == 2
    assert g.meta_f32("dflash.rope.freq_base") == 10000.0
    hp = g.hparams()
    assert (hp.n_layers, hp.n_embd, hp.n_ff, hp.n_heads, hp.n_kv_heads, hp.head_dim, hp.rope_dim, hp.n_aux) == \
        (2, 512, 768, 4, 2, 128, 128, 3)
    assert hp.rope_base == 10000.0 and hp.norm_eps == pytest.approx(1e-5) and hp.qk_eps == pytest.approx(1e-6)
    with pytest.raises(lc.LagunaError):
        g.read("missing.weight")
    g.close()


def test_hparam_aliases_and_arrays(tmp_path):
    # laguna.* keys, head_count given as arrays (first / second element,
    # src/gguf.rs:540-560), no key_length (-> n_embd / n_heads), default base
    path = str(tmp_path / "a.gguf")
    meta = {"laguna.block_count": 3, "laguna.embedding_length": 256, "laguna.attention.head_count": [2, 9],
            "laguna.attention.head_count_kv": [7, 1], "feed_forward_length": 512}
    write_gguf(path, meta, [])
    hp = Gguf(path).hparams()
    assert (hp.n_layers, hp.n_embd, hp.n_heads, hp.n_kv_heads, hp.head_dim, hp.n_ff) == (3, 256, 2, 1, 128, 512)
    assert hp.rope_base == 500000.0 and hp.n_aux == 0


def test_rejects_bad_files(tmp_path):
    p = tmp_path / "bad.gguf"
    p.write_bytes(b"NOPE" + bytes(20))
    with pytest.raises(lc.LagunaError) as e:
        Gguf(str(p))
    assert e.value.status == lc.LC_ERR_IO
    p.write_bytes(b"GGUF" + (2).to_bytes(4, "little") + bytes(16))
    with pytest.raises(lc.LagunaError):
        Gguf(str(p))  # only v3 (src/gguf.rs:330-336)
    with pytest.raises(lc.LagunaError):
        Gguf(str(tmp_path / "missing.gguf"))
    good = str(tmp_path / "t.gguf")
    write_gguf(good, {"block_count": 1}, [("x", lc.F32, (4,), np.zeros(4, np.float32))])
    raw = open(good, "rb").read()
    trunc = tmp_path / "trunc.gguf"
    trunc.write_bytes(raw[:30])
    with pytest.raises(lc.LagunaError):
        Gguf(str(trunc))
    os.remove(str(trunc))


def test_mapped_view_matches_read(tmp_path):
    """lc_gguf_tensor_data hands out the tensor bytes from the file mapping:
    the same bytes lc_gguf_read copies, at 32-byte aligned file offsets."""
    rng = np.random.default_rng(4)
    w4 = synth.q4k_blocks(16, 1024, rng)
    b16 = rng.integers(0, 1 << 16, size=333, dtype=np.uint16)
    path = str(tmp_path / "v.gguf")
    write_gguf(path, {"block_count": 1}, [("q.weight", lc.Q4_K, (1024, 16), w4), ("h.weight", lc.BF16, (333,), b16),
                                          ("e.weight", lc.F32, (0,), np.zeros(0, np.float32))])
    g = Gguf(path)
    for name in ("q.weight", "h.weight", "e.weight"):
        v = g.view(name)
        assert not v.flags.writeable
        assert np.array_equal(v, g.read(name)), name
    assert np.array_equal(g.view("h.weight").view(np.uint16), b16)
    g.close()


def test_tensor_past_end_of_file(tmp_path):
    """A file cut inside its data section opens (the header is whole), and
    reading a tensor that lies past the end is LC_ERR_IO -- read_exact's short
    read in GGUFReader::read_tensor_data (src/gguf.rs:415-421)."""
    rng = np.random.default_rng(5)
    a = rng.standard_normal(64).astype(np.float32)
    b = rng.standard_normal(4096).astype(np.float32)
    good = str(tmp_path / "g.gguf")
    write_gguf(good, {"block_count": 1}, [("a.weight", lc.F32, (64,), a), ("b.weight", lc.F32, (4096,), b)])
    raw = open(good, "rb").read()
    cut = tmp_path / "cut.gguf"
    cut.write_bytes(raw[:-100])
    g = Gguf(str(cut))
    assert np.array_equal(g.read("a.weight").view(np.float32), a)
    for fn in (g.read, g.view):
        with pytest.raises(lc.LagunaError) as e:
            fn("b.weight")
        assert e.value.status == lc.LC_ERR_IO
    g.close()
