"""CPU tests of the target-model side: the GGUF hyper-parameter reader
(lc_gguf_target_hparams, host code of the library) against Model::from_reader's
rules (src/model.rs:29-129), and the oracle's restatement of the router
(src/target.rs:653-677) and of forward_token_impl (src/target.rs:314-578)."""
import numpy as np
import pytest

import oracle as orc
import target_oracle as T
from gguf_writer import write_gguf
from laguna_raw_halo_strix_b200 import lc
from laguna_raw_halo_strix_b200.target import target_hparams


def test_hparams_from_metadata(tmp_path):
    hp = T.default_hp()
    t = T.make_target(hp, orc.Q8_0, np.random.default_rng(0))
    path = str(tmp_path / "t.gguf")
    write_gguf(path, T.gguf_meta(hp), T.gguf_tensors(t, hp))
    got = target_hparams(path)
    for k in ("n_layers", "n_embd", "n_ff", "n_heads", "n_kv_heads", "head_dim", "rope_dim", "rope_dim_swa",
              "n_expert", "n_expert_used", "n_ff_exp", "n_ff_shexp", "n_vocab"):
        assert getattr(got, k) == hp[k], k
    assert got.swa == 1 and got.has_moe == 1 and got.has_shexp == 1 and got.expert_weights_norm == 1
    assert got.expert_weights_scale == pytest.approx(2.5) and got.rope_base_swa == pytest.approx(10000.0)
    assert got.norm_eps == pytest.approx(1e-5) and got.qk_eps == pytest.approx(1e-6)


def test_hparams_fallbacks_from_shapes(tmp_path):
    """No expert.* keys: expert width from ffn_gate_exps / ffn_gate_shexp dim 1,
    the expert count from the stack's last dim and 10 experts used
    (src/model.rs:43-107); sliding_window alone switches SWA on; head_dim has
    no fallback; a u8 value is not an integer to the reader (as_u64 takes
    U32/U64/I32/I64 only, src/gguf.rs:228-237)."""
    import struct

    hp = T.default_hp(n_layers=2, n_expert=12, n_ff_exp=128, n_ff_shexp=128, rope_dim_swa=0)
    t = T.make_target(hp, orc.Q8_0, np.random.default_rng(1))
    meta = {k: v for k, v in T.gguf_meta(hp).items() if not k.startswith("expert.") and "swa" not in k}
    meta["laguna.attention.sliding_window"] = 4096
    del meta["laguna.attention.key_length"]
    path = str(tmp_path / "f.gguf")
    write_gguf(path, meta, T.gguf_tensors(t, hp))
    got = target_hparams(path)
    assert (got.n_expert, got.n_expert_used, got.n_ff_exp, got.n_ff_shexp) == (12, 10, 128, 128)
    assert got.swa == 1 and got.rope_dim_swa == 0 and got.head_dim == 0
    # a block_count stored as u8 reads as absent
    raw = bytearray(open(path, "rb").read())
    key = b"laguna.block_count"
    i = raw.index(struct.pack("<Q", len(key)) + key) + 8 + len(key)
    assert struct.unpack_from("<I", raw, i)[0] == 4  # GGUF u32
    struct.pack_into("<I", raw, i, 0)  # -> u8 (type 0) whose byte is the old u32's low byte
    bad = tmp_path / "u8.gguf"
    bad.write_bytes(bytes(raw[:i + 5]) + bytes(raw[i + 8:]))
    assert target_hparams(str(bad)).n_layers == 0


def test_router_selection_rules():
    o = orc.Oracle()
    # equal selections keep expert order (stable sort); bias shifts the choice
    logits = np.zeros(6, np.float32)
    bias = np.array([0, 0.1, 0.1, 0, 0.1, 0], np.float32)
    ids, sc = o.moe_select(logits, bias, 4)
    assert list(ids) == [1, 2, 4, 0]
    assert np.all(sc == np.float32(0.5))
    # normalisation by the sum in slot order, then the scale
    ids, sc = o.moe_select(logits, bias, 4, norm=True, scale=2.0)
    assert np.allclose(sc, 0.5, atol=0) and sc.dtype == np.float32
    # more used than experts: all of them
    ids, _ = o.moe_select(np.array([3.0, -1.0, 2.0], np.float32), np.zeros(3, np.float32), 10)
    assert list(ids) == [0, 2, 1]
    # the floor of the normaliser (2^-14) for vanishing probabilities
    ids, sc = o.moe_select(np.full(4, -200.0, np.float32), np.arange(4, dtype=np.float32), 2, norm=True)
    assert list(ids) == [3, 2] and np.all(sc == 0.0)


def test_l2_rescale():
    o = orc.Oracle()
    h = np.array([3.0, 4.0], np.float32)
    hs, col = o.moe_l2_scale(h)
    assert col == np.float32(5.0) and np.array_equal(hs, np.array([3 * 32768 / 5, 4 * 32768 / 5], np.float32))
    hs, col = o.moe_l2_scale(np.zeros(3, np.float32))
    assert col == np.float32(1e-8) and np.all(hs == 0)


@pytest.mark.parametrize("wtype", [orc.Q4_K, orc.Q8_0])
def test_first_cached_token_is_forward_token(wtype):
    """With an empty cache, forward_token_cached attends to its own key only,
    at position 0 -- forward_token's computation; the next cached token
    differs (it attends to two positions at position 1)."""
    hp = T.default_hp(n_layers=2, n_embd=256, n_ff=512, n_vocab=300, q_heads={}, gate_layers=(1,))
    rng = np.random.default_rng(2)
    t = T.make_target(hp, wtype, rng)
    om = T.TargetOracle(hp, t)
    x = rng.standard_normal((2, hp["n_embd"])).astype(np.float32)
    c0, h0, l0 = om.forward(x[:1], capture=(0, 1, 2))
    c1, h1, l1 = om.forward(x[:1], capture=(0, 1, 2), cached=True)
    assert np.array_equal(h0, h1) and np.array_equal(l0, l1) and np.array_equal(c0, c1)
    assert c0.shape == (1, 3, hp["n_embd"]) and np.array_equal(c0[0, 0], x[0])
    _, h2, _ = om.forward(x[1:], cached=True)
    _, h3, _ = T.TargetOracle(hp, t).forward(x[1:])
    assert not np.array_equal(h2, h3)
    assert om.cache_len == 2
    om.truncate(1)
    assert om.cache_len == 1 and len(om.cache_k[0]) == 1


def test_expert_offset_quirk_in_oracle():
    """ref_expert_offset reads expert 0 for every Q8_0 expert; Q4_K experts
    are offset either way (src/target.rs:1098-1162)."""
    hp = T.default_hp(n_layers=2, n_embd=256, n_ff=512, n_vocab=300, q_heads={}, gate_layers=())
    for et, differs in ((orc.Q8_0, True), (orc.Q4_K, False)):
        rng = np.random.default_rng(3)
        t = T.make_target(hp, orc.Q8_0, rng, expert_type=et)
        nx = rng.standard_normal(hp["n_embd"]).astype(np.float32)
        a, ids, _ = T.TargetOracle(hp, t).moe_ffn(1, nx)
        b, ids_b, _ = T.TargetOracle(hp, t, ref_expert_offset=True).moe_ffn(1, nx)
        assert np.array_equal(ids, ids_b) and 0 not in ids[:1]
        assert (not np.array_equal(a, b)) == differs
