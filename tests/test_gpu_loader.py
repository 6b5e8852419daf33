"""GPU tests of the GGUF loader fast path (lc_dflash_load_gguf_ex): the file is
mapped, every tensor the draft path uses is staged through pinned buffers into
one device image, and F16 / BF16 tensors are decoded to f32 on the device.
The reference's loader is DFlashModel::load (src/dflash.rs:34-119) over
GGUFReader::read_tensor_data (src/gguf.rs:415-421)."""
import time

import numpy as np
import pytest

import oracle as orc
from conftest import to_dev
from dflash_oracle import DFlashOracle, make_model, tensor_shape
from gguf_writer import write_gguf
from laguna_raw_halo_strix_b200 import lc, synth
from laguna_raw_halo_strix_b200.model import DFlash, hparams

pytestmark = pytest.mark.gpu

HP = dict(n_layers=2, n_embd=512, n_heads=4, n_kv_heads=2, head_dim=128, rope_dim=128, n_ff=768, n_aux=2,
          rope_base=500000.0, norm_eps=1e-5, qk_eps=1e-6)


def rel_l2(a, b):
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def meta(hp):
    return {"general.architecture": "dflash", "dflash.block_count": hp["n_layers"],
            "dflash.embedding_length": hp["n_embd"], "dflash.feed_forward_length": hp["n_ff"],
            "dflash.attention.head_count": hp["n_heads"], "dflash.attention.head_count_kv": hp["n_kv_heads"],
            "dflash.attention.key_length": hp["head_dim"], "dflash.rope.dimension_count": hp["rope_dim"],
            "dflash.rope.freq_base": hp["rope_base"], "dflash.target_layers": list(range(hp["n_aux"]))}


def d2h(addr, n):
    from cuda.bindings import runtime as rt

    out = np.empty(n, np.uint8)
    (err,) = rt.cudaMemcpy(out.ctypes.data, addr, n, rt.cudaMemcpyKind.cudaMemcpyDeviceToHost)
    assert int(err) == 0, err
    return out


def write_model(path, t, hp, extra=()):
    tensors = [(name, dt, tensor_shape(name, hp), np.ascontiguousarray(a).view(np.uint8)) for name, (dt, a) in t.items()]
    write_gguf(path, meta(hp), tensors + list(extra))


def test_every_slot_and_type(ctx, oracle, tmp_path):
    """Raw Q4_K / Q8_0 / F32 blocks arrive byte for byte; F16 and BF16 norm
    weights are decoded with dequant_to_f32's rules (BF16 read with the f16
    layout, src/dflash.rs:351-378), or as bfloat16 with LC_LOAD_BF16_NATIVE;
    tensors the draft path does not use are skipped."""
    rng = np.random.default_rng(11)
    t = make_model(HP, orc.Q4_K, rng)
    t["blk.0.ffn_up.weight"] = (orc.Q8_0, synth.q8_0_blocks(HP["n_ff"], HP["n_embd"], rng).reshape(-1))  # mixed
    E = HP["n_embd"]
    f16 = rng.standard_normal(E).astype(np.float16)
    f16[:4] = [np.inf, -np.inf, 6e-8, -0.0]
    bf = rng.integers(0, 1 << 16, size=E, dtype=np.uint16)
    bf[:3] = [0x7F80, 0x7FC1, 0x0001]  # inf, NaN, a subnormal in either reading
    t["blk.1.attn_norm.weight"] = (orc.F16, f16.view(np.uint16))
    t["output_norm.weight"] = (orc.BF16, bf)
    unused = ("rope_freqs.weight", orc.F32, (17,), np.arange(17, dtype=np.float32).view(np.uint8))
    path = str(tmp_path / "mixed.gguf")
    write_model(path, t, HP, extra=[unused])
    for flags in (0, lc.LOAD_BF16_NATIVE):
        m = DFlash(ctx, gguf_path=path, max_ctx=8, max_block=4, flags=flags)
        for name, (dt, a) in t.items():
            addr, sdt, nbytes = m.weight(name)
            raw = np.ascontiguousarray(a).view(np.uint8).ravel()
            assert addr % 256 == 0, name
            if dt in (orc.F16, orc.BF16):
                n = raw.size // 2
                assert (sdt, nbytes) == (lc.F32, 4 * n), name
                got = d2h(addr, nbytes).view(np.float32)
                if dt == orc.BF16 and flags:
                    want = (a.astype(np.uint32) << 16).view(np.float32)
                else:
                    want = oracle.dequant_to_f32(raw, dt, n)
                assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), (name, flags)
            else:
                assert (sdt, nbytes) == (dt, raw.size), name
                assert np.array_equal(d2h(addr, nbytes), raw), name
        with pytest.raises(lc.LagunaError):
            m.weight("rope_freqs.weight")
        m.close()
    with pytest.raises(lc.LagunaError):
        DFlash(ctx, gguf_path=path, max_ctx=8, max_block=4, flags=4)  # unknown flag


def test_image_across_staging_chunks(ctx, oracle, dev, tmp_path):
    """A model whose device image spans several 64 MB staging chunks (the ring
    of pinned buffers wraps) and a tensor that straddles chunk boundaries: the
    bytes still arrive exactly, and the loaded model decodes like one built
    tensor by tensor with lc_dflash_set_tensor (and like the oracle)."""
    import torch

    hp = dict(HP, n_embd=1024, n_ff=4096, n_heads=8, head_dim=128, n_kv_heads=2)
    rng = np.random.default_rng(12)
    t = make_model(hp, orc.Q8_0, rng)
    vocab = 60000  # token_embd F32: 1024 x 60000 x 4 B = 246 MB
    emb = (0.1 * rng.standard_normal(hp["n_embd"] * vocab)).astype(np.float32)
    path = str(tmp_path / "big.gguf")
    tensors = [("token_embd.weight", orc.F32, (hp["n_embd"], vocab), emb.view(np.uint8))]
    tensors += [(n, dt, tensor_shape(n, hp), np.ascontiguousarray(a).view(np.uint8)) for n, (dt, a) in t.items()]
    write_gguf(path, meta(hp), tensors)
    t0 = time.perf_counter()
    m = DFlash(ctx, gguf_path=path, max_ctx=16, max_block=4)
    load_s = time.perf_counter() - t0
    addr, dt, nbytes = m.weight("token_embd.weight")
    assert (dt, nbytes) == (lc.F32, emb.nbytes)
    assert np.array_equal(d2h(addr, nbytes).view(np.float32), emb)
    for name, (dt, a) in t.items():
        addr, _, nbytes = m.weight(name)
        assert np.array_equal(d2h(addr, nbytes), np.ascontiguousarray(a).view(np.uint8).ravel()), name
    # same decode as a model filled with lc_dflash_set_tensor
    ref = DFlash(ctx, hparams(**hp), max_ctx=16, max_block=4)
    for name, (dt, a) in t.items():
        ref.set_tensor(name, dt, np.ascontiguousarray(a).view(np.uint8))
    feats = to_dev((0.5 * rng.standard_normal((3, hp["n_aux"] * hp["n_embd"]))).astype(np.float32), dev)
    x = to_dev((0.5 * rng.standard_normal((4, hp["n_embd"]))).astype(np.float32), dev)
    outs = []
    for mm in (m, ref):
        enc = torch.empty(3, hp["n_embd"], device=dev)
        hid = torch.empty(4, hp["n_embd"], device=dev)
        mm.encode(feats, 3, enc)
        mm.set_context(enc, 3)
        mm.decode_block(x, 4, hid)
        torch.cuda.synchronize()
        outs.append(hid.cpu().numpy())
    # the split-k partial sums of the block projections are added in arrival
    # order, so two decodes agree to rounding, not bit for bit
    assert rel_l2(outs[0], outs[1]) <= 1e-4
    om = DFlashOracle(hp, t)
    want = om.decode_block(x.cpu().numpy(), om.context_kv(om.encode(feats.cpu().numpy())))
    assert rel_l2(outs[0], want) <= 2e-3
    m.close()
    ref.close()
    print(f"loaded {(emb.nbytes + sum(a.nbytes for _, a in t.values())) / 1e6:.0f} MB in {load_s * 1e3:.0f} ms")


def test_truncated_file_is_an_error(ctx, tmp_path):
    """A file cut inside the data section fails with LC_ERR_IO and leaves
    nothing allocated behind (the context still works)."""
    rng = np.random.default_rng(13)
    t = make_model(HP, orc.Q4_K, rng)
    path = str(tmp_path / "m.gguf")
    write_model(path, t, HP)
    raw = open(path, "rb").read()
    cut = tmp_path / "cut.gguf"
    cut.write_bytes(raw[:-4096])
    with pytest.raises(lc.LagunaError) as e:
        DFlash(ctx, gguf_path=str(cut), max_ctx=8, max_block=4)
    assert e.value.status == lc.LC_ERR_IO
    m = DFlash(ctx, gguf_path=path, max_ctx=8, max_block=4)
    m.close()
