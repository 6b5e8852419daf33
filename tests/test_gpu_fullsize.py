"""GPU parity at BASELINE.json's full sizes for the decoder and the lm_head:

* config 3: the 6-layer DFlash decoder (hidden 4096, 32 Q / 8 KV heads of 128,
  FFN 14336, Q4_K projections) for one 16-token block over 2048 context rows
  of encoder output -- hidden states within rel-L2 <= 2e-3 of the oracle's,
  then projected through a 128256-row Q8_0 lm_head: the draft tokens must be
  identical to the oracle chain's (src/dflash.rs:877-976, src/target.rs:580-605,
  src/lib.rs:456-464);
* config 4: the 128256 x 4096 Q8_0 lm_head for 1024 rows (the tcgen05 tiles)
  -- tokens of a sample of rows identical, logits of 40 rows within
  1e-3 * ||logits||_inf.

The oracle's projections here dequantise the weights bit-exactly with the
shader formula and sum with f32 BLAS (oracle/dflash_oracle.py proj_blas), which runs
these sizes in seconds; every other op is the C restatement.  A mismatching
token is reported with its top-2 logit margin.
"""
import numpy as np
import pytest

import oracle as orc
from conftest import to_dev
from dflash_oracle import DFlashOracle, proj_blas
from laguna_raw_halo_strix_b200 import lc, synth
from laguna_raw_halo_strix_b200.model import DFlash, hparams

pytestmark = pytest.mark.gpu

HP3 = dict(n_layers=6, n_embd=4096, n_heads=32, n_kv_heads=8, head_dim=128, rope_dim=128, n_ff=14336, n_aux=5,
           rope_base=500000.0, norm_eps=1e-5, qk_eps=1e-6)
CTX, BLOCK, VOCAB = 2048, 16, 128256


def rel_l2(a, b):
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def oracle_tokens(o, logits):
    """argmax per row with the reference's rule (last maximum wins)."""
    return np.array([o.argmax(r) for r in logits], np.int64)


def margins(logits, rows):
    out = []
    for r in rows:
        s = np.sort(np.asarray(logits[r], np.float64))
        out.append(float(s[-1] - s[-2]))
    return out


def gpu_tokens(ctx, dev, hidden, w, m, k, vocab):
    import torch

    keys = torch.empty(m, dtype=torch.int64, device=dev)
    ctx.lm_head_argmax(lc.Q8_0, to_dev(np.ascontiguousarray(hidden, np.float32), dev), w, m, k, vocab, 0, keys)
    torch.cuda.synchronize()
    return np.array([lc.key_index(int(v)) for v in keys.cpu().numpy().view(np.uint64)], np.int64)


@pytest.fixture(scope="module")
def lm_head_w():
    return synth.q8_0_blocks(VOCAB, HP3["n_embd"], np.random.default_rng(44))


@pytest.fixture(scope="module")
def config3(ctx, dev):
    import torch

    rng = np.random.default_rng(3)
    tensors = synth.dflash_tensors(HP3, lc.Q4_K, rng)  # distinct weights in every layer
    gm = DFlash(ctx, hparams(**HP3), max_ctx=CTX, max_block=BLOCK)
    for name, (dt, a) in tensors.items():
        gm.set_tensor(name, dt, a)
    E, A = HP3["n_embd"], HP3["n_aux"]
    feats = rng.standard_normal((CTX, A * E)).astype(np.float32)
    toks = rng.standard_normal((BLOCK, E)).astype(np.float32)
    enc = torch.empty(CTX, E, device=dev)
    hid = torch.empty(BLOCK, E, device=dev)
    gm.encode(to_dev(feats, dev), CTX, enc)
    gm.set_context(enc, CTX)
    gm.decode_block(to_dev(toks, dev), BLOCK, hid)
    torch.cuda.synchronize()
    enc_g, hid_g = enc.cpu().numpy(), hid.cpu().numpy()
    gm.close()
    om = DFlashOracle(HP3, tensors, fast_proj=True)
    enc_r = om.encode(feats)
    hid_r = om.decode_block(toks, om.context_kv(enc_r))
    return enc_g, hid_g, enc_r, hid_r, om


def test_config3_encoder_and_hidden(config3):
    enc_g, hid_g, enc_r, hid_r, _ = config3
    assert rel_l2(enc_g, enc_r) <= 2e-3, rel_l2(enc_g, enc_r)
    for r in range(BLOCK):
        e = rel_l2(hid_g[r], hid_r[r])
        assert e <= 2e-3, f"block token {r}: rel-L2 {e:.3e}"
    print(f"config 3: encoder rel-L2 {rel_l2(enc_g, enc_r):.2e}, hidden rel-L2 {rel_l2(hid_g, hid_r):.2e}")


def test_config3_draft_tokens(config3, lm_head_w, ctx, dev):
    """Decoder -> lm_head -> argmax on the GPU against the oracle's chain."""
    _, hid_g, _, hid_r, om = config3
    E = HP3["n_embd"]
    w = to_dev(lm_head_w, dev)
    got = gpu_tokens(ctx, dev, hid_g, w, BLOCK, E, VOCAB)
    logits_r = proj_blas(om.o, orc.Q8_0, hid_r, lm_head_w, E, VOCAB)
    ref = oracle_tokens(om.o, logits_r)
    bad = np.nonzero(got != ref)[0]
    print(f"config 3 draft tokens: {BLOCK - bad.size}/{BLOCK} identical; top-2 margins min "
          f"{min(margins(logits_r, range(BLOCK))):.3e}")
    assert bad.size == 0, f"rows {bad.tolist()} differ; top-2 margins {margins(logits_r, bad)}"


def test_config4_lm_head_full(lm_head_w, ctx, dev, oracle):
    """1024 rows through the tcgen05 lm_head tiles: sampled rows' tokens and
    40 rows' logits against the oracle."""
    import torch

    rng = np.random.default_rng(4)
    m, k = 1024, HP3["n_embd"]
    x = synth.activations(m, k, rng)
    w = to_dev(lm_head_w, dev)
    got = gpu_tokens(ctx, dev, x, w, m, k, VOCAB)
    sample = np.sort(rng.choice(m, 24, replace=False))
    logits_r = proj_blas(oracle, orc.Q8_0, x[sample], lm_head_w, k, VOCAB)
    ref = oracle_tokens(oracle, logits_r)
    bad = np.nonzero(got[sample] != ref)[0]
    assert bad.size == 0, f"sampled rows {sample[bad].tolist()} differ; top-2 margins {margins(logits_r, bad)}"
    # logits of 40 rows (more than 32: the lm_head tiles) with the argmax
    m2 = 40
    keys = torch.empty(m2, dtype=torch.int64, device=dev)
    logits = torch.empty(m2, VOCAB, device=dev)
    ctx.lm_head_argmax(lc.Q8_0, to_dev(x[:m2], dev), w, m2, k, VOCAB, 0, keys, logits)
    torch.cuda.synchronize()
    lr = proj_blas(oracle, orc.Q8_0, x[:m2], lm_head_w, k, VOCAB)
    lg = logits.cpu().numpy()
    for r in range(m2):
        err = np.abs(lg[r].astype(np.float64) - lr[r]).max()
        assert err <= 1e-3 * np.abs(lr[r]).max(), f"row {r}: max|err| {err:.3e}"
    print(f"config 4: {sample.size} sampled rows' tokens identical; 40 rows' logits within tolerance")
