"""GPU parity of the target (Laguna) model -- lc_target_* -- against the CPU
oracle's restatement of TargetModel (src/target.rs:314-748): forward_token
rows, the cached verify block, K/V rollback, the on-device MoE routing and
expert FFNs, and the token embedding.

Tolerances follow the spec: hidden states within rel-L2 <= 2e-3 and identical
argmax tokens (rows whose two best oracle logits are closer than 1e-3 of the
row's largest |logit| are ties the tolerance cannot order, and are not
compared); projection-level outputs within 1e-3 * ||y||_inf."""
import numpy as np
import pytest

import oracle as orc
import target_oracle as T
from conftest import check_tol, to_dev
from gguf_writer import write_gguf
from laguna_raw_halo_strix_b200 import lc
from laguna_raw_halo_strix_b200.target import Target

pytestmark = pytest.mark.gpu


def rel_l2(a, b):
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def build(tmp_path, hp, t, name="t.gguf"):
    path = str(tmp_path / name)
    write_gguf(path, T.gguf_meta(hp), T.gguf_tensors(t, hp))
    return path


def check_tokens(keys, ref_logits):
    for r in range(ref_logits.shape[0]):
        row = ref_logits[r].astype(np.float64)
        top2 = np.sort(row)[-2:]
        if top2[1] - top2[0] < 1e-3 * np.abs(row).max():
            continue
        want = len(row) - 1 - int(np.argmax(row[::-1]))  # the last maximum wins (src/lib.rs:456-464)
        assert lc.key_index(int(keys[r])) == want, r


@pytest.fixture(scope="module", params=[orc.Q4_K, orc.Q8_0])
def model(request, ctx, tmp_path_factory):
    hp = T.default_hp()
    rng = np.random.default_rng(100 + request.param)
    t = T.make_target(hp, request.param, rng)
    path = build(tmp_path_factory.mktemp("target"), hp, t)
    tm = Target(ctx, path, max_ctx=64, max_block=16)
    yield hp, t, tm
    tm.close()


def test_layout(model):
    hp, t, tm = model
    assert [tm.layer_info(l) for l in range(hp["n_layers"])] == [(False, 4), (True, 4), (True, 8), (True, 4)]
    assert tm.hp.n_vocab == hp["n_vocab"] and tm.hp.has_moe == 1


@pytest.mark.parametrize("m", [1, 5, 16])
def test_forward_token_rows(model, dev, m):
    """Without the cache every row is forward_token (src/target.rs:314): the
    captured layer inputs, the output_norm'ed state, the logits and the argmax."""
    import torch

    hp, t, tm = model
    E, V = hp["n_embd"], hp["n_vocab"]
    rng = np.random.default_rng(m)
    x = rng.standard_normal((m, E)).astype(np.float32)
    cap_layers = [0, 2, 4]
    cap = torch.full((m, 3, E), float("nan"), device=dev)
    hid = torch.empty(m, E, device=dev)
    logits = torch.empty(m, V, device=dev)
    keys = torch.empty(m, dtype=torch.int64, device=dev)
    tm.forward(to_dev(x, dev), m, capture=cap_layers, captured=cap, hidden=hid, logits=logits, keys=keys)
    torch.cuda.synchronize()
    assert tm.cache_len == 0
    om = T.TargetOracle(hp, t)
    rc, rh, rl = om.forward(x, capture=cap_layers)
    got_c = cap.cpu().numpy()
    assert np.array_equal(got_c[:, 0], x)
    for j in (1, 2):
        assert rel_l2(got_c[:, j], rc[:, j]) <= 2e-3, j
    assert rel_l2(hid.cpu().numpy(), rh) <= 2e-3
    assert rel_l2(logits.cpu().numpy(), rl) <= 2e-3
    check_tokens(keys.cpu().numpy(), rl)


def test_cached_verify_blocks_and_rollback(model, dev):
    """Blocks of 4 and 3 draft tokens through the cache equal 7 sequential
    forward_token_cached calls; truncating to 5 positions and verifying 2 new
    tokens equals the oracle rolled back the same way."""
    import torch

    hp, t, tm = model
    E, V = hp["n_embd"], hp["n_vocab"]
    rng = np.random.default_rng(7)
    xs = rng.standard_normal((9, E)).astype(np.float32)
    om = T.TargetOracle(hp, t)
    tm.truncate(0)

    def step(rows):
        m = rows.shape[0]
        hid = torch.empty(m, E, device=dev)
        logits = torch.empty(m, V, device=dev)
        keys = torch.empty(m, dtype=torch.int64, device=dev)
        tm.forward(to_dev(rows, dev), m, cached=True, hidden=hid, logits=logits, keys=keys)
        torch.cuda.synchronize()
        _, rh, rl = om.forward(rows, cached=True)
        assert rel_l2(hid.cpu().numpy(), rh) <= 2e-3
        assert rel_l2(logits.cpu().numpy(), rl) <= 2e-3
        check_tokens(keys.cpu().numpy(), rl)

    step(xs[0:4])
    step(xs[4:7])
    assert tm.cache_len == 7 and om.cache_len == 7
    tm.truncate(5)
    om.truncate(5)
    step(xs[7:9])
    assert tm.cache_len == 7
    with pytest.raises(lc.LagunaError):
        tm.forward(to_dev(xs[:1], dev), 17, cached=True)  # more rows than max_block
    tm.truncate(0)


@pytest.mark.parametrize("m", [2, 12])
def test_moe_routing_and_experts(model, dev, m):
    """lc_target_moe_ffn: the selected experts and their order are the
    oracle's, the scores agree to rounding, the FFN output to the projection
    bound -- for a 2-row block (only the selected experts are read) and a
    12-row block (its 48 selections can cover the 16 experts: every expert's
    gate / up run as one tensor-core GEMM)."""
    import torch

    hp, t, tm = model
    E, NU = hp["n_embd"], hp["n_expert_used"]
    rng = np.random.default_rng(11 + m)
    nx = rng.standard_normal((m, E)).astype(np.float32)
    om = T.TargetOracle(hp, t)
    for layer in (1, 3):
        y = torch.empty(m, E, device=dev)
        ids = torch.empty(m, NU, dtype=torch.int32, device=dev)
        sc = torch.empty(m, NU, device=dev)
        tm.moe_ffn(layer, to_dev(nx, dev), m, y, ids, sc)
        logged, rows = tm.routing(layer)  # lc_target_routing: the same selection
        torch.cuda.synchronize()
        assert rows == m and torch.equal(logged, ids)
        for r in range(m):
            ry, rids, rsc = om.moe_ffn(layer, nx[r])
            assert list(ids[r].cpu().numpy()) == list(rids), (layer, r)
            assert np.allclose(sc[r].cpu().numpy(), rsc, rtol=1e-5, atol=0), (layer, r)
            check_tol(y[r].cpu().numpy(), ry, 1e-3, f"moe layer {layer} row {r}")


@pytest.mark.parametrize("expert_type", [orc.F32, orc.Q8_0])
def test_expert_formats_and_reference_offset_quirk(ctx, dev, tmp_path, expert_type):
    """F32 and Q8_0 expert stacks read their own expert by default; with
    LC_TARGET_REF_EXPERT_OFFSET every one reads expert 0, as the reference's
    dispatch_proj_quant_expert does (src/target.rs:1098-1162)."""
    import torch

    hp = T.default_hp(n_layers=2, q_heads={}, gate_layers=(0,))
    rng = np.random.default_rng(20 + expert_type)
    t = T.make_target(hp, orc.Q4_K, rng, expert_type=expert_type)
    path = build(tmp_path, hp, t)
    E, m = hp["n_embd"], 6
    nx = rng.standard_normal((m, E)).astype(np.float32)
    for flags, quirk in ((0, False), (lc.TARGET_REF_EXPERT_OFFSET, True)):
        tm = Target(ctx, path, max_ctx=8, max_block=8, flags=flags)
        y = torch.empty(m, E, device=dev)
        tm.moe_ffn(1, to_dev(nx, dev), m, y)
        torch.cuda.synchronize()
        om = T.TargetOracle(hp, t, ref_expert_offset=quirk)
        for r in range(m):
            check_tol(y[r].cpu().numpy(), om.moe_ffn(1, nx[r])[0], 1e-3, f"experts {expert_type} quirk {quirk}")
        tm.close()


@pytest.mark.parametrize("embd_type", [orc.F32, orc.Q8_0, orc.Q4_K])
def test_embed(ctx, dev, tmp_path, embd_type):
    """target_token_embedding (src/lib.rs:431-454): dequant_to_f32 of the
    token's row, bit for bit -- including the CPU decoder's own Q4_K branch."""
    import torch

    hp = T.default_hp(n_layers=1, has_moe=0, q_heads={}, gate_layers=())
    rng = np.random.default_rng(30)
    t = T.make_target(hp, orc.Q8_0, rng, embd_type=embd_type)
    tm = Target(ctx, build(tmp_path, hp, t), max_ctx=4, max_block=4)
    toks = [0, 999, 17, 500]
    x = torch.empty(len(toks), hp["n_embd"], device=dev)
    tm.embed(toks, x)
    torch.cuda.synchronize()
    om = T.TargetOracle(hp, t)
    for r, tok in enumerate(toks):
        assert np.array_equal(x[r].cpu().numpy().view(np.uint32), om.embed(tok).view(np.uint32)), tok
    with pytest.raises(lc.LagunaError):
        tm.embed([1000], x)
    tm.close()
