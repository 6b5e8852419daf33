"""GPU tests of speculative decoding (laguna_raw_halo_strix_b200/speculative.py)
against the oracles: the reference's run_target_dflash_verify loop
(src/lib.rs:466-528) and the cached block verify with rollback.

Token checks follow the spec (identical argmax tokens); a step whose two best
oracle logits are closer than 1e-3 of the row's largest |logit| is a tie the
tolerance cannot order, and its token is not compared.  The oracle is fed the
GPU's chosen tokens, so one such tie cannot derail the later steps."""
import numpy as np
import pytest

import oracle as orc
import target_oracle as T
from dflash_oracle import DFlashOracle, make_model
from gguf_writer import write_gguf
from laguna_raw_halo_strix_b200 import speculative
from laguna_raw_halo_strix_b200.model import DFlash, hparams
from laguna_raw_halo_strix_b200.target import Target

pytestmark = pytest.mark.gpu

DHP = dict(n_layers=2, n_embd=512, n_heads=4, n_kv_heads=2, head_dim=128, rope_dim=128, n_ff=768, n_aux=2,
           rope_base=500000.0, norm_eps=1e-5, qk_eps=1e-6)
TARGET_LAYERS = (1, 3)


def decided(row):
    row = np.asarray(row, np.float64)
    top2 = np.sort(row)[-2:]
    return top2[1] - top2[0] >= 1e-3 * np.abs(row).max()


def last_argmax(row):
    row = np.asarray(row)
    return len(row) - 1 - int(np.argmax(row[::-1]))


@pytest.fixture(scope="module")
def pair(ctx, tmp_path_factory):
    rng = np.random.default_rng(77)
    hp = T.default_hp()
    tt = T.make_target(hp, orc.Q4_K, rng, embd_type=orc.Q8_0)
    path = str(tmp_path_factory.mktemp("spec") / "target.gguf")
    write_gguf(path, T.gguf_meta(hp), T.gguf_tensors(tt, hp))
    target = Target(ctx, path, max_ctx=64, max_block=8)
    dt = make_model(DHP, orc.Q8_0, rng)
    draft = DFlash(ctx, hparams(**DHP), max_ctx=4, max_block=4)
    for name, (d, a) in dt.items():
        draft.set_tensor(name, d, a)
    yield hp, tt, target, dt, draft
    draft.close()
    target.close()


def test_verify_steps_match_reference_loop(pair):
    hp, tt, target, dt, draft = pair
    steps = 6
    accepted, drafts, targets = speculative.verify_steps(target, draft, 17, steps, TARGET_LAYERS)
    to = T.TargetOracle(hp, tt)
    do = DFlashOracle(DHP, dt)
    token = 17
    checked = 0
    for s in range(steps):
        emb = to.embed(token)
        cap, _, tlog = to.forward_token(emb, capture=TARGET_LAYERS)
        dh = do.forward_injected_decode_hidden(np.concatenate(cap), emb)
        dlog = to._proj("output.weight", dh, hp["n_embd"], hp["n_vocab"])
        if decided(tlog):
            assert targets[s] == last_argmax(tlog), s
            checked += 1
        if decided(dlog):
            assert drafts[s] == last_argmax(dlog), s
            checked += 1
        assert accepted[s] == targets[s]  # the target's token is always the next input
        token = accepted[s]
    assert checked >= steps


def test_verify_block_accepts_the_agreed_prefix(pair, dev):
    """Proposals that follow the target's own greedy choice for two steps and
    then differ: two are accepted and the cache keeps the verified positions;
    the next block continues from there."""
    hp, tt, target, _, _ = pair
    target.truncate(0)
    to = T.TargetOracle(hp, tt)
    toks = [5]
    for _ in range(2):  # the oracle's greedy continuation through its cache
        _, _, lg = to.forward(to.embed(toks[-1])[None, :], cached=True)
        assert decided(lg[0])
        toks.append(last_argmax(lg[0]))
    _, _, lg = to.forward(to.embed(toks[-1])[None, :], cached=True)
    wrong = (last_argmax(lg[0]) + 1) % hp["n_vocab"]
    n, pred = speculative.verify_block(target, toks + [wrong])
    assert n == 2 and pred[:3] == [toks[1], toks[2], last_argmax(lg[0])]
    assert target.cache_len == 3
    # continue from the last verified position with the corrected token
    to.truncate(3)
    n2, pred2 = speculative.verify_block(target, [pred[2]])
    _, _, lg2 = to.forward(to.embed(pred[2])[None, :], cached=True)
    assert n2 == 0 and target.cache_len == 4
    if decided(lg2[0]):
        assert pred2[0] == last_argmax(lg2[0])
    target.truncate(0)
