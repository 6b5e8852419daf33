"""GPU tests of the target-model subcommands of the laguna-cuda CLI
(csrc/cli/laguna_cuda_cli.cpp) against the target and DFlash oracles: the
reference's run_target_info / run_target_forward / run_target_generate /
run_target_dflash / run_target_dflash_verify / run_project_ref
(src/lib.rs:257-556, dispatched by src/main.rs:57-101).

Printed logits are compared within 2e-3 of the row's largest |logit|; tokens
are compared where the two best oracle logits are at least 1e-3 of that apart
(closer ones are ties the tolerance cannot order).  The oracle is fed the
CLI's chosen tokens, so one such tie cannot derail the later steps."""
import os
import re
import subprocess

import numpy as np
import pytest

import oracle as orc
import target_oracle as T
from conftest import ROOT
from dflash_oracle import DFlashOracle, make_model, tensor_shape
from gguf_writer import write_gguf

pytestmark = pytest.mark.gpu

CLI = os.path.join(ROOT, "laguna_raw_halo_strix_b200", "laguna-cuda")
DHP = dict(n_layers=2, n_embd=512, n_heads=4, n_kv_heads=2, head_dim=128, rope_dim=128, n_ff=768, n_aux=2,
           rope_base=500000.0, norm_eps=1e-5, qk_eps=1e-6)
TARGET_LAYERS = [3, 1]  # listed out of order: the capture runs in layer order
LOGIT = re.compile(r"^  logit\[(\d+)\] = (\S+)$")


def decided(row):
    top2 = np.sort(np.asarray(row, np.float64))[-2:]
    return top2[1] - top2[0] >= 1e-3 * np.abs(row).max()


def last_argmax(row):
    row = np.asarray(row)
    return len(row) - 1 - int(np.argmax(row[::-1]))


def run(*args, rc=0):
    r = subprocess.run([CLI] + [str(a) for a in args], capture_output=True, text=True, timeout=300)
    assert r.returncode == rc, (args, r.stdout, r.stderr)
    return r


def sections(text):
    """{heading: [(index, value)]} of the logit lists the CLI prints."""
    out, cur = {}, None
    for line in text.splitlines():
        m = LOGIT.match(line)
        if m:
            out[cur].append((int(m.group(1)), float(m.group(2))))
        else:
            cur = line
            out[cur] = []
    return {k: v for k, v in out.items() if v}


def check_logits(pairs, ref):
    tol = 2e-3 * np.abs(ref).max()
    for i, v in pairs:
        assert abs(v - ref[i]) <= tol, (i, v, ref[i])


def check_top(pairs, ref, n):
    """The top list: n entries in non-increasing order, each close to the
    oracle, and the first one the oracle's maximum when it is decided."""
    assert len(pairs) == n
    check_logits(pairs, ref)
    vals = [v for _, v in pairs]
    assert vals == sorted(vals, reverse=True)
    if decided(ref):
        assert pairs[0][0] == int(np.argmax(ref))


def tokens(line):
    return [int(v) for v in re.findall(r"\d+", line.split(":", 1)[1])]


@pytest.fixture(scope="module")
def files(tmp_path_factory):
    rng = np.random.default_rng(91)
    d = tmp_path_factory.mktemp("cli")
    hp = T.default_hp()
    tt = T.make_target(hp, orc.Q4_K, rng, embd_type=orc.Q8_0)
    tpath = str(d / "target.gguf")
    write_gguf(tpath, T.gguf_meta(hp), T.gguf_tensors(tt, hp))
    dt = make_model(DHP, orc.Q8_0, rng)
    meta = {"general.architecture": "dflash", "dflash.block_count": DHP["n_layers"],
            "dflash.embedding_length": DHP["n_embd"], "dflash.feed_forward_length": DHP["n_ff"],
            "dflash.attention.head_count": DHP["n_heads"], "dflash.attention.head_count_kv": DHP["n_kv_heads"],
            "dflash.attention.key_length": DHP["head_dim"], "dflash.rope.dimension_count": DHP["rope_dim"],
            "dflash.rope.freq_base": DHP["rope_base"], "dflash.target_layers": TARGET_LAYERS}
    dpath = str(d / "dflash.gguf")
    write_gguf(dpath, meta, [(n, t, tensor_shape(n, DHP), np.ascontiguousarray(a).view(np.uint8))
                             for n, (t, a) in dt.items()])
    return hp, tt, tpath, dt, dpath, d


def test_target_info(files):
    hp, tt, tpath, *_ = files
    out = run("target-info", tpath).stdout
    for key, val in (("layers", hp["n_layers"]), ("embedding_length", hp["n_embd"]), ("expert_count", hp["n_expert"]),
                     ("expert_used_count", hp["n_expert_used"]), ("vocab_size", hp["n_vocab"]),
                     ("has_moe", "true"), ("target_layers", "[]")):
        assert f"  {key}: {val}\n" in out, (key, out)
    to = T.TargetOracle(hp, tt)
    for l in range(hp["n_layers"]):
        assert f"  layer {l} [{'MoE' if to.is_moe(l) else 'Dense'}]\n" in out


def test_target_forward(files):
    hp, tt, tpath, *_ = files
    tok = 17
    out = run("target-forward", tpath, tok).stdout
    assert f"Running target model forward pass with token_id={tok}\n" in out
    assert f"Forward pass complete: {hp['n_vocab']} logits, {hp['n_layers']} captured states\n" in out
    to = T.TargetOracle(hp, tt)
    _, _, ref = to.forward_token(to.embed(tok))
    s = sections(out)
    check_top(s["Top logits:"], ref, 10)
    assert [i for i, _ in s["Specific indices:"]] == list(range(10))
    check_logits(s["Specific indices:"], ref)
    r = run("target-forward", tpath, hp["n_vocab"], rc=1)
    assert f"token_id {hp['n_vocab']} >= vocab_size {hp['n_vocab']}" in r.stderr


def test_target_generate(files):
    hp, tt, tpath, *_ = files
    start, n = 29, 5
    out = run("target-generate", tpath, start, n).stdout
    steps = re.findall(r"^  step (\d+): input=(\d+) -> next=(\d+)$", out, re.M)
    gen = tokens([l for l in out.splitlines() if l.startswith("Generated tokens:")][0])
    assert len(steps) == n and gen == [int(s[2]) for s in steps]
    to = T.TargetOracle(hp, tt)
    cur, checked = start, 0
    for i, (st, inp, nxt) in enumerate(steps):
        assert (int(st), int(inp)) == (i, cur)
        _, _, lg = to.forward_token(to.embed(cur), cached=True)
        if decided(lg):
            assert int(nxt) == last_argmax(lg), i
            checked += 1
        cur = int(nxt)
    assert checked >= n - 1


def draft_step(to, do, hp, tok):
    emb = to.embed(tok)
    cap, _, tlog = to.forward_token(emb, capture=sorted(TARGET_LAYERS))
    dh = do.forward_injected_decode_hidden(np.concatenate(cap), emb)
    return tlog, to._proj("output.weight", dh, hp["n_embd"], hp["n_vocab"])


def test_target_dflash(files):
    hp, tt, tpath, dt, dpath, _ = files
    tok = 41
    out = run("target-dflash", tpath, dpath, tok).stdout
    assert "DFlash target layers: [3, 1]\n" in out
    assert f"Captured 2 states, {2 * hp['n_embd']} feature floats\n" in out
    assert f"DFlash draft logits: {hp['n_vocab']}\n" in out
    _, dlog = draft_step(T.TargetOracle(hp, tt), DFlashOracle(DHP, dt), hp, tok)
    check_top(sections(out)["Top draft logits:"], dlog, 10)


def test_target_dflash_verify(files):
    hp, tt, tpath, dt, dpath, _ = files
    tok, n = 17, 5
    out = run("target-dflash-verify", tpath, dpath, tok, n).stdout
    steps = re.findall(r"^step (\d+): input=(\d+) draft=(\d+) target=(\d+) (ACCEPT|REJECT) -> accepted=(\d+)$",
                       out, re.M)
    assert len(steps) == n
    to, do = T.TargetOracle(hp, tt), DFlashOracle(DHP, dt)
    checked = exact = 0
    for i, (st, inp, d, t, verdict, acc) in enumerate(steps):
        assert (int(st), int(inp)) == (i, tok)
        assert (verdict == "ACCEPT") == (d == t) and int(acc) == int(t)
        exact += d == t
        tlog, dlog = draft_step(to, do, hp, tok)
        if decided(tlog):
            assert int(t) == last_argmax(tlog), i
            checked += 1
        if decided(dlog):
            assert int(d) == last_argmax(dlog), i
            checked += 1
        tok = int(acc)
    assert checked >= n
    acc_line = [l for l in out.splitlines() if l.startswith("accepted tokens:")][0]
    assert tokens(acc_line) == [int(s[5]) for s in steps]
    assert f"exact draft accept rate: {exact}/{n}\n" in out


def test_project_ref(files):
    hp, tt, tpath, *_, d = files
    rng = np.random.default_rng(5)
    hidden = rng.standard_normal(hp["n_embd"]).astype("<f4")
    hpath = str(d / "hidden.f32")
    hidden.tofile(hpath)
    out = run("project-ref", tpath, hpath).stdout
    ref = T.TargetOracle(hp, tt)._proj("output.weight", hidden, hp["n_embd"], hp["n_vocab"])
    s = sections(out)
    check_top(s["Top logits:"], ref, 10)
    assert [i for i, _ in s["Specific indices:"]] == list(range(8))
    check_logits(s["Specific indices:"], ref)
    hidden[:-1].tofile(hpath)  # one value short
    assert "expected" in run("project-ref", tpath, hpath, rc=1).stderr
