"""Speculative decoding with the DFlash draft model and the target model, on
the device through the C ABI.

verify_steps() is the reference's run_target_dflash_verify loop
(src/lib.rs:466-528): per step the target runs forward_token on the current
token, capturing the draft's target_layers; the draft decodes from those
features; the target's lm_head scores the draft's hidden state; the draft
token is accepted when it equals the target's argmax, and the target's token
is always the next input.  Every tensor stays on the device; the host reads
two token ids per step.

verify_block() is the batched form a serving loop uses: the target runs a
whole block of proposed tokens through its K/V cache in one pass, the longest
prefix whose tokens the target itself predicts is kept, and the cache is
rolled back past it.
"""
from __future__ import annotations

import numpy as np

from . import lc
from .model import DFlash
from .target import Target


def verify_steps(target: Target, draft: DFlash, start_token: int, n_steps: int, target_layers):
    """Returns (accepted, draft_tokens, target_tokens), one entry per step."""
    import torch

    dev = torch.device("cuda", target.ctx.device)
    E = target.hp.n_embd
    layers = sorted(set(int(v) for v in target_layers))
    n_aux = len(layers)
    if draft.hp.n_embd != E or draft.hp.n_aux != n_aux:
        raise ValueError(f"draft (n_embd {draft.hp.n_embd}, {draft.hp.n_aux} target layers) does not fit the target "
                         f"(n_embd {E}, {n_aux} capture layers)")
    w_out, dt_out, _ = target.weight("output.weight")
    V = target.hp.n_vocab
    emb = torch.empty(1, E, device=dev)
    cap = torch.empty(1, n_aux, E, device=dev)
    enc = torch.empty(1, E, device=dev)
    dh = torch.empty(1, E, device=dev)
    keys = torch.empty(2, dtype=torch.int64, device=dev)  # target, draft
    token = int(start_token)
    accepted, drafts, targets = [], [], []
    for _ in range(n_steps):
        target.embed([token], emb)
        target.forward(emb, 1, capture=layers, captured=cap, keys=keys[0:1])
        draft.encode(cap.view(1, n_aux * E), 1, enc)
        draft.set_context(enc, 1)
        draft.decode_block(emb, 1, dh)
        target.ctx.lm_head_argmax(dt_out, dh, w_out, 1, E, V, 0, keys[1:2])
        k = keys.cpu().numpy()
        t_tok, d_tok = lc.key_index(int(k[0])), lc.key_index(int(k[1]))
        drafts.append(d_tok)
        targets.append(t_tok)
        accepted.append(d_tok if d_tok == t_tok else t_tok)
        token = accepted[-1]
    return accepted, drafts, targets


def verify_block(target: Target, tokens, emb=None, keys=None):
    """Run the proposed tokens (tokens[0] is the last accepted token, the rest
    the draft's proposals) through the target's cache; keep the prefix the
    target agrees with.  Returns (n_accepted_proposals, target_tokens) and
    leaves the cache holding the verified positions only."""
    import torch

    toks = np.asarray(tokens, np.uint32)
    m = toks.size
    E = target.hp.n_embd
    dev = torch.device("cuda", target.ctx.device)
    if emb is None:
        emb = torch.empty(m, E, device=dev)
    if keys is None:
        keys = torch.empty(m, dtype=torch.int64, device=dev)
    start = target.cache_len
    target.embed(toks, emb)
    target.forward(emb, m, cached=True, keys=keys)
    pred = [lc.key_index(int(k)) for k in keys[:m].cpu().numpy()]
    n = 0
    while n + 1 < m and pred[n] == int(toks[n + 1]):
        n += 1
    target.truncate(start + n + 1)
    return n, pred
