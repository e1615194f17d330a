"""Speculative decoding on two GPU sessions for many sequences at once: SpeculativeDecodeGreedy
(Brain/Reasoning/SpeculativeDecode.ts:32-98) and, further below, stochastic SpeculativeSample
(Brain/Reasoning/SpeculativeSampling.ts:38-115).

A draft session proposes up to Gamma tokens per sequence with cached greedy steps; the target session
checks all of them in one verify pass (shahd_verify: the proposals are appended to its cache with the LM
head on every row); each sequence keeps the longest prefix the target agrees with, plus the target's
correction at the first disagreement or its bonus token when all were accepted. Rejected rows are then
dropped from both caches (shahd_truncate). Within the context window the ids are those of plain greedy
decoding with the target (SpeculativeDecode.ts:5-10); this implementation requires the whole run to fit
the window (prompt + new tokens <= BlockSize of both models) instead of sliding it.

Every id comes from a device argmax (first index of the max); the host only compares ids.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np

from .decode import Session


@dataclass
class SpeculativeResult:
    ids: list            # per sequence: prompt + generated ids
    target_calls: list   # verify passes each sequence took part in
    draft_tokens: list   # tokens the draft proposed
    accepted_tokens: list  # proposals the target accepted


def speculative_decode_greedy(target: Session, draft: Session, prompts, max_new: int, gamma: int = 4,
                              slots=None) -> SpeculativeResult:
    """Decode each prompt with the target, using `draft` to propose `gamma` tokens per target pass."""
    prompts = [[int(t) for t in p] for p in prompts]
    n = len(prompts)
    slots = list(range(n)) if slots is None else [int(x) for x in slots]
    if any(len(p) == 0 for p in prompts):
        raise ValueError("SpeculativeDecodeGreedy: empty prompt")
    c_t, c_d = target.cfg.block_size, draft.cfg.block_size
    for p in prompts:
        if len(p) + max_new > min(c_t, c_d):
            raise ValueError(f"speculative decoding here needs prompt + new tokens <= the context window "
                             f"({len(p)} + {max_new} > {min(c_t, c_d)})")
    ids = [list(p) for p in prompts]
    calls, proposed_n, accepted_n = [0] * n, [0] * n, [0] * n
    if max_new < 1:
        return SpeculativeResult(ids, calls, proposed_n, accepted_n)
    # both caches hold every id but the last one; the last id is fed by the next step or pass
    for s in (target, draft):
        s.prefill(slots, [p[:-1] for p in prompts])
    dlen = [len(p) - 1 for p in prompts]  # the draft's cached length per sequence
    while True:
        active = [i for i in range(n) if len(ids[i]) - len(prompts[i]) < max_new]
        if not active:
            break
        g = {i: min(gamma, c_t - 1, max_new - (len(ids[i]) - len(prompts[i]))) for i in active}
        # the draft catches up on ids it has not cached yet (the target's bonus token of the last pass)
        while True:
            behind = [i for i in active if dlen[i] < len(ids[i]) - 1]
            if not behind:
                break
            draft.step([slots[i] for i in behind], [ids[i][dlen[i]] for i in behind], want_logits=False)
            for i in behind:
                dlen[i] += 1
        # 1) the draft proposes g[i] tokens greedily (cached steps, every sequence batched per step)
        prop = {i: [] for i in active}
        for k in range(max(g.values())):
            rows = [i for i in active if g[i] > k]
            feed = [ids[i][-1] if k == 0 else prop[i][-1] for i in rows]
            _, nxt = draft.step([slots[i] for i in rows], feed, want_logits=False)
            for i, t in zip(rows, nxt):
                prop[i].append(int(t))
                dlen[i] += 1
        for i in active:
            proposed_n[i] += g[i]
        # 2) the target checks all proposals of every sequence in one pass
        checks = target.verify([slots[i] for i in active], [[ids[i][-1]] + prop[i] for i in active])
        keep_t, keep_d = [], []
        for i, t_ids in zip(active, checks):
            calls[i] += 1
            corrected = False
            acc = 0
            for j in range(g[i]):
                if int(t_ids[j]) == prop[i][j]:
                    ids[i].append(prop[i][j])
                    acc += 1
                    accepted_n[i] += 1
                    if len(ids[i]) - len(prompts[i]) >= max_new:
                        break
                else:
                    ids[i].append(int(t_ids[j]))  # correction at the first divergence
                    corrected = True
                    break
            # 3) all accepted with budget left: the target's own next argmax is free
            if not corrected and acc == g[i] and len(ids[i]) - len(prompts[i]) < max_new:
                ids[i].append(int(t_ids[g[i]]))
            keep_t.append(len(ids[i]) - 1)
            dlen[i] = min(dlen[i], len(ids[i]) - 1)
            keep_d.append(dlen[i])
        # 4) rows of rejected proposals leave both caches
        target.truncate([slots[i] for i in active], keep_t)
        draft.truncate([slots[i] for i in active], keep_d)
    return SpeculativeResult([x[:len(p) + max_new] for x, p in zip(ids, prompts)], calls, proposed_n, accepted_n)


# ---- stochastic speculative sampling -------------------------------------------------------------------

@dataclass
class SpeculativeSampleRound:
    """What one verification round of one sequence saw (kept when record=True, for checking)."""
    seq: int
    draft_logits: np.ndarray   # [g, V] the distributions the proposals were drawn from
    proposals: list
    target_logits: np.ndarray  # [g + 1, V]
    budget: int
    rng_at_start: int          # SeededRng state before the proposals' draws
    rng_before_round: int      # SeededRng state after the proposals' draws, before the round's draws
    appended: list
    accepted: int


def speculative_sample(target: Session, draft: Session, prompts, max_new: int, sampling, rng_states: np.ndarray,
                       gamma: int = 4, slots=None, record: bool = False):
    """SpeculativeSample (Brain/Reasoning/SpeculativeSampling.ts:38-115) for many sequences at once.

    Each round: the draft proposes min(gamma, BlockSize - 1, budget) ids per sequence with cached steps,
    each drawn on the device from its distribution with the sequence's SeededRng (rng_states, uint32 [n],
    advanced in place, one draw per proposal); the target scores all proposals in one verify pass
    (shahd_verify); the device round (shahd_speculative_round) accepts each proposal with probability
    min(1, p/q), replaces the first rejection from the residual max(0, p - q), or draws a bonus id, with the
    same Rng; rejected rows then leave both caches. Needs temperature > 0 and prompt + new ids within both
    context windows. Returns (SpeculativeResult, rounds) where rounds lists SpeculativeSampleRound records
    when record=True."""
    from . import _lib
    from .decode import sample_from_logits

    if not (sampling.temperature > 0):
        raise ValueError("SpeculativeSample: temperature must be > 0 here (greedy: speculative_decode_greedy)")
    prompts = [[int(t) for t in p] for p in prompts]
    n = len(prompts)
    if rng_states is None or len(rng_states) != n:
        raise ValueError("SpeculativeSample: one SeededRng state per sequence is required")
    slots = list(range(n)) if slots is None else [int(x) for x in slots]
    if any(len(p) == 0 for p in prompts):
        raise ValueError("SpeculativeSample: empty prompt")
    c_t, c_d = target.cfg.block_size, draft.cfg.block_size
    for p in prompts:
        if len(p) + max_new > min(c_t, c_d):
            raise ValueError(f"speculative sampling here needs prompt + new tokens <= the context window "
                             f"({len(p)} + {max_new} > {min(c_t, c_d)})")
    V = target.cfg.vocab_size
    ids = [list(p) for p in prompts]
    calls, proposed_n, accepted_n = [0] * n, [0] * n, [0] * n
    rounds = []
    if max_new < 1:
        return SpeculativeResult(ids, calls, proposed_n, accepted_n), rounds
    for s in (target, draft):
        s.prefill(slots, [p[:-1] for p in prompts])
    dlen = [len(p) - 1 for p in prompts]
    lib = _lib.load()
    while True:
        active = [i for i in range(n) if len(ids[i]) - len(prompts[i]) < max_new]
        if not active:
            break
        g = {i: min(gamma, c_t - 1, max_new - (len(ids[i]) - len(prompts[i]))) for i in active}
        while True:  # the draft caches every id but the last one before proposing
            behind = [i for i in active if dlen[i] < len(ids[i]) - 1]
            if not behind:
                break
            draft.step([slots[i] for i in behind], [ids[i][dlen[i]] for i in behind], want_logits=False)
            for i in behind:
                dlen[i] += 1
        # 1) the draft proposes: cached steps, each row's id drawn on the device with its own Rng
        rng_start = {i: int(rng_states[i]) for i in active}
        prop = {i: [] for i in active}
        dlog = {i: [] for i in active}
        for k in range(max(g.values())):
            rows = [i for i in active if g[i] > k]
            feed = [ids[i][-1] if k == 0 else prop[i][-1] for i in rows]
            logits, _ = draft.step([slots[i] for i in rows], feed)
            st = np.ascontiguousarray([rng_states[i] for i in rows], dtype=np.uint32)
            toks = sample_from_logits(logits, sampling, st)
            for j, i in enumerate(rows):
                rng_states[i] = st[j]
                prop[i].append(int(toks[j]))
                dlog[i].append(logits[j])
                dlen[i] += 1
        for i in active:
            proposed_n[i] += g[i]
        # 2) the target scores every proposal in one pass
        _, tlog = target.verify([slots[i] for i in active], [[ids[i][-1]] + prop[i] for i in active], want_logits=True)
        # 3) the device round: accept / residual / bonus for every sequence at once
        na = len(active)
        gmax = max(g.values())
        t_rows = np.zeros((na, gmax + 1, V), np.float32)
        d_rows = np.zeros((na, gmax, V), np.float32)
        props = np.zeros((na, gmax), np.int32)
        gs = np.array([g[i] for i in active], np.int32)
        budget = np.array([max_new - (len(ids[i]) - len(prompts[i])) for i in active], np.int32)
        for j, i in enumerate(active):
            t_rows[j, : g[i] + 1] = tlog[j]
            if g[i]:
                d_rows[j, : g[i]] = np.stack(dlog[i])
                props[j, : g[i]] = prop[i]
        st = np.ascontiguousarray([rng_states[i] for i in active], dtype=np.uint32)
        st_before = st.copy()
        out = np.zeros((na, gmax + 1), np.int32)
        cnt = np.zeros(na, np.int32)
        acc = np.zeros(na, np.int32)
        o = sampling.to_c()
        fp = ctypes.POINTER(ctypes.c_float)
        ip = ctypes.POINTER(ctypes.c_int32)
        _lib.check(lib.shahd_speculative_round(t_rows.ctypes.data_as(fp), d_rows.ctypes.data_as(fp),
                                               props.ctypes.data_as(ip), gs.ctypes.data_as(ip),
                                               budget.ctypes.data_as(ip), na, gmax, V, ctypes.byref(o),
                                               st.ctypes.data_as(ctypes.POINTER(ctypes.c_uint32)),
                                               out.ctypes.data_as(ip), cnt.ctypes.data_as(ip),
                                               acc.ctypes.data_as(ip)))
        keep_t, keep_d = [], []
        for j, i in enumerate(active):
            rng_states[i] = st[j]
            calls[i] += 1
            appended = out[j, : cnt[j]].tolist()
            ids[i].extend(appended)
            accepted_n[i] += int(acc[j])
            if record:
                rounds.append(SpeculativeSampleRound(i, d_rows[j, : g[i]].copy(), list(prop[i]),
                                                     t_rows[j, : g[i] + 1].copy(), int(budget[j]), rng_start[i],
                                                     int(st_before[j]), appended, int(acc[j])))
            keep_t.append(len(ids[i]) - 1)
            dlen[i] = min(dlen[i], len(ids[i]) - 1)
            keep_d.append(dlen[i])
        # 4) rows of rejected proposals leave both caches
        target.truncate([slots[i] for i in active], keep_t)
        draft.truncate([slots[i] for i in active], keep_d)
    return SpeculativeResult([x[:len(p) + max_new] for x, p in zip(ids, prompts)], calls, proposed_n, accepted_n), rounds
