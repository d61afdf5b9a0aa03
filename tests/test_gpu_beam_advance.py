"""GPU parity of the beam loop's on-device decision (sv_beam_advance) against the
reference's host bookkeeping (runtime_shared.py:237-259), restated here on lists:
hits from _ends on the candidates (eos, stop sequence, last step), live scores in
float64, the stable descending order of the first `beams`, running scores as
float32, the padding with order[0], and the seen / token-history reorder.  Every
output is compared exactly."""
import random
from array import array

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


def reference_decision(picks, scores, beams, vocab, step, last, stop_ids, eos_id, running):
    """runtime_shared.py:237-248 on host lists; running = the rows' token lists."""
    parents, tokens = zip(*(divmod(p, vocab) for p in picks))
    candidates = [running[p] + [t] for p, t in zip(parents, tokens)]
    hits = [last or c[-1] == eos_id or c[-len(stop_ids):] == stop_ids for c in candidates]
    live = [s - 1e9 * h for s, h in zip(scores, hits)]
    order = sorted(range(len(scores)), key=live.__getitem__, reverse=True)[:beams]
    running_scores = [live[j] for j in order] + [-1e9] * (beams - len(order))
    order += [order[0]] * (beams - len(order))
    return ([parents[j] for j in order], [tokens[j] for j in order], array("f", running_scores).tolist(),
            [candidates[j] for j in order])


def run_device(picks, scores, status, beams, vocab, step, last, stop_ids, eos_id, running, num_picks, sv,
               with_state=True):
    n = len(picks)
    S = len(stop_ids)
    o = {"picks": torch.tensor(picks + [-1] * (num_picks - n), dtype=torch.int64, device=DEV),
         "scores": torch.tensor(scores + [0.0] * (num_picks - n), dtype=torch.float32, device=DEV),
         "n": torch.tensor([n], dtype=torch.int32, device=DEV),
         "status": torch.tensor([status], dtype=torch.int32, device=DEV)}
    tails = torch.full((2, beams, max(S, 1)), -1, dtype=torch.int64, device=DEV)
    for r, seq in enumerate(running):
        tail = seq[-S:] if S else []
        for k, t in enumerate(tail):
            tails[0, r, S - len(tail) + k] = t
    words = (vocab + 31) // 32
    seen_in = torch.randint(-2**31, 2**31 - 1, (beams, words + 3), dtype=torch.int32, device=DEV)
    seen_out = torch.zeros_like(seen_in)
    cap = step + 5
    hist_in = torch.zeros((beams, cap), dtype=torch.int32, device=DEV)
    for r, seq in enumerate(running):
        if seq:
            hist_in[r, :len(seq)] = torch.tensor(seq, dtype=torch.int32)
    hist_out = torch.full_like(hist_in, -7)
    out = dict(running=torch.full((beams,), 5.0, device=DEV), parents=torch.full((beams,), -3, dtype=torch.int64,
                                                                                 device=DEV),
               tokens=torch.full((beams,), -3, dtype=torch.int64, device=DEV))
    stop_dev = torch.tensor(stop_ids, dtype=torch.int64, device=DEV) if S else None
    sv.ops.beam_advance(o, beams=beams, vocab=vocab, step=step, last=last, stop_ids=stop_dev, eos_id=eos_id,
                        tails_in=tails[0], tails_out=tails[1], running_out=out["running"],
                        parents_out=out["parents"], tokens_out=out["tokens"],
                        seen_in=seen_in[:, :words + 3] if with_state else None,
                        seen_out=seen_out if with_state else None,
                        hist_in=hist_in if with_state else None, hist_out=hist_out if with_state else None)
    torch.cuda.synchronize()
    return out, tails, seen_in, seen_out, hist_out


def expected_seen(seen_in, parents, tokens, words):
    exp = seen_in[parents].clone()
    for b, t in enumerate(tokens):
        w = t >> 5
        v = int(exp[b, w]) & 0xffffffff
        v |= 1 << (t & 31)
        exp[b, w] = v - (1 << 32) if v >= 1 << 31 else v
    return exp[:, :words]


@pytest.mark.parametrize("beams", [1, 2, 3, 8])
@pytest.mark.parametrize("stop", [[], [3], [3, 4], [5, 6, 7]])
def test_decision_matches_reference(sv, beams, stop):
    rng = random.Random(beams * 31 + len(stop))
    vocab = 97
    num_picks = 2 * beams
    for trial in range(40):
        step = rng.randrange(0, 12)
        running = [[rng.choice([3, 4, 5, 6, 7, 8]) for _ in range(step)] for _ in range(beams)]
        n = rng.randint(1, num_picks)
        flat = rng.sample(range(beams * vocab), n)
        # Candidates that end with the stop sequence or eos, and tied scores.
        for j in range(n):
            if stop and rng.random() < 0.3:
                flat[j] = (flat[j] // vocab) * vocab + stop[-1]
            if rng.random() < 0.1:
                flat[j] = (flat[j] // vocab) * vocab + 11
        flat = list(dict.fromkeys(flat))
        n = len(flat)
        scores = [float(array("f", [rng.choice([-1.5, -2.25, rng.uniform(-30, 0)])])[0]) for _ in range(n)]
        last = trial % 9 == 8
        parents, tokens, rs, cands = reference_decision(flat, scores, beams, vocab, step, last, stop, 11, running)
        out, tails, seen_in, seen_out, hist_out = run_device(flat, scores, 0, beams, vocab, step, last, stop, 11,
                                                             running, num_picks, sv)
        assert out["parents"].tolist() == parents
        assert out["tokens"].tolist() == tokens
        assert out["running"].tolist() == rs
        S = len(stop)
        if S:
            want = [([-1] * S + c)[-S:] for c in cands]
            assert tails[1].tolist() == want
        words = (vocab + 31) // 32
        assert torch.equal(seen_out[:, :words], expected_seen(seen_in, parents, tokens, words))
        assert hist_out[:, :step + 1].tolist() == cands
        assert (hist_out[:, step + 1:] == -7).all()


def test_failed_step_keeps_rows(sv):
    beams, vocab = 4, 64
    running = [[1, 2], [3, 4], [5, 6], [7, 8]]
    out, tails, seen_in, seen_out, hist_out = run_device([5, 70], [-1.0, -2.0], 1, beams, vocab, 2, False, [3, 4],
                                                         None, running, 8, sv)
    assert out["parents"].tolist() == [0, 1, 2, 3]
    assert out["tokens"].tolist() == [0, 0, 0, 0]
    assert out["running"].tolist() == array("f", [0.0, -1e9, -1e9, -1e9]).tolist()
    assert torch.equal(tails[1], tails[0])
    assert torch.equal(seen_out[:, :2], seen_in[:, :2])


def test_fewer_picks_than_beams_pad_with_the_best(sv):
    beams, vocab = 4, 50
    running = [[], [], [], []]
    out, *_ = run_device([7, 3], [-4.0, -1.0], 0, beams, vocab, 0, False, [9, 9], None, running, 8, sv)
    assert out["parents"].tolist() == [0, 0, 0, 0]
    assert out["tokens"].tolist() == [3, 7, 3, 3]
    assert out["running"].tolist() == array("f", [-1.0, -4.0, -1e9, -1e9]).tolist()


def test_without_optional_state(sv):
    beams, vocab = 2, 40
    out, *_ = run_device([41, 2, 5], [-1.0, -3.0, -0.5], 0, beams, vocab, 0, False, [], None, [[], []], 4, sv,
                         with_state=False)
    assert out["parents"].tolist() == [0, 1]
    assert out["tokens"].tolist() == [5, 1]


@pytest.mark.parametrize("window,repeats", [(8, 3), (64, 3)])
def test_beam_guard_table_tracks_running_row_0(sv, window, repeats):
    """A 400-step beam run whose rows are reordered every step: the incremental
    guard (windows entered by sv_beam_advance, probed for row 0) agrees at every
    16th step with a full rescan of row 0's history (the oracle)."""
    from oracle import oracle as O
    rng = random.Random(window)
    beams, vocab, steps = 4, 50, 400
    period = [rng.randrange(vocab) for _ in range(7)]
    hist = torch.zeros((2, beams, steps), dtype=torch.int32, device=DEV)
    whash = torch.zeros((2, beams), dtype=torch.int32, device=DEV)
    table = sv.ops.guard_table(beams * steps, DEV)
    tails = torch.full((2, beams, 1), -1, dtype=torch.int64, device=DEV)
    running = torch.zeros((beams,), device=DEV)
    parents = torch.zeros((beams,), dtype=torch.int64, device=DEV)
    tokens = torch.zeros((beams,), dtype=torch.int64, device=DEV)
    verdict = torch.zeros(1, dtype=torch.uint8, device=DEV)
    checked = hits = 0
    for step in range(steps):
        cur, nxt = step % 2, 1 - step % 2
        flat = []
        for _ in range(64):  # up to 2 * beams distinct picks (fewer in the periodic stretch)
            if len(flat) == 2 * beams:
                break
            p = rng.randrange(beams)
            # Periodic in steps [100, 300) (the guard fires there), noisy elsewhere.
            t = period[step % 7] if 100 <= step < 300 or rng.random() < 0.85 else rng.randrange(vocab)
            if p * vocab + t not in flat:
                flat.append(p * vocab + t)
                if rng.random() < 0.3:
                    break
        pad = 2 * beams - len(flat)
        o = {"picks": torch.tensor(flat + [-1] * pad, dtype=torch.int64, device=DEV),
             "scores": torch.tensor([rng.uniform(-20, 0) for _ in flat] + [0.0] * pad, dtype=torch.float32,
                                    device=DEV),
             "n": torch.tensor([len(flat)], dtype=torch.int32, device=DEV),
             "status": torch.zeros(1, dtype=torch.int32, device=DEV)}
        sv.ops.beam_advance(o, beams=beams, vocab=vocab, step=step, last=False, stop_ids=None, eos_id=None,
                            tails_in=tails[cur], tails_out=tails[nxt], running_out=running, parents_out=parents,
                            tokens_out=tokens, hist_in=hist[cur], hist_out=hist[nxt], whash_in=whash[cur],
                            whash_out=whash[nxt], guard_table=table, window=window)
        if step % 16 == 15:
            sv.ops.loop_guard_incremental(table, hist[nxt, 0], step + 1, step + 1, window, repeats, out=verdict)
            row0 = hist[nxt, 0, :step + 1].cpu().numpy()
            want = bool(O.repeating(row0[None], None, window, repeats)[0])
            assert bool(verdict.item()) == want, step
            checked += 1
            hits += want
    assert checked == steps // 16 and 0 < hits < checked
