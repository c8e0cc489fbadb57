"""CPU: the host side of the speculative path (kernel_optim_b200/spec.py) against a model stand-in.

The stand-in is a deterministic "language model" whose greedy next token depends on the two tokens
before it; its verify forward writes the rows' tokens into a per-sequence cache at their positions
(as the prologue appends K/V) and picks the next token after each row position, so the tokens that
``speculate`` + ``drain_one_token`` emit must equal plain greedy decoding token for token, whatever
the drafts were, the sequences' different rates and the break-even fallback included.
"""

import random

import pytest

from kernel_optim_b200.spec import Lookup, accept, draft_len, drain_one_token, speculate

V = 11


def nxt(a: int, b: int) -> int:
    """The stand-in's greedy pick after tokens a, b (small vocabulary: it falls into loops)."""
    return (7 * a + 3 * b + (a * b) % 5) % V


def greedy(prompt, n):
    s = list(prompt)
    for _ in range(n):
        s.append(nxt(s[-2], s[-1]))
    return s[len(prompt):]


class StandIn:
    """Per-sequence token cache indexed by position; verify and one-token steps on it."""

    def __init__(self, prompts):
        self.cache = [dict(enumerate(p)) for p in prompts]
        self.calls = 0

    def verify(self, rows, positions):
        self.calls += 1
        picks = []
        for b, (row, p) in enumerate(zip(rows, positions)):
            c = self.cache[b]
            for t, tok in enumerate(row):
                c[p + t] = tok
            picks.append([nxt(c[p + t - 1], c[p + t]) for t in range(len(row))])
        return picks

    def one_token(self, last, pos, n):
        """n one-token steps from each sequence's last token at its own position."""
        last, pos = list(last), list(pos)
        for _ in range(n):
            toks = []
            for b in range(len(last)):
                c = self.cache[b]
                c[pos[b]] = last[b]
                toks.append(nxt(c[pos[b] - 1], c[pos[b]]))
            last = toks
            pos = [p + 1 for p in pos]
            yield toks


def run(prompts, N, K, breakeven, window=8):
    B, S = len(prompts), len(prompts[0])
    m = StandIn(prompts)
    first = [nxt(p[-2], p[-1]) for p in prompts]
    out = [first]
    gen = speculate(prompts, first, N, K, m.verify, breakeven, window)
    try:
        while True:
            out.append(next(gen))
    except StopIteration as stop:
        outs = stop.value
    ready = min(len(o) for o in outs)
    if ready < N:
        steps = m.one_token([o[-1] for o in outs], [S + len(o) - 1 for o in outs], N - ready)
        out.extend(drain_one_token(outs, N, steps))
    return out, m.calls


@pytest.mark.parametrize("seed", range(6))
@pytest.mark.parametrize("breakeven", [0.0, 1.5, 100.0])
def test_speculative_tokens_equal_plain_greedy(seed, breakeven):
    rng = random.Random(seed)
    B, S, N = rng.choice([1, 3, 8]), rng.choice([2, 5, 17]), rng.choice([3, 9, 40])
    K = draft_len(B)
    prompts = [[rng.randrange(V) for _ in range(S)] for _ in range(B)]
    out, calls = run(prompts, N, K, breakeven)
    assert len(out) == N and all(len(step) == B for step in out)
    want = [greedy(p, N) for p in prompts]
    assert [[step[b] for step in out] for b in range(B)] == want
    if breakeven == 100.0 and N > 1:
        assert calls <= 8                     # stopped at the first break-even check


def test_speculation_saves_forwards_on_a_looping_model():
    rng = random.Random(1)
    prompts = [[rng.randrange(V) for _ in range(6)] for _ in range(2)]
    N = 64
    out, calls = run(prompts, N, draft_len(2), breakeven=0.0)
    assert calls < N - 1, calls              # several tokens per verify forward on average


def test_lookup_drafts_the_latest_continuation_longest_ngram_first():
    lk = Lookup([1, 2, 3, 9, 1, 2, 3, 4, 5, 2, 3])
    # the last trigram "5 2 3" has not occurred before; the bigram "2 3" was last continued at
    # index 7 (token 4): draft 4 5 2 3
    assert lk.draft(4) == [4, 5, 2, 3]
    lk.append([4])
    assert lk.draft(2) == [5, 2]             # trigram "2 3 4" -> 5
    assert Lookup([7]).draft(3) == [7, 7, 7]
    loop = Lookup([1, 2, 1, 2])
    assert loop.draft(5) == [1, 2, 1, 2, 1]  # the continuation runs into the draft itself


def test_accept_takes_the_agreeing_prefix_and_one_more():
    assert accept([5, 6, 7], [5, 6, 9, 1]) == [5, 6, 9]
    assert accept([5, 6, 7], [4, 6, 7, 1]) == [4]
    assert accept([5, 6, 7], [5, 6, 7, 1]) == [5, 6, 7, 1]
    assert accept([], [3]) == [3]


def test_draft_len_follows_the_batch():
    assert [draft_len(b) for b in (1, 4, 5, 16, 17, 32, 33, 64)] == [6, 6, 4, 4, 2, 2, 0, 0]
