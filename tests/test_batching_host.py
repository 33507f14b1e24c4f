"""The continuous-batching scheduler's host logic (batching.ContinuousBatcher) on a stand-in engine:
every request gets its tokens, a sequence's positions advance by one per step from its prompt length,
no more sequences run than there are slots, freed slots take queued requests at once, and each step
feeds every active sequence its own last token. The stand-in's next token depends only on (slot's
request, position, input token), so a mix-up of rows would show. No GPU needed."""
import batching


class FakeEngine:
    V = 1000

    def __init__(self):
        self.slots = 0
        self.owner = {}  # slot -> prompt of the sequence in it
        self.max_rows = 0

    def set_slots(self, n):
        self.slots = n
        return 0

    def next_tok(self, prompt, pos, tok):
        return (sum(prompt) * 7 + pos * 13 + tok * 3) % self.V

    def prefill_slot(self, slot, prompt, n_batch):
        assert 0 <= slot < self.slots
        self.owner[slot] = list(prompt)
        return 0, self.next_tok(prompt, len(prompt) - 1, prompt[-1])

    def step_slots(self, slots, pos, toks):
        assert len(set(slots)) == len(slots) <= self.slots
        self.max_rows = max(self.max_rows, len(slots))
        return 0, [self.next_tok(self.owner[s], p, t) for s, p, t in zip(slots, pos, toks)]


def alone(e, prompt, n_gen):
    toks = [e.next_tok(prompt, len(prompt) - 1, prompt[-1])]
    pos = len(prompt)
    while len(toks) < n_gen:
        toks.append(e.next_tok(prompt, pos, toks[-1]))
        pos += 1
    return toks


def test_scheduler_matches_sequences_run_alone():
    e = FakeEngine()
    b = batching.ContinuousBatcher(e, n_slots=3)
    reqs = [b.submit([i + 1] * (3 + 2 * i), n_gen=2 + (5 * i) % 9) for i in range(8)]
    b.run()
    assert e.max_rows <= 3
    for r in reqs:
        assert r.tokens == alone(e, r.prompt, r.n_gen)
    assert b.rows == sum(r.n_gen - 1 for r in reqs)  # every token after the first came from a step
    assert not b.active and not b.queue


def test_scheduler_admits_into_freed_slots():
    e = FakeEngine()
    b = batching.ContinuousBatcher(e, n_slots=2)
    short = b.submit([5, 6], n_gen=2)
    long_ = b.submit([7, 8, 9], n_gen=6)
    late = b.submit([1], n_gen=3)
    b.step()  # both admitted; the short one finishes after this step
    assert short.slot in (0, 1) and late.slot == -1
    b.step()  # the freed slot takes the queued request
    assert late.slot == short.slot
    b.run()
    assert late.tokens == alone(e, late.prompt, 3) and long_.tokens == alone(e, long_.prompt, 6)
