"""Scheduling of the continuously batched server (r4q.serve) on CPU, driven by
a stand-in backend whose logits are a known function of (token, position):
admission order, per-slot positions, stop / length / cache-limit retirement,
slot reuse, and the sampler's greedy / top-p rules (api_server.py:80-91)."""
import pytest
import torch

from r4q import serve

V = 97


class FakeBackend:
    """Row b at position p with token t: logits peak at (3 t + p) % V.
    Records every call so the test can check what the engine asked for."""

    def __init__(self, batch, max_seq):
        self.batch, self.max_seq = batch, max_seq
        self.logits = torch.zeros(batch, V)
        self.calls = []
        self.prefills = []

    @staticmethod
    def nxt(tok, pos):
        return (3 * tok + pos) % V

    def prefill(self, slot, prompt):
        self.prefills.append((slot, list(prompt)))
        lg = torch.zeros(V)
        lg[self.nxt(sum(prompt), len(prompt) - 1)] = 5.0
        return lg

    def step(self, tokens, positions):
        self.calls.append((list(tokens), list(positions)))
        self.logits.zero_()
        for b in range(self.batch):
            self.logits[b, self.nxt(tokens[b], positions[b])] = 5.0
        return self.logits


def expected(prompt, n, max_seq, stop=()):
    """The tokens one request gets when decoded alone."""
    toks = [FakeBackend.nxt(sum(prompt), len(prompt) - 1)]
    pos = len(prompt)
    while len(toks) < n and toks[-1] not in stop and pos < max_seq:
        toks.append(FakeBackend.nxt(toks[-1], pos))
        pos += 1
    return toks


def test_more_requests_than_slots_each_matches_alone():
    be = FakeBackend(batch=3, max_seq=64)
    eng = serve.BatchedEngine(be)
    prompts = [[1, 2, 3], [4], [5, 6, 7, 8, 9], [10, 11], [12], [13, 14, 15, 16], [17, 18, 19]]
    lens = [5, 2, 9, 4, 7, 3, 6]
    reqs = [eng.submit(p, max_new_tokens=n) for p, n in zip(prompts, lens)]
    eng.run()
    for r, p, n in zip(reqs, prompts, lens):
        assert r.tokens == expected(p, n, 64), r.id
        assert r.finish_reason == "length"
    # FIFO admission: the first three fill slots 0..2 in order
    assert [s for s, _ in be.prefills[:3]] == [0, 1, 2]
    assert [p for _, p in be.prefills] == prompts
    # never more rows than slots, and the batch stayed full while work remained
    assert all(len(t) == 3 for t, _ in be.calls)
    assert eng.active == 0 and not eng.queue


def test_positions_are_per_row():
    be = FakeBackend(batch=2, max_seq=64)
    eng = serve.BatchedEngine(be)
    eng.submit([1, 1, 1, 1, 1], max_new_tokens=3)
    eng.submit([2], max_new_tokens=3)
    eng.step()
    toks, pos = be.calls[0]
    assert pos == [5, 1]                       # each row decodes right after its own prompt


def test_stop_id_and_cache_limit():
    be = FakeBackend(batch=2, max_seq=8)
    eng = serve.BatchedEngine(be)
    p = [3, 4]
    alone = expected(p, 50, 8)
    stop_tok = alone[2]
    r1 = eng.submit(p, max_new_tokens=50, stop_ids=[stop_tok])
    r2 = eng.submit([9, 9, 9], max_new_tokens=50)
    eng.run()
    assert r1.finish_reason == "stop" and r1.tokens == alone[:alone.index(stop_tok) + 1]
    # 3 prompt positions + the generated ones: the last decode runs at max_seq - 1
    assert r2.finish_reason == "cache" and r2.tokens == expected([9, 9, 9], 50, 8)
    assert len(r2.tokens) == 8 - 3 + 1


def test_slot_reuse_resets_position():
    be = FakeBackend(batch=1, max_seq=32)
    eng = serve.BatchedEngine(be)
    a = eng.submit([1, 2, 3, 4], max_new_tokens=2)
    b = eng.submit([7], max_new_tokens=3)
    eng.run()
    assert a.tokens == expected([1, 2, 3, 4], 2, 32) and b.tokens == expected([7], 3, 32)
    assert [pos for _, pos in be.calls] == [[4], [1], [2]]


def test_on_token_streams_in_order():
    be = FakeBackend(batch=2, max_seq=32)
    eng = serve.BatchedEngine(be)
    seen = []
    r = eng.submit([5, 5], max_new_tokens=4, on_token=lambda req, t: seen.append(t))
    eng.run()
    assert seen == r.tokens


def test_submit_rejects_bad_requests():
    eng = serve.BatchedEngine(FakeBackend(batch=1, max_seq=8))
    with pytest.raises(ValueError):
        eng.submit([], max_new_tokens=2)
    with pytest.raises(ValueError):
        eng.submit(list(range(8)), max_new_tokens=2)
    with pytest.raises(ValueError):
        eng.submit([1], max_new_tokens=0)


def test_sampler_greedy_and_nucleus():
    lg = torch.tensor([0.0, 3.0, 1.0, 3.0, -2.0])
    assert serve.sample(lg, 0.0, 1.0, None) == 1            # first maximum
    # top_p below the top probability keeps only the first maximum's tie set
    # member ranked first by the sort; with distinct logits it is the argmax
    lg2 = torch.tensor([0.0, 5.0, 1.0, 2.0])
    g = torch.Generator().manual_seed(0)
    assert all(serve.sample(lg2, 1.0, 0.5, g) == 1 for _ in range(50))
    # top_p = 1: every id with positive probability can appear, frequencies
    # follow softmax(lg / T)
    g = torch.Generator().manual_seed(1)
    lg3 = torch.tensor([1.0, 0.0, 0.5])
    n = 4000
    cnt = torch.bincount(torch.tensor([serve.sample(lg3, 0.7, 1.0, g) for _ in range(n)]), minlength=3)
    p = torch.softmax(lg3 / 0.7, 0)
    assert torch.allclose(cnt.float() / n, p, atol=0.03)
    # nucleus: ids whose higher-ranked mass already reaches top_p never appear
    probs = torch.softmax(lg3, 0)                            # T = 1: [0.51, 0.19, 0.31]
    g = torch.Generator().manual_seed(2)
    got = {serve.sample(lg3, 1.0, 0.6, g) for _ in range(500)}
    assert got == {0, 2} and probs[0] < 0.6
