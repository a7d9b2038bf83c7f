"""Continuously batched request serving over the batch-B decode context.

The reference's OpenAI-style server (api_server.py) decodes one request at a
time: a global lock (api_server.py:40) serialises requests, each request
prefills its prompt into a private B = 1 KV cache and then runs the decode
step token by token (api_server.py:58-150).  Here up to ``batch`` requests
share one decode step: every row of the batch-B context is a slot holding one
request with its own position (``r4q_decode_step_rows``), a new request is
admitted into a free slot between steps (its prompt is prefilled straight
into that slot's rows of the KV caches), and a finished request frees its
slot for the next one.  Per-token sampling follows the reference: greedy at
temperature 0, else temperature + nucleus (top-p) sampling
(api_server.py:80-91).

This is the surface only (no HTTP, no tokenizer): requests are token-id
lists; the server holds no lock of its own beyond ``BatchedEngine.lock`` around
a step.  The model is the dict of per-layer tensors the decode runtime takes
(``r4q.synth.build_decode_model`` or ``r4q.loader``) with KV caches of batch
dimension ``batch``."""
from __future__ import annotations

import itertools
import threading
from dataclasses import dataclass, field
from typing import Callable, Optional, Sequence

import torch

from . import decode
from . import prefill as P

_ids = itertools.count(1)


@dataclass
class Request:
    """One generation request.  ``tokens`` collects the generated ids;
    ``finish_reason`` is None while running, then "stop" (a stop id was
    sampled, and is kept as the last token, as the reference keeps EOS),
    "length" (max_new_tokens reached) or "cache" (the KV cache is full)."""
    prompt: Sequence[int]
    max_new_tokens: int = 64
    stop_ids: Sequence[int] = ()
    temperature: float = 0.0
    top_p: float = 1.0
    seed: Optional[int] = None
    id: int = field(default_factory=lambda: next(_ids))
    tokens: list = field(default_factory=list)
    finish_reason: Optional[str] = None
    on_token: Optional[Callable[["Request", int], None]] = None

    @property
    def done(self) -> bool:
        return self.finish_reason is not None


def sample(logits: torch.Tensor, temperature: float, top_p: float,
           gen: Optional[torch.Generator]) -> int:
    """Next id from one row of logits: argmax (first maximum) at temperature
    0, else softmax(logits / temperature) restricted to the smallest set of
    most likely ids whose probability reaches top_p (an id is dropped when the
    mass of the ids ranked above it already reaches top_p)."""
    if temperature <= 0:
        return int(torch.argmax(logits))
    z = logits.float() / temperature
    if top_p < 1.0:
        zs, order = torch.sort(z, descending=True)
        p = torch.softmax(zs, dim=-1)
        above = torch.cumsum(p, dim=-1) - p
        zs = zs.masked_fill(above >= top_p, float("-inf"))
        z = torch.full_like(z, float("-inf")).scatter(0, order, zs)
    probs = torch.softmax(z, dim=-1)
    return int(torch.multinomial(probs, 1, generator=gen))


class SlotBackend:
    """The model side of the engine: prefill of one prompt into a slot and the
    batched decode step.  Separate from the scheduling so the scheduler can
    be driven by a stand-in (tests on CPU)."""

    def __init__(self, model: dict, cfg: dict, batch: int, use_graph: bool = True):
        self.m, self.cfg, self.batch, self.use_graph = model, cfg, int(batch), use_graph
        kc = model['k_caches'][0]
        if kc.shape[0] != self.batch:
            raise ValueError(f"KV caches have batch {kc.shape[0]}, engine batch {batch}")
        self.max_seq = int(kc.shape[2])
        self.vocab = int(cfg['vocab'])
        self.dev = kc.device
        m = model
        self.ctx = decode.get_context(
            m['qkv_w'], m['qkv_s'], m['o_w'], m['o_s'], m['gu_w'], m['gu_s'], m['down_w'], m['down_s'],
            m['in_norm_w'], m['post_norm_w'], m['q_norm_w'], m['k_norm_w'], m['rope_cos'], m['rope_sin'],
            cfg['num_heads'], cfg['num_kv_heads'], cfg['head_dim'], cfg['hidden'], cfg['intermediate'],
            cfg['rms_eps'], m['k_caches'], m['v_caches'], m['final_norm_w'], m['lm_w'], m['lm_s'],
            self.vocab, batch=self.batch)
        self.logits = torch.empty(self.batch, self.vocab, dtype=torch.float16, device=self.dev)
        self.hidden = torch.zeros(self.batch, cfg['hidden'], dtype=torch.float16, device=self.dev)

    def prefill(self, slot: int, prompt: Sequence[int]) -> torch.Tensor:
        """Writes the prompt's K/V into row ``slot`` at positions 0..M-1 and
        returns the last position's logits [vocab]."""
        m, c = self.m, self.cfg
        ids = torch.as_tensor(list(prompt), dtype=torch.long, device=self.dev)
        h = m['embed'][ids]
        lg = P.prefill_logits(h, m['qkv_w'], m['qkv_s'], m['o_w'], m['o_s'], m['gu_w'], m['gu_s'],
                              m['down_w'], m['down_s'], m['in_norm_w'], m['post_norm_w'], m['q_norm_w'],
                              m['k_norm_w'], m['rope_cos'], m['rope_sin'], c['num_heads'], c['num_kv_heads'],
                              c['head_dim'], c['hidden'], c['intermediate'], c['rms_eps'], m['final_norm_w'],
                              m['lm_w'], m['lm_s'], self.vocab, k_caches=m['k_caches'],
                              v_caches=m['v_caches'], batch_row=slot, last_only=True)
        return lg.reshape(-1)

    def step(self, tokens: Sequence[int], positions: Sequence[int]) -> torch.Tensor:
        """One decode step of every row: row b takes token tokens[b] at
        positions[b]; returns the logits [batch, vocab] (device)."""
        ids = torch.as_tensor(list(tokens), dtype=torch.long, device=self.dev)
        torch.index_select(self.m['embed'], 0, ids, out=self.hidden)
        self.ctx.step_rows(self.hidden, positions, logits_out=self.logits, use_graph=self.use_graph)
        return self.logits


class BatchedEngine:
    """Slots, admission and retirement around a backend (``SlotBackend``).

    ``submit`` queues a request (FIFO); ``step`` admits queued requests into
    free slots (prefill + first token), then runs one batched decode step for
    the occupied slots and samples each row's next token; ``run`` steps until
    every submitted request is done.  Idle slots ride along in the batch at
    position 0 of their own cache rows (the next prefill into the slot
    overwrites them)."""

    def __init__(self, backend, batch: Optional[int] = None):
        self.be = backend
        self.batch = int(batch if batch is not None else backend.batch)
        self.max_seq = backend.max_seq
        self.slots: list = [None] * self.batch       # Request or None
        self.pos = [0] * self.batch                  # position of the slot's next token
        self.next_tok = [0] * self.batch
        self.gens: dict = {}
        self.queue: list = []
        self.lock = threading.Lock()
        self.steps = 0

    def submit(self, prompt: Sequence[int], **kw) -> Request:
        r = Request(prompt=list(prompt), **kw)
        if len(r.prompt) < 1:
            raise ValueError("empty prompt")
        if len(r.prompt) >= self.max_seq:
            raise ValueError(f"prompt of {len(r.prompt)} tokens does not fit the KV cache ({self.max_seq})")
        if r.max_new_tokens < 1:
            raise ValueError("max_new_tokens must be >= 1")
        with self.lock:
            self.queue.append(r)
        return r

    def _gen(self, r: Request):
        if r.temperature <= 0:
            return None
        g = self.gens.get(r.id)
        if g is None:
            g = torch.Generator(device=self.be.logits.device if hasattr(self.be, 'logits') else 'cpu')
            g.manual_seed(r.seed if r.seed is not None else r.id)
            self.gens[r.id] = g
        return g

    def _emit(self, slot: int, r: Request, tok: int):
        r.tokens.append(tok)
        if r.on_token is not None:
            r.on_token(r, tok)
        if tok in r.stop_ids:
            r.finish_reason = "stop"
        elif len(r.tokens) >= r.max_new_tokens:
            r.finish_reason = "length"
        elif self.pos[slot] >= self.max_seq:
            r.finish_reason = "cache"
        if r.done:
            self.slots[slot] = None
            self.gens.pop(r.id, None)
            self.pos[slot] = 0
            self.next_tok[slot] = 0
        else:
            self.next_tok[slot] = tok

    def _admit(self):
        for s in range(self.batch):
            if self.slots[s] is None and self.queue:
                r = self.queue.pop(0)
                self.slots[s] = r
                lg = self.be.prefill(s, r.prompt)
                self.pos[s] = len(r.prompt)
                self._emit(s, r, sample(lg, r.temperature, r.top_p, self._gen(r)))

    @property
    def active(self) -> int:
        return sum(r is not None for r in self.slots)

    def step(self) -> int:
        """Admit, then one decode step; returns the number of rows decoded."""
        with self.lock:
            self._admit()
            rows = [s for s in range(self.batch) if self.slots[s] is not None]
            if not rows:
                return 0
            logits = self.be.step(self.next_tok, self.pos)
            greedy = [s for s in rows if self.slots[s].temperature <= 0]
            if greedy:
                am = torch.argmax(logits[greedy], dim=-1).tolist()
            picks = dict(zip(greedy, am)) if greedy else {}
            for s in rows:
                r = self.slots[s]
                tok = picks[s] if s in picks else sample(logits[s], r.temperature, r.top_p, self._gen(r))
                self.pos[s] += 1
                self._emit(s, r, tok)
            self.steps += 1
            return len(rows)

    def run(self, max_steps: Optional[int] = None) -> None:
        n = 0
        while self.queue or self.active:
            self.step()
            n += 1
            if max_steps is not None and n >= max_steps:
                break

    def generate(self, prompts: Sequence[Sequence[int]], **kw) -> list:
        """Submits every prompt, runs to completion, returns the Requests."""
        reqs = [self.submit(p, **kw) for p in prompts]
        self.run()
        return reqs
