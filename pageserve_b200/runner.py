"""Batched step driver for the reference's continuous-batching scheduler.

The reference's runner (engine/runner.py:55-83) takes one ``Scheduler.step()``
batch (engine/scheduler.py:77-119: prefill chunks and decode tokens of many
sequences) and calls ``process_chunk(input_ids, block_table, start_pos)``
once per entry, each a full model pass (server.py:43-47: ``forward_step`` then
``int(logits[-1].argmax())``, a host sync per sequence). Here the same batch is
one ``PagedCausalLM.forward_batch`` — every entry's chunk concatenated, the
block tables packed once, one greedy token per sequence read back in one copy.

* :func:`plan_batch` turns a scheduler batch into the batched call's inputs,
  choosing each entry's tokens and start position exactly as
  engine/runner.py:65-77 does (prompt chunk while prefill is incomplete, else
  the last sampled token at ``prompt_len + outputs - 1``).
* :func:`make_process_batch` binds a model: plan -> next token per entry.
* :func:`make_process_chunk` is the reference's per-chunk callback on this
  build's kernels (the drop-in for server.py's ``_process_chunk``).
* :class:`BatchedRunner` has ContinuousBatchingRunner's interface (``submit``,
  ``wait_until_finished``, ``stop``) and drives one batched call per step.
"""

from __future__ import annotations

import threading
from dataclasses import dataclass, field
from typing import Callable

import numpy as np


@dataclass
class BatchPlan:
    """Inputs of one batched step, in the scheduler's entry order."""
    entries: list = field(default_factory=list)   # the scheduler's BatchEntry objects
    input_ids: list[int] = field(default_factory=list)   # every entry's chunk, concatenated
    q_lens: list[int] = field(default_factory=list)
    start_pos: list[int] = field(default_factory=list)
    block_tables: list[list[int]] = field(default_factory=list)

    def __len__(self) -> int:
        return len(self.entries)

    def chunk(self, i: int) -> tuple[list[int], list[int], int]:
        """(input_ids, block_table, start_pos) of entry i: the arguments the
        reference runner passes to process_chunk."""
        a = sum(self.q_lens[:i])
        return self.input_ids[a:a + self.q_lens[i]], self.block_tables[i], self.start_pos[i]


def snapshot(scheduler) -> tuple[dict, dict]:
    """Per running sequence, prompt tokens processed and outputs sampled,
    taken before ``scheduler.step()`` (engine/runner.py:61-64)."""
    prompt = {s.seq_id: s.num_prompt_tokens_processed for s in scheduler.running}
    out = {s.seq_id: len(s.output_tokens) for s in scheduler.running}
    return prompt, out


def chunk_inputs(seq, chunk: int, before_prompt: int, before_output_len: int) -> tuple[list[int], int]:
    """engine/runner.py:69-77: the tokens an entry feeds and their start
    position. While the prompt is incomplete, the next ``chunk`` prompt tokens
    at ``before_prompt``; else the most recently sampled token, whose cache
    position is one behind the output count."""
    if before_prompt < seq.prompt_len:
        return list(seq.prompt_tokens[before_prompt:before_prompt + chunk]), before_prompt
    return [seq.output_tokens[-1]], seq.prompt_len + before_output_len - 1


def plan_batch(batch, prev_prompt: dict, prev_out: dict) -> BatchPlan:
    plan = BatchPlan()
    for entry in batch:
        s = entry.seq
        ids, start = chunk_inputs(s, entry.chunk, prev_prompt.get(s.seq_id, 0), prev_out.get(s.seq_id, 0))
        plan.entries.append(entry)
        plan.input_ids.extend(int(t) for t in ids)
        plan.q_lens.append(len(ids))
        plan.start_pos.append(int(start))
        plan.block_tables.append(list(s.block_table))
    return plan


ProcessBatch = Callable[[BatchPlan], list[int]]


def make_process_batch(model) -> ProcessBatch:
    """plan -> greedy next token of every entry (one forward_batch, one
    device->host copy of the tokens)."""
    def process_batch(plan: BatchPlan) -> list[int]:
        if not len(plan):
            return []
        _, nxt = model.forward_batch(np.asarray(plan.input_ids, np.int64), plan.q_lens, plan.start_pos,
                                     plan.block_tables, return_logits=False)
        return nxt.cpu().tolist()
    return process_batch


def make_process_chunk(model) -> Callable[[list[int], list[int], int], int]:
    """The reference's per-entry callback (server.py:43-47:
    forward_step, then the argmax of the last row) on this build's kernels;
    the argmax runs on the device."""
    import torch

    def process_chunk(input_ids: list[int], block_table: list[int], start_pos: int) -> int:
        logits = model.forward_step(torch.as_tensor(input_ids, dtype=torch.int64), block_table, start_pos)
        return int(model.argmax(logits[-1:])[0])
    return process_chunk


class BatchedRunner:
    """engine/runner.py:20-83 with one batched model call per scheduler step.

    One daemon thread loops: snapshot + ``scheduler.step()`` under the lock,
    the batched call outside it, then ``append_token`` for the entries that
    produce a token (in entry order, under the lock). Callers ``submit`` a
    Sequence and ``wait_until_finished``."""

    def __init__(self, scheduler, process_batch: ProcessBatch):
        self.scheduler = scheduler
        self.process_batch = process_batch
        self.lock = threading.Lock()
        self.cv = threading.Condition(self.lock)
        self._stop = False
        self.steps = 0
        self.error: BaseException | None = None
        self.thread = threading.Thread(target=self._loop, daemon=True)
        self.thread.start()

    def submit(self, seq) -> None:
        with self.cv:
            self.scheduler.add_request(seq)
            self.cv.notify_all()

    def wait_until_finished(self, seq, timeout: float | None = None) -> None:
        with self.cv:
            done = self.cv.wait_for(lambda: self._is_finished(seq) or self.error is not None, timeout=timeout)
        if self.error is not None:
            raise RuntimeError("the batched runner stopped on an error") from self.error
        if not done:
            raise TimeoutError(f"sequence {seq.seq_id} did not finish within {timeout}s")

    def stop(self) -> None:
        with self.cv:
            self._stop = True
            self.cv.notify_all()
        self.thread.join(timeout=10)

    @staticmethod
    def _is_finished(seq) -> bool:
        """seq.status is SeqStatus.FINISHED (engine/sequence.py:8-11)."""
        return getattr(seq.status, "name", None) == "FINISHED"

    def _loop(self) -> None:
        try:
            while True:
                with self.cv:
                    while not self._stop and not self.scheduler.has_work():
                        self.cv.wait()
                    if self._stop:
                        return
                    prev_prompt, prev_out = snapshot(self.scheduler)
                    batch = self.scheduler.step()
                plan = plan_batch(batch, prev_prompt, prev_out)
                tokens = self.process_batch(plan) if len(plan) else []
                with self.cv:
                    self.steps += 1
                    for entry, tok in zip(plan.entries, tokens):
                        if entry.produces_token:
                            self.scheduler.append_token(entry.seq, int(tok))
                    self.cv.notify_all()
        except BaseException as e:  # surface to waiters instead of dying silently
            with self.cv:
                self.error = e
                self.cv.notify_all()

