"""The batched step driver (pageserve_b200/runner.py) against the reference's
own continuous batching, on CPU.

tests/golden/sched_trace.npz holds a run of the reference's unmodified
Scheduler + ContinuousBatchingRunner (engine/scheduler.py:77-119,
engine/runner.py:55-83) over a pool small enough to chunk prefills, stall a
sequence and preempt one for recompute, with a deterministic fake model. A
replay scheduler re-issues the reference's recorded decisions (entries, block
tables, preemption resets); BatchedRunner drives them with one batched call
per step. Every entry's (input_ids, block_table, start_pos) must equal the
reference runner's process_chunk call, step by step, and every sequence must
end with the reference's output tokens."""

from pathlib import Path

import numpy as np

import cases
from pageserve_b200.runner import BatchedRunner, BatchPlan, chunk_inputs, plan_batch, snapshot

GOLDEN = Path(__file__).resolve().parent / "golden"


class _Status:
    def __init__(self, name):
        self.name = name


class _Seq:
    """The Sequence fields the runner reads (engine/sequence.py:18-40)."""

    def __init__(self, sid, prompt, max_new):
        self.seq_id = sid
        self.prompt_tokens = [int(t) for t in prompt]
        self.max_new_tokens = max_new
        self.output_tokens = []
        self.block_table = []
        self.num_prompt_tokens_processed = 0
        self.status = _Status("RUNNING")

    @property
    def prompt_len(self):
        return len(self.prompt_tokens)


class _Entry:
    def __init__(self, seq, chunk, produces_token):
        self.seq, self.chunk, self.produces_token = seq, chunk, produces_token


class ReplayScheduler:
    """Re-issues the reference scheduler's recorded steps."""

    def __init__(self, g, seqs):
        self.g, self.seqs = g, seqs
        self.k = 0
        self.n = int(g["n_steps"])
        self.ci = 0
        self.calls = [(g[f"call{j}/ids"].tolist(), g[f"call{j}/table"].tolist(), *g[f"call{j}/meta"].tolist())
                      for j in range(int(g["n_calls"]))]
        self.snapshots_seen = []

    @property
    def running(self):
        snap = self.g[f"{self.k}/snapshot"]
        self.snapshots_seen.append(snap.tolist())
        for sid, done, nout in snap.tolist():  # the replay reproduces the reference's pre-step state
            s = self.seqs[sid]
            assert (s.num_prompt_tokens_processed, len(s.output_tokens)) == (done, nout), (self.k, sid)
        return [self.seqs[sid] for sid, _, _ in snap.tolist()]

    def has_work(self):
        return self.k < self.n

    def add_request(self, seq):
        pass

    def step(self):
        out = []
        for sid, chunk, prod in self.g[f"{self.k}/entries"].tolist():
            s = self.seqs[sid]
            ids, table, start, _tok, k = self.calls[self.ci]
            assert k == self.k
            self.ci += 1
            if start == 0 and start < s.prompt_len and (s.output_tokens or s.num_prompt_tokens_processed):
                s.output_tokens = []  # preempted earlier: recompute from scratch (engine/sequence.py:55-68)
                s.num_prompt_tokens_processed = 0
            s.block_table = list(table)
            if s.num_prompt_tokens_processed < s.prompt_len:
                s.num_prompt_tokens_processed += chunk
            out.append(_Entry(s, chunk, bool(prod)))
        self.k += 1
        return out

    def append_token(self, seq, tok):
        seq.output_tokens.append(tok)
        if len(seq.output_tokens) >= seq.max_new_tokens:
            seq.status = _Status("FINISHED")


def _load():
    g = np.load(GOLDEN / "sched_trace.npz")
    spec = cases.SCHED_TRACE
    seqs = [_Seq(i, p, n) for i, (p, n) in enumerate(zip(cases.sched_trace_prompts(), spec["max_new"]))]
    return g, seqs


def test_batched_runner_reproduces_reference_runner_calls():
    g, seqs = _load()
    sched = ReplayScheduler(g, seqs)
    plans: list[BatchPlan] = []

    def process_batch(plan):
        plans.append(plan)
        return [cases.fake_next_token(*plan.chunk(i)[::2]) for i in range(len(plan))]

    runner = BatchedRunner(sched, process_batch)
    for s in seqs:
        runner.wait_until_finished(s, timeout=30)
    runner.stop()
    assert runner.error is None
    calls = [(g[f"call{j}/ids"].tolist(), g[f"call{j}/table"].tolist(), int(g[f"call{j}/meta"][0]))
             for j in range(int(g["n_calls"]))]
    got = [plan.chunk(i) for plan in plans for i in range(len(plan))]
    assert got == calls, "per-entry (input_ids, block_table, start_pos) differ from the reference runner's calls"
    assert [len(p) for p in plans] == [len(g[f"{k}/entries"]) for k in range(int(g["n_steps"]))]
    for i, s in enumerate(seqs):
        assert s.output_tokens == g[f"out{i}"].tolist(), f"sequence {i}"


def test_plan_batch_concatenates_in_entry_order():
    a, b = _Seq(0, [5, 6, 7, 8], 4), _Seq(1, [9, 10], 4)
    a.block_table, b.block_table = [3, 1], [2]
    b.output_tokens = [44, 45]
    b.num_prompt_tokens_processed = 2
    plan = plan_batch([_Entry(a, 3, False), _Entry(b, 1, True)], {0: 0, 1: 2}, {0: 0, 1: 1})
    assert plan.input_ids == [5, 6, 7, 45] and plan.q_lens == [3, 1]
    assert plan.start_pos == [0, 2 + 1 - 1] and plan.block_tables == [[3, 1], [2]]
    assert chunk_inputs(a, 2, 3, 0) == ([8], 3)  # a short last prompt chunk
    prompt, out = snapshot(type("S", (), {"running": [a, b]})())
    assert prompt == {0: 0, 1: 2} and out == {0: 0, 1: 2}


def test_runner_surfaces_a_failing_model_call():
    g, seqs = _load()

    def broken(plan):
        raise ValueError("model failed")

    runner = BatchedRunner(ReplayScheduler(g, seqs), broken)
    try:
        runner.wait_until_finished(seqs[0], timeout=10)
        raise AssertionError("expected the model error")
    except RuntimeError as e:
        assert isinstance(e.__cause__, ValueError)
    runner.stop()
