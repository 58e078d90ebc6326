"""End-to-end decode timing on a Qwen2 runner. Public names and timing semantics follow the
reference's kernels/e2e/run.py (without the HF download, perplexity and chat prompts, which need the
network); the implementation is this package's own.

- `GraphDecoder`: greedy decoding with one captured CUDA graph per token step (reference
  run.py:58-111), for batch 1 or more. The step itself is `QwenRunner.greedy_step`, which the fused
  backends run as a single decode-step kernel.
- `decode_speed`: median tok/s over repeated generations (reference run.py:114-122).
- `prefill_speed`, `layers_only_ms`: reference run.py:142-201.
- `GraphDecoder.step_host`: the per-token API of a server loop - the token comes from pinned host
  memory, the graph runs, the next token is read back to the host.
- `greedy_parity`: the reference's parity figures (run.py:289-303) between two runners - max |logit
  diff| and the first greedy divergence - for batch-1 synthetic prompts.
"""

from __future__ import annotations

import statistics
from collections.abc import Callable

import torch

from kernels.bench.harness import capture
from kernels.e2e.model import QwenRunner


def _device_seconds(work: Callable[[], None]) -> float:
    """Seconds `work()` takes on the current stream, by CUDA events."""
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    work()
    t1.record()
    t1.synchronize()
    return t0.elapsed_time(t1) / 1e3


def _replay(graph, times: int) -> Callable[[], None]:
    def run():
        for _ in range(times):
            graph.replay()

    return run


class GraphDecoder:
    """Greedy decoding, one CUDA graph per token step.

    Device state: `tok` [B, 1], the token the next step consumes; `pos` [1], its position; `out`
    [B, max_len], the greedy token chosen at each position. A step (`QwenRunner.greedy_step`) feeds
    `tok` at `pos`, stores the pick in `out[:, pos]`, makes it the next `tok` and advances `pos`, all on
    the device, so the graph captured once replays for every token.
    """

    WARM_STEPS = 3

    def __init__(self, runner: QwenRunner):
        self.r = runner
        dev = runner.embed.device
        rows = runner.batch
        self.tok = torch.zeros(rows, 1, dtype=torch.long, device=dev)
        self.pos = torch.zeros(1, dtype=torch.long, device=dev)
        self.out = torch.zeros(rows, runner.max_len, dtype=torch.long, device=dev)
        self.graph = None
        self.host_tok = torch.zeros(rows, 1, dtype=torch.long).pin_memory()
        self.host_next = torch.zeros(rows, 1, dtype=torch.long).pin_memory()

    def _step(self):
        self.r.greedy_step(self.tok, self.pos, self.out)

    def prefill(self, ids: torch.Tensor) -> int:
        """Run the prompt ids [B, P] (on the device) through the model: fills the KV cache, and the
        first generated token becomes `tok` at position P (also recorded at out[:, P - 1])."""
        n = ids.shape[1]
        first = self.r.greedy(self.r.forward(ids, torch.arange(n, device=ids.device)))
        self.out.zero_()
        self.out[:, n - 1] = first
        self.tok[:, 0] = first
        self.pos.fill_(n)
        return n

    def capture(self, ids):
        """Warm up (kernel choices and library loads happen outside the graph), then capture one
        step from the state right after the prompt."""
        self.prefill(ids)
        self._step()
        torch.cuda.synchronize()
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for _ in range(self.WARM_STEPS):
                self._step()
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        self.prefill(ids)
        self.graph, _ = capture(self._step)
        torch.cuda.synchronize()

    def generate(self, ids, steps: int) -> tuple[list, float]:
        """(tokens [B][steps + 1] from the first generated one on, device seconds of the steps)."""
        n = self.prefill(ids)
        torch.cuda.synchronize()
        sec = _device_seconds(_replay(self.graph, steps))
        return self.out[:, n - 1: n + steps].tolist(), sec

    def step_host(self, token_host: torch.Tensor) -> torch.Tensor:
        """One token through the public API from host memory: pinned host -> device copy of the
        token, one graph replay, device -> pinned host copy of the next token, host wait."""
        self.host_tok.copy_(token_host)
        self.tok.copy_(self.host_tok, non_blocking=True)
        self.graph.replay()
        self.host_next.copy_(self.tok, non_blocking=True)
        torch.cuda.current_stream().synchronize()
        return self.host_next


def decode_speed(runner, ids, steps: int, repeats: int = 3) -> dict:
    """Batch x steps / device time of `steps` graph-replayed greedy steps; median over `repeats`."""
    dec = GraphDecoder(runner)
    dec.capture(ids)
    rows = runner.batch
    rates = sorted(rows * steps / dec.generate(ids, steps)[1] for _ in range(repeats))
    mid = statistics.median(rates)
    return {"tok_s": mid, "tok_s_min": rates[0], "tok_s_max": rates[-1], "ms_per_step": 1e3 * rows / mid,
            "steps": steps, "batch": rows}


def _graph_median_seconds(body: Callable, warm: int, samples: int, replays: int = 1) -> float:
    """Median device seconds of one call of `body`, captured in a graph after `warm` eager calls."""
    for _ in range(warm):
        body()
    torch.cuda.synchronize()
    graph, _ = capture(body)
    try:
        graph.replay()
        torch.cuda.synchronize()
        return statistics.median(_device_seconds(_replay(graph, replays)) / replays for _ in range(samples))
    finally:
        del graph


def prefill_speed(runner, T: int, repeats: int = 5) -> dict:
    """Prompt tokens per second of one T-token forward (random ids), graph-captured."""
    dev = runner.embed.device
    ids = torch.randint(0, runner.embed.shape[0], (runner.batch, T), device=dev)
    positions = torch.arange(T, device=dev)
    sec = _graph_median_seconds(lambda: runner.forward(ids, positions), warm=2, samples=repeats)
    return {"T": T, "ms": sec * 1e3, "tok_s": runner.batch * T / sec}


def layers_only_ms(runner, M: int = 1) -> float:
    """Milliseconds of the swapped ops of one decode step in a graph: per layer the qkv, o,
    gate_up(+act) and down projections and the two fused add+norms; no attention, embedding or
    lm_head (reference run.py:166-201)."""
    be, eps = runner.backend, runner.eps
    dev = runner.embed.device
    hidden = runner.embed.shape[1]
    q_width = runner.n_heads * runner.head_dim
    x = torch.randn(1, M, hidden, device=dev, dtype=torch.float16)
    res0 = torch.randn_like(x)

    def layers():
        h, res = be.norm(x, runner.layers[0].ln1, eps, residual=res0)
        for L in runner.layers:
            q = be.linear(h, L.qkv)[..., :q_width].contiguous()
            h, res = be.norm(be.linear(q, L.o), L.ln2, eps, residual=res)
            h = be.linear(be.gate_up_act(h, L.gate_up), L.down)
            h, res = be.norm(h, L.ln1, eps, residual=res)

    return 1e3 * _graph_median_seconds(layers, warm=3, samples=7, replays=10)


@torch.no_grad()
def greedy_parity(runner: QwenRunner, ref: QwenRunner, ids: torch.Tensor, steps: int = 32) -> dict:
    """Greedy decode of `steps` tokens after the prompt `ids` [1, T] by `runner` and by `ref`, each on
    its own KV cache (eager forward steps), fed the same tokens until they disagree. Reports what
    the reference's parity check reports (kernels/e2e/run.py:289-303): the max |logit diff| over the
    compared positions and the index of the first greedy divergence (`steps` if none; greedy streams
    part for good after one near-tie, so where they part is the figure, not a match fraction), plus
    the reference's top-2 logit margin at that position (a divergence needs a logit error of at
    least half of it) and the largest |reference logit| (for relative tolerances)."""
    T = ids.shape[1]
    dev = ids.device

    def last_logits(r, tokens, positions):
        return r.forward(tokens, positions)[:, -1].float()

    la = last_logits(runner, ids, torch.arange(T, device=dev))
    lb = last_logits(ref, ids, torch.arange(T, device=dev))
    worst, ref_abs = 0.0, 0.0
    agreed: list[int] = []
    first, margin = steps, None
    for i in range(steps):
        worst = max(worst, (la - lb).abs().max().item())
        ref_abs = max(ref_abs, lb.abs().max().item())
        pick_a, pick_b = int(la[0].argmax()), int(lb[0].argmax())
        if pick_a != pick_b:
            top = lb[0].topk(2).values
            first, margin = i, (top[0] - top[1]).item()
            break
        agreed.append(pick_b)
        if i + 1 < steps:
            tok = torch.tensor([[pick_b]], device=dev)
            p = torch.tensor([T + i], device=dev)
            la, lb = last_logits(runner, tok, p), last_logits(ref, tok, p)
    return {"max_abs_logit_diff": worst, "max_abs_ref_logit": ref_abs, "first_divergence": first,
            "compared_tokens": steps, "ref_margin_at_divergence": margin, "tokens": agreed}
